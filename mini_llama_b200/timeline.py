"""Phase timeline of the persistent decode kernel (mlb_session_trace).

    python -m mini_llama_b200.timeline [--steps 16] [--pos 64]

Builds the Qwen2-0.5B-architecture Q8_0 model with seeded random weights,
decodes `steps` tokens from position `pos` through the persistent kernel with
the %globaltimer timeline on, and prints one JSON line of medians in
microseconds: per layer the span of each phase across the CTAs that run it
(first CTA past its wait to last CTA signalled), the gaps between phases (the
counter hand-over), the per-CTA sub-steps of each phase, the lm_head phase and
the whole step.  The first step is skipped (it pays the launch).
"""
from __future__ import annotations

import argparse
import json

import numpy as np

from . import capi
from .device import DeviceArray, Model, Session

QWEN2_Q8 = dict(vocab_size=151936, dim=896, hidden_dim=4864, n_layers=24, n_heads=14, n_kv_heads=2,
                head_dim=64, max_seq_len=256, rope_theta=1e6, rms_norm_eps=1e-6, rope_neox=1,
                qkv_bias=1, tied_embedding=1, qtype=capi.Q8_0, seed=3, prompt_seed=3)
EVENTS = 16  # stamps per (step, layer, CTA); see mlb_session_trace in include/mlb.h


def _first(a):
    a = a[a > 0]
    return int(a.min()) if a.size else 0


def _last(a):
    a = a[a > 0]
    return int(a.max()) if a.size else 0


def summarise(t: np.ndarray) -> dict:
    """t: [steps, n_layers + 1, EVENTS, ctas] stamps (ns, 0 = not stamped)."""
    steps, lp1 = t.shape[0], t.shape[1]
    L = lp1 - 1
    spans = {k: [] for k in ("qkv", "att", "ffn", "lm_head", "step")}
    gaps = {k: [] for k in ("qkv_to_att", "att_to_ffn", "ffn_to_next")}
    for st in range(1, steps):
        for l in range(L):
            e = t[st, l]
            q0, q1 = _first(e[0]), _last(e[1])
            a0, a1 = _first(e[2]), _last(e[3])
            f0, f1 = _first(e[4]), _last(e[5])
            nxt = _first(t[st, l + 1, 0])
            spans["qkv"].append(q1 - q0)
            spans["att"].append(a1 - a0)
            spans["ffn"].append(f1 - f0)
            gaps["qkv_to_att"].append(a0 - q1)
            gaps["att_to_ffn"].append(f0 - a1)
            gaps["ffn_to_next"].append(nxt - f1)
        spans["lm_head"].append(_last(t[st, L, 1]) - _first(t[st, L, 0]))
        if st + 1 < steps:
            spans["step"].append(_first(t[st + 1, 0, 0]) - _first(t[st, 0, 0]))

    def seg(a, b):
        v = []
        for st in range(1, steps):
            for l in range(L):
                x, y = t[st, l, a], t[st, l, b]
                ok = (x > 0) & (y > 0)
                v.extend((y[ok] - x[ok]).tolist())
        return round(float(np.median(v)) / 1e3, 3) if v else None

    out = {"span_us": {k: round(float(np.median(v)) / 1e3, 3) for k, v in spans.items() if v},
           "handover_us": {k: round(float(np.median(v)) / 1e3, 3) for k, v in gaps.items() if v},
           "per_cta_us": {"qkv_input": seg(0, 11), "qkv_products": seg(11, 10), "qkv_signal": seg(10, 1),
                          "att_softmax_v": seg(2, 8), "att_o_proj": seg(8, 9), "att_signal": seg(9, 3),
                          "ffn_input": seg(4, 7), "ffn_products": seg(7, 6), "ffn_signal": seg(6, 5)}}
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=16)
    ap.add_argument("--pos", type=int, default=64)
    ap.add_argument("--device", type=int, default=0)
    args = ap.parse_args(argv)
    lib = capi.load()
    dev = args.device
    m = Model(lib, dev, QWEN2_Q8)
    m.synthesize(seed=QWEN2_Q8["seed"], tied=True)
    s = Session(m)
    try:
        if s.path() != 2:
            raise RuntimeError("the persistent decode kernel is not selected for this model")
        G = lib.device_info(dev).sm_count
        L = QWEN2_Q8["n_layers"]
        n = args.steps * (L + 1) * EVENTS * G
        buf = DeviceArray(lib, dev, n, np.uint64)
        buf.upload(np.zeros(n, np.uint64))
        toks = DeviceArray(lib, dev, args.steps + 1, np.int32)
        first = np.zeros(args.steps + 1, np.int32)
        first[0] = 1234
        toks.upload(first)
        s.decode_device(toks.ptr, args.pos, args.steps)  # warm-up
        lib.sync(dev)
        lib.call("mlb_session_trace", s.handle, buf.ptr, n)
        s.decode_device(toks.ptr, args.pos, args.steps)
        lib.sync(dev)
        lib.call("mlb_session_trace", s.handle, None, 0)
        t = buf.download().reshape(args.steps, L + 1, EVENTS, G).astype(np.int64)
        print(json.dumps(summarise(t)))
    finally:
        s.close()
        m.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
