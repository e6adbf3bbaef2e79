"""Decode-attention microbenchmark: the GQA sweep over an fp32 KV cache.

    python -m mini_llama_b200.attention_bench [--heads 14x2x64,32x8x128]
        [--ctx 128,1024,8192,32768] [--batch 1,32]

Head configurations (query heads x KV heads x head_dim) 14 x 2 x 64 and
32 x 8 x 128; P = 128, 1024, 8192 and 32768 cached positions (the call attends
over positions 0 .. P - 1, so pos = P - 1); batches of 1 and 32 independent
sequences.  Q, K, V ~ N(0, 1) from the seeded device generator (seed 4).  The
cache is the reference layout [batch][n_layers = 1][P][n_kv][head_dim] fp32.
Batch 1 runs mlb_attention_decode, batch 32 mlb_attention_decode_batched
(every sequence at the same position), each timed with CUDA events on the
library stream after warm-up, the L2 flushed (a 256 MB write, then a read of
it, leaving clean lines) before every
launch and all reps queued before the first is waited for, and printed as one
JSON line per case:
  bytes   algorithmic bytes: K and V rows read (2 x P x n_kv x head_dim x 4
          per sequence) + q read + out written
  gbs     bytes / time, against the measured HBM copy bandwidth
          (MEASURED_PEAKS.json): the bound once the cache is larger than a
          few MB; the short contexts are launch-latency bound
"""
from __future__ import annotations

import argparse
import json

import numpy as np

from . import capi
from .linear_bench import peaks

HEADS = [(14, 2, 64), (32, 8, 128)]
CONTEXTS = [128, 1024, 8192, 32768]
BATCHES = [1, 32]


def time_case(lib, dev, torch, stream, nh, nkv, hd, ctx, batch, reps=10):
    cache_floats = batch * ctx * nkv * hd
    kc = lib.malloc(dev, cache_floats * 4)
    vc = lib.malloc(dev, cache_floats * 4)
    q = lib.malloc(dev, batch * nh * hd * 4)
    out = lib.malloc(dev, batch * nh * hd * 4)
    lib.call("mlb_synth_normal", dev, kc, cache_floats, 4, 1, 1.0)
    lib.call("mlb_synth_normal", dev, vc, cache_floats, 4, 2, 1.0)
    lib.call("mlb_synth_normal", dev, q, batch * nh * hd, 4, 3, 1.0)
    pos = ctx - 1
    positions = None
    if batch > 1:
        positions = lib.malloc(dev, batch * 4)
        host = np.full(batch, pos, dtype=np.int32)
        lib.call("mlb_memcpy_h2d", dev, positions, host.ctypes.data, host.nbytes)
    flush = lib.malloc(dev, 256 << 20)
    idx = lib.malloc(dev, 16)

    def run():
        if batch == 1:
            lib.call("mlb_attention_decode", dev, q, kc, vc, 1, ctx, 0, pos, nh, nkv, hd, out)
        else:
            lib.call("mlb_attention_decode_batched", dev, batch, q, kc, vc, 1, ctx, 0, positions,
                     pos, nh, nkv, hd, out)

    for _ in range(3):
        run()
    lib.call("mlb_synchronize", dev)
    events = []
    for _ in range(reps):
        # flush: a 256 MB write, then a read of it (the L2 keeps clean lines)
        lib.call("mlb_memset", dev, flush, 1, 256 << 20)
        lib.call("mlb_argmax", dev, flush, (256 << 20) // 4, idx)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        run()
        e1.record(stream)
        events.append((e0, e1))
    lib.call("mlb_synchronize", dev)
    secs = sum(e0.elapsed_time(e1) for e0, e1 in events) / 1e3 / reps
    for p in (kc, vc, q, out, flush, idx) + ((positions,) if positions else ()):
        lib.free(dev, p)
    algo = batch * (2 * ctx * nkv * hd * 4 + 2 * nh * hd * 4)
    return secs, algo


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--heads", default=",".join(f"{a}x{b}x{c}" for a, b, c in HEADS))
    ap.add_argument("--ctx", default=",".join(str(c) for c in CONTEXTS))
    ap.add_argument("--batch", default=",".join(str(b) for b in BATCHES))
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--device", type=int, default=0)
    args = ap.parse_args(argv)
    import torch
    lib = capi.load()
    dev = args.device
    torch.cuda.set_device(dev)
    stream = torch.cuda.ExternalStream(lib.stream(dev), device=torch.device("cuda", dev))
    pk = peaks()
    heads = [tuple(int(v) for v in s.split("x")) for s in args.heads.split(",")]
    for nh, nkv, hd in heads:
        for batch in (int(v) for v in args.batch.split(",")):
            for ctx in (int(v) for v in args.ctx.split(",")):
                secs, algo = time_case(lib, dev, torch, stream, nh, nkv, hd, ctx, batch, args.reps)
                gbs = algo / secs / 1e9
                print(json.dumps({"heads": f"{nh}/{nkv}x{hd}", "ctx": ctx, "batch": batch,
                                  "us": round(secs * 1e6, 2), "bytes": algo, "gbs": round(gbs, 1),
                                  "hbm_frac": round(gbs / pk["hbm_gbs"], 3),
                                  "peaks": pk["source"]}), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
