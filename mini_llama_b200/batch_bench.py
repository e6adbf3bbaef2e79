"""Batched (and tensor-parallel) greedy decoding throughput.

    python -m mini_llama_b200.batch_bench [--model llama7b] [--batch 64] [--prompt 512] [--new 256]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m mini_llama_b200.batch_bench ...                      # N-way tensor parallel

Workload (default): the Llama-2-7B architecture (32 layers, dim 4096, 32
heads, 32 KV heads, head_dim 128, SwiGLU 11008, vocab 32000), weights
N(0, 0.02) seeded and quantized to Q4_0 on the device; `batch` independent
sequences of `prompt` uniform token ids (seeded), greedy continuation by
`new` tokens.  With N processes every linear's rows and the KV heads are
split N ways (mlb_batch with tp_size N; NCCL all-gathers inside each captured
step).  Prompt steps and decode steps are timed separately with CUDA events
on the library stream, the maximum over ranks taken; rank 0 prints one JSON
line: decode tokens/s = batch x (new - 1) / decode time, prefill tokens/s =
batch x prompt / prefill time.
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np

from . import capi
from .device import BatchSession, Model, nccl_unique_id
from .tp import max_over_ranks, share_nccl_id

MODELS = {
    "llama7b": dict(vocab_size=32000, dim=4096, hidden_dim=11008, n_layers=32, n_heads=32, n_kv_heads=32,
                    head_dim=128, rope_theta=1e4, rms_norm_eps=1e-5, rope_neox=0, qkv_bias=0,
                    tied_embedding=0, qtype=capi.Q4_0, seed=5),
    "qwen2": dict(vocab_size=151936, dim=896, hidden_dim=4864, n_layers=24, n_heads=14, n_kv_heads=2,
                  head_dim=64, rope_theta=1e6, rms_norm_eps=1e-6, rope_neox=1, qkv_bias=1,
                  tied_embedding=1, qtype=capi.Q8_0, seed=3),
}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama7b", choices=sorted(MODELS))
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--new", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=1)
    args = ap.parse_args(argv)
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dev = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        dist.init_process_group("gloo")
    lib = capi.load()
    torch.cuda.set_device(dev)
    spec = dict(MODELS[args.model], max_seq_len=args.prompt + args.new)
    m = Model(lib, dev, spec)
    b = None
    try:
        m.synthesize(seed=spec["seed"], tied=bool(spec["tied_embedding"]))
        nid = share_nccl_id(dist, lambda: nccl_unique_id(lib)) if world > 1 else None
        b = BatchSession(m, args.batch, rank, world, nid)
        rng = np.random.default_rng(spec["seed"] + 1)
        prompts = rng.integers(0, spec["vocab_size"], size=(args.batch, args.prompt), dtype=np.int32)
        for _ in range(args.warmup):
            b.generate(prompts[:, :8], 4)
        toks, pre_ms, dec_ms = b.generate(prompts, args.new)
        if world > 1:
            pre_ms, dec_ms = max_over_ranks(dist, [pre_ms, dec_ms])
            dist.barrier()
        if rank == 0:
            dec_tok = args.batch * (args.new - 1)
            print(json.dumps({
                "metric": "batched greedy decode tok/s", "value": round(dec_tok / (dec_ms / 1e3), 1),
                "unit": "tok/s", "prefill_tok_s": round(args.batch * args.prompt / (pre_ms / 1e3), 1),
                "decode_ms": round(dec_ms, 2), "prefill_ms": round(pre_ms, 2),
                "ms_per_decode_step": round(dec_ms / max(1, args.new - 1), 3),
                "n_gpus": world, "parallelism": f"tp{world}", "dtype": "q4_0" if spec["qtype"] == capi.Q4_0 else "q8_0",
                "data": "synthetic (seeded N(0, 0.02) weights, uniform prompt ids)",
                "config": {"model": args.model, "batch": args.batch, "prompt": args.prompt, "new": args.new},
                "first_tokens": toks[0, :8].tolist()}), flush=True)
    finally:
        if b is not None:
            b.close()
        m.close()
        if world > 1:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
