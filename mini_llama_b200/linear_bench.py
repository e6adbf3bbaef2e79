"""Quantized-linear microbenchmark: the reference's linear shapes at every batch.

    python -m mini_llama_b200.linear_bench [--qtypes q8_0,q4_0,q4_1] [--m 1,8,64,512]

Weights W ~ N(0, 0.02) (seeded generator on the device) quantized on the
device to each block type; x ~ N(0, 1); shapes [N, K] = [896, 896],
[4864, 896], [896, 4864], [151936, 896]; M rows of x.  Each case is timed
through the public entry point (mlb_quant_linear: M <= 8 runs a GEMV, 9..64
rows the integer-MMA linear or the tcgen05 kernel, more the tcgen05 kernel,
including their x pre-passes) with CUDA events on the
library stream, after warm-up, with the L2 flushed before every launch (a
256 MB write, then a read of the same buffer, which leaves clean lines) and
all reps queued before the first is waited for (device time, not host launch
latency), and printed as one JSON line:
  gbs     algorithmic bytes (W blocks + 4 M K + 4 M N) / time, against the
          measured HBM copy bandwidth (MEASURED_PEAKS.json) -- the bound for
          M <= 8
  tflops  2 M N K / time against the measured dense bf16 GEMM throughput --
          the reference point for M >= 64 (the tensor cores run three fp16
          products per multiply-add here, for fp32-level accuracy)
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np

from . import capi
from .device import DeviceArray

SHAPES = [(896, 896), (4864, 896), (896, 4864), (151936, 896)]
QTYPES = {"q8_0": capi.Q8_0, "q4_0": capi.Q4_0, "q4_1": capi.Q4_1}
BLOCK_BYTES = {capi.Q8_0: 34, capi.Q4_0: 18, capi.Q4_1: 20}
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def time_case(lib, dev, torch, stream, qtype, n, k, m, reps=10):
    nb = (k + 31) // 32
    wbytes = n * nb * BLOCK_BYTES[qtype]
    w = lib.malloc(dev, wbytes)
    scratch = lib.malloc(dev, n * k * 4)
    lib.call("mlb_synth_normal", dev, scratch, n * k, 2, 8, 0.02)
    lib.call("mlb_quantize", dev, qtype, scratch, n, k, w)
    lib.free(dev, scratch)
    xs = lib.malloc(dev, m * k * 4)
    lib.call("mlb_synth_normal", dev, xs, m * k, 2, 9, 1.0)
    y = DeviceArray(lib, dev, (m, n))
    flush = lib.malloc(dev, 256 << 20)
    idx = lib.malloc(dev, 16)

    def run():
        lib.call("mlb_quant_linear", dev, qtype, xs, w, n * nb, m, k, n, None, y.ptr)

    for _ in range(3):
        run()
    lib.call("mlb_synchronize", dev)
    # every rep is queued behind its own L2 flush (a 256 MB write that keeps
    # the GPU busy while the host queues the rep), so the events bracket
    # device time only, not host launch latency
    events = []
    for _ in range(reps):
        # flush: a 256 MB write, then a read of it, so the L2 holds clean lines
        # of the flush buffer (no write-back of dirty lines lands in the timed
        # call)
        lib.call("mlb_memset", dev, flush, 1, 256 << 20)
        lib.call("mlb_argmax", dev, flush, (256 << 20) // 4, idx)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        run()
        e1.record(stream)
        events.append((e0, e1))
    lib.call("mlb_synchronize", dev)
    total = sum(e0.elapsed_time(e1) for e0, e1 in events) / 1e3
    for p in (w, xs, flush, idx):
        lib.free(dev, p)
    secs = total / reps
    algo = wbytes + 4 * m * k + 4 * m * n
    return secs, algo


def path_of(qtype: int, n: int, k: int, m: int, sm_count: int) -> str:
    """The kernel the library's planner picks (csrc/linear.cu LinearRows and
    PlanBlockMma, csrc/wide.cu WidePreferred), restated for labelling: from 9
    rows of x the integer-MMA linear ("int-mma") up to 32 rows, or up to 64 on
    weights of at most 8 M elements (even block count for Q8_0 / Q4_0), else
    tcgen05; below,
    the integer-MMA GEMV ("block-mma") on shapes with at least 4 row tiles of
    16 rows per SM, an even block count (Q8_0 / Q4_0) and whole rows within
    20 KB per 16 rows or a 16-byte row pitch, else the SIMT GEMV ("gemv").
    The shared-memory check of x's tables (long K at many rows, which makes
    the library run fewer rows per launch) is not restated."""
    nb = (k + 31) // 32
    if m >= 9:
        wide = m <= 64 and (m <= 32 or n * k <= (8 << 20)) and (qtype == capi.Q4_1 or nb % 2 == 0)
        return "int-mma" if wide else "tcgen05"
    rowbytes = nb * BLOCK_BYTES[qtype]
    if (n + 15) // 16 < 4 * sm_count or (qtype != capi.Q4_1 and nb % 2):
        return "gemv"
    if 16 * rowbytes > 20 * 1024 and rowbytes % 16:
        return "gemv"
    return "block-mma"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--qtypes", default="q8_0,q4_0,q4_1")
    ap.add_argument("--m", default="1,8,64,512")
    ap.add_argument("--shapes", default="all", help="'all' or e.g. 151936x896,896x896")
    ap.add_argument("--device", type=int, default=0)
    args = ap.parse_args(argv)
    import torch
    lib = capi.load()
    dev = args.device
    torch.cuda.set_device(dev)
    stream = torch.cuda.ExternalStream(lib.stream(dev), device=torch.device("cuda", dev))
    pk = peaks()
    sm_count = torch.cuda.get_device_properties(dev).multi_processor_count
    shapes = SHAPES if args.shapes == "all" else [tuple(int(v) for v in s.split("x")) for s in args.shapes.split(",")]
    for qn in args.qtypes.split(","):
        for n, k in shapes:
            for m in (int(v) for v in args.m.split(",")):
                secs, algo = time_case(lib, dev, torch, stream, QTYPES[qn], n, k, m)
                gbs = algo / secs / 1e9
                tflops = 2.0 * m * n * k / secs / 1e12
                print(json.dumps({"qtype": qn, "n": n, "k": k, "m": m, "us": round(secs * 1e6, 2),
                                  "gbs": round(gbs, 1), "hbm_frac": round(gbs / pk["hbm_gbs"], 3),
                                  "tflops": round(tflops, 2),
                                  "bf16_frac": round(tflops / pk["bf16_tflops"], 4),
                                  "path": path_of(QTYPES[qn], n, k, m, sm_count), "peaks": pk["source"]}),
                      flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
