"""Decode benchmark: Qwen2-0.5B architecture, Q8_0 weights, batch 1, greedy.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

A step decodes 128 tokens (positions 64..191 after a 64-token prompt) through
the device session: one launch of the persistent decode kernel per step (every
layer of every token in one cooperative kernel, tokens fed back on the
device); --graph selects the CUDA graph per token instead.
  value  tokens/s with everything resident in HBM (CUDA events on the library
         stream, max over ranks); weights (528 MB/token) exceed the 126 MB L2,
         so no flush is needed between steps
  e2e    the same through mlb_session_generate with host buffers: the step's
         start token copied host->device and the 128 generated ids copied back
  roofline  the dominant kernel: the persistent decode kernel, algorithmic
         bytes of its 128 tokens / its CUDA-event time per launch vs measured
         HBM (graph path: the Q8_0 GEMV timed alone on the lm_head shape)
  cpu_baseline  the reference CPU implementation (its RunBenchmark decode loop,
         built from the reference sources into oracle/_ref) on a bounded
         sample of the same workload: the 64-token prompt prefilled once,
         untimed, then steps of 4 greedy tokens continuing from position 64
  prefill  the 64-token prompt pass alone (mlb_session_generate with one new
         token): prompt tokens/s
  dropin the reference's own, unchanged forward.cpp device path linked
         against this library (oracle/_ref/forward_on_b200): decode tokens/s
         of 128 greedy tokens after the same prompt
  tp_batch  batched greedy decoding of the Llama-2-7B architecture (Q4_0)
         for 64 sequences, 128 prompt ids + 64 tokens, through mlb_batch_*,
         tensor parallel over all N GPUs (NCCL inside the library): decode
         tokens/s of the whole job, max over ranks (strong scaling in N)
With N > 1 (torchrun) every GPU decodes its own sequence (replicas; weak scaling).
--impl reference times the reference CPU implementation alone, on the same
config, one line from rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (Qwen2-0.5B-arch Q8_0, bs1)"
UNIT = "tokens/s"
PROMPT = 64
NEW = 128  # decode tokens per step (bench --decode-tokens may lower it for profiling)
QWEN2 = dict(vocab_size=151936, dim=896, hidden_dim=4864, n_layers=24, n_heads=14, n_kv_heads=2,
             head_dim=64, max_seq_len=256, rope_theta=1e6, rms_norm_eps=1e-6, rope_neox=1,
             qkv_bias=1, tied_embedding=1, qtype=1, seed=3, prompt_seed=3)


def algorithmic_bytes_per_token(pos: int) -> int:
    """Weight bytes + fp32 norms/biases/embedding row + KV read/write at position pos."""
    D, F, V, L = 896, 4864, 151936, 24
    qd, kd = 14 * 64, 2 * 64
    blk = lambda r, c: r * ((c + 31) // 32) * 34  # noqa: E731
    layer = blk(qd, D) + 2 * blk(kd, D) + blk(D, qd) + 2 * blk(F, D) + blk(D, F)
    small = L * (2 * D + qd + 2 * kd) * 4 + D * 4 + D * 4  # norms, biases, final norm, embedding row
    kv = L * (pos + 1) * 2 * kd * 4 + L * 2 * kd * 4       # read 0..pos, write pos
    return L * layer + blk(V, D) + small + kv


CONFIG = {"workload": "Qwen2-0.5B-arch Q8_0 random-init, batch 1, prompt 64 + 128 greedy decode",
          "model": "qwen2-0.5b-arch", "weights": "Q8_0 (lm_head tied, Q8_0)", "global_batch": 1,
          "seq_len": PROMPT + NEW, "decode_tokens_per_step": NEW,
          "l2": "inputs larger than L2 (528 MB of weights streamed per token)"}
REF_TOKENS = 4  # reference decode tokens per timed step (a bounded sample of the 128)


def ref_tokens_per_step(steps: int, warmup: int) -> int:
    """Tokens per reference step: REF_TOKENS while the whole run stays inside
    the workload's positions 64..191, fewer for long runs."""
    return max(1, min(REF_TOKENS, NEW // max(1, steps + warmup)))


def config_for(world: int) -> dict:
    """The workload both arms report: one independent sequence per GPU."""
    return dict(CONFIG, global_batch=world,
                parallelism=f"replicas x{world}" if world > 1 else "single GPU")


class Clocks:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def committed_traffic(name: str):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f).get(name)
    return None


def reference_sample(threads: int, steps: int, warmup: int):
    """The reference's decode loop on the same seeded model: prompt prefilled
    once (untimed), then `steps` timed steps of REF_TOKENS greedy tokens
    continuing the sequence from position PROMPT (oracle/_ref/ref_harness
    decode).  Returns (tokens/s over the timed steps, their records)."""
    from oracle.binding import run_ref_decode
    recs = run_ref_decode("qwen2", threads, PROMPT, ref_tokens_per_step(steps, warmup), steps, warmup)
    timed = [r for r in recs if r.get("event") == "step" and r.get("timed")]
    if not timed:
        return None, timed
    toks = sum(r["decode_tokens"] for r in timed)
    ms = sum(r["decode_ms"] for r in timed)
    return toks * 1000.0 / ms, timed


def reference_sample_text(threads: int, steps: int, timed) -> str:
    n = timed[0]["decode_tokens"] if timed else 0
    first = timed[0]["first_pos"] if timed else PROMPT
    last = timed[-1]["first_pos"] + n - 1 if timed else PROMPT
    return (f"reference RunBenchmark decode loop (src/debug.cpp:112-127) on the same seeded model, "
            f"{threads} threads: 64-token prompt prefilled once (untimed), {steps} timed steps of "
            f"{n} greedy tokens at positions {first}..{last}")


def max_over_ranks(dist, value: float, device: str) -> float:
    """The largest value over all ranks (every rank calls it, in the same
    order); the value itself with a single process (dist None)."""
    if dist is None:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_throughput(world: int, tokens_per_rank_step: int, steps: int, secs: float) -> float:
    """Whole-job tokens/s: every rank decodes its own sequence (replicas), the
    job takes the slowest rank's time."""
    return world * tokens_per_rank_step * steps / secs


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    try:
        value, timed = reference_sample(threads, args.steps, args.warmup)
    except Exception as e:  # the harness is built here from the reference tree
        print(json.dumps({"impl": "reference", "unavailable": f"reference harness failed: {e}"}))
        return 0
    ms = statistics.mean(r["decode_ms"] for r in timed) if timed else None
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights and prompt ids)", "impl": "reference",
            "config": config_for(world),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                             "sample": reference_sample_text(threads, args.steps, timed)},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def dropin_numbers(timeout: float = 900.0):
    """The reference's unchanged forward.cpp device path on this library
    (ForwardBatch over the prompt, then 128 single-token steps with the
    reference's host arg-max): prompt and decode tokens/s."""
    exe = os.path.join(ROOT, "oracle", "_ref", "forward_on_b200")
    if not os.path.exists(exe):
        return {"value": None, "unit": UNIT, "unavailable": "oracle/_ref/forward_on_b200 not built"}
    out = subprocess.run([exe, "qwen2", str(PROMPT), str(NEW + 1)], capture_output=True, text=True,
                         timeout=timeout)
    if out.returncode != 0:
        return {"value": None, "unit": UNIT, "unavailable": out.stderr.strip()[-200:]}
    r = json.loads(out.stdout.strip().splitlines()[-1])
    return {"value": r["decode_tokens"] * 1000.0 / r["decode_ms"], "unit": UNIT,
            "prefill_tok_s": PROMPT * 1000.0 / r["prefill_ms"], "decode_tokens": r["decode_tokens"],
            "path": "reference src/forward.cpp ForwardBatch + GetArgMax over the include/cuda_*.h adapter "
                    "(one library call per op, logits copied to the host every token)"}


def gemv_roofline(lib, dev, torch, stream):
    """Times the decode's GEMV kernel (integer-MMA over R16 weights, M = 1) alone
    on the lm_head shape [151936, 896] with CUDA events, L2 flushed between
    launches."""
    import numpy as np

    from mini_llama_b200.device import DeviceArray
    N, K = 151936, 896
    nb = K // 32
    wbytes = N * nb * 34
    w = lib.malloc(dev, wbytes)
    r16 = lib.malloc(dev, lib.dll.mlb_r16_bytes(N, K))
    scratch = lib.malloc(dev, N * K * 4)
    lib.call("mlb_synth_normal", dev, scratch, N * K, 2, 8, 0.02)
    lib.call("mlb_quantize", dev, 1, scratch, N, K, w)
    lib.call("mlb_q80_repack_r16", dev, w, N, K, r16)
    x = DeviceArray.from_host(lib, dev, np.ones(K, np.float32))
    y = DeviceArray(lib, dev, N)
    flush = lib.malloc(dev, 256 << 20)  # > L2: each launch reads the weights from HBM
    for _ in range(3):
        lib.call("mlb_q80_linear_r16", dev, x.ptr, r16, 1, K, N, None, y.ptr)
    reps, total = 20, 0.0
    for _ in range(reps):
        lib.call("mlb_memset", dev, flush, 1, 256 << 20)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        lib.call("mlb_q80_linear_r16", dev, x.ptr, r16, 1, K, N, None, y.ptr)
        e1.record(stream)
        e1.synchronize()
        total += e0.elapsed_time(e1) / 1e3
    lib.sync(dev)
    for p in (w, r16, scratch, flush):
        lib.free(dev, p)
    per_launch = total / reps
    algo = wbytes + K * 4 + N * 4
    return algo, per_launch


TP_BATCH, TP_PROMPT, TP_NEW = 64, 128, 64


def tp_batch_leg(lib, dev, dist, world: int, rank: int):
    """Batched greedy decoding of the Llama-2-7B architecture (Q4_0, seeded
    random-init weights) for TP_BATCH sequences of TP_PROMPT uniform prompt ids
    plus TP_NEW tokens through mlb_batch_*, tensor parallel over all ranks
    (every linear's rows and the KV heads split world ways, NCCL all-gathers
    inside the library's captured step; tp_size 1 on one GPU).  Device times
    from CUDA events on the library stream, maximum over ranks."""
    import numpy as np

    from mini_llama_b200.batch_bench import MODELS
    from mini_llama_b200.device import BatchSession, Model, nccl_unique_id
    from mini_llama_b200.tp import share_nccl_id

    spec = dict(MODELS["llama7b"], max_seq_len=TP_PROMPT + TP_NEW)
    m = Model(lib, dev, spec)
    b = None
    try:
        m.synthesize(seed=spec["seed"], tied=False)
        nid = share_nccl_id(dist, lambda: nccl_unique_id(lib)) if world > 1 else None
        b = BatchSession(m, TP_BATCH, rank, world, nid)
        rng = np.random.default_rng(spec["seed"] + 1)
        prompts = rng.integers(0, spec["vocab_size"], size=(TP_BATCH, TP_PROMPT), dtype=np.int32)
        b.generate(prompts[:, :8], 4)  # warm-up: captures the step graphs
        toks, pre_ms, dec_ms = b.generate(prompts, TP_NEW)
        if dist is not None:
            pre_ms = max_over_ranks(dist, pre_ms, f"cuda:{dev}")
            dec_ms = max_over_ranks(dist, dec_ms, f"cuda:{dev}")
        dec_tok = TP_BATCH * (TP_NEW - 1)
        return {"workload": f"Llama-2-7B-arch Q4_0 random-init, {TP_BATCH} sequences, prompt {TP_PROMPT} + "
                            f"{TP_NEW} greedy tokens",
                "path": "mlb_batch_create / mlb_batch_generate",
                "parallelism": f"tp{world}", "n_gpus": world,
                "decode_tok_s": dec_tok / (dec_ms / 1e3), "unit": "tokens/s",
                "ms_per_decode_step": dec_ms / (TP_NEW - 1),
                "prefill_tok_s": TP_BATCH * TP_PROMPT / (pre_ms / 1e3),
                "first_tokens": toks[0, :8].tolist()}
    finally:
        if b is not None:
            b.close()
        m.close()


def run_ours(args):
    import numpy as np
    import torch

    from mini_llama_b200 import capi
    from mini_llama_b200 import synth
    from mini_llama_b200.device import DeviceArray, Model, Session

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    lib = capi.load()
    dev = local
    stream = torch.cuda.ExternalStream(lib.stream(dev), device=torch.device("cuda", dev))
    if args.roofline_only:
        algo, launch_s = gemv_roofline(lib, dev, torch, stream)
        print(json.dumps({"kernel": "QmmaGemvKernel<M=1> (Q8_0, R16) on [151936, 896]", "bytes": algo,
                          "launch_us": launch_s * 1e6, "gbs": algo / launch_s / 1e9}))
        return 0

    model = Model(lib, dev, QWEN2)
    model.synthesize(seed=QWEN2["seed"], tied=True)
    sess = Session(model)
    if args.graph:
        sess.use_persistent(False)
    path = sess.path()
    prompt = synth.tokens(PROMPT, QWEN2["prompt_seed"], QWEN2["vocab_size"])
    if args.no_prefill:  # profiling runs: decode from position 64 over an empty cache
        first = np.array([int(prompt[-1])], np.int32)
    else:
        first = sess.generate(prompt, 1)  # prefill, first greedy token at position 64
    toks = DeviceArray(lib, dev, NEW + 1, np.int32)
    init = np.zeros(NEW + 1, np.int32)
    init[0] = first[0]
    toks.upload(init)

    new = args.decode_tokens

    def step():
        sess.decode_device(toks.ptr, PROMPT, new)

    def barrier():
        torch.cuda.synchronize(dev)
        lib.sync(dev)
        if dist is not None:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    barrier()
    clocks = Clocks(dev)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    e1.synchronize()
    barrier()
    clk = clocks.stop()
    secs = max_over_ranks(dist, e0.elapsed_time(e1) / 1e3, f"cuda:{dev}")
    value = job_throughput(world, new, args.steps, secs)

    # e2e: host start token in, host token ids out, through mlb_session_generate
    start = torch.empty(1, dtype=torch.int32, pin_memory=True)
    out = torch.empty(NEW, dtype=torch.int32, pin_memory=True)
    start[0] = int(first[0])

    def e2e_step():
        lib.call("mlb_session_generate", sess.handle, start.data_ptr(), 1, PROMPT, NEW,
                 out.data_ptr())

    e2e = None
    if not args.no_e2e:
        for _ in range(max(1, args.warmup)):
            e2e_step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        barrier()
        e2e_secs = max_over_ranks(dist, time.perf_counter() - t0, f"cuda:{dev}")
        e2e = job_throughput(world, NEW, args.steps, e2e_secs)

    peaks = measured_peaks()
    step_bytes = sum(algorithmic_bytes_per_token(p) for p in range(PROMPT, PROMPT + new))
    step_gbs = step_bytes * args.steps / secs / 1e9 if world == 1 else None
    launches_per_token = 1 + 5 * QWEN2["n_layers"] + 1
    if path == 2:
        # one kernel per step; its launch time is the step time less the
        # few-microsecond state copies around it
        roof = {"bound": "hbm", "kernel": f"MegaDecodeKernel (persistent, {new} tokens per launch)",
                "achieved": step_bytes * args.steps / secs / 1e9, "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "peak_source": peaks["source"], "bytes_per_launch": step_bytes,
                "launch_us": secs / args.steps * 1e6, "traffic": committed_traffic("mega_decode")}
        gpu_launches = args.steps
    else:
        algo, launch_s = gemv_roofline(lib, dev, torch, stream)
        roof = {"bound": "hbm", "kernel": "QmmaGemvKernel<M=1> (Q8_0, R16) on [151936, 896]",
                "achieved": algo / launch_s / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "peak_source": peaks["source"], "bytes_per_launch": algo,
                "launch_us": launch_s * 1e6, "traffic": committed_traffic("qmma_lm_head")}
        gpu_launches = launches_per_token * new * args.steps
    roof["frac"] = roof["achieved"] / roof["peak"]

    # the prompt pass alone: 64 prompt tokens through every layer at once and
    # the first greedy token, host prompt in, host token out
    prefill = None
    if not args.no_prefill:
        pbuf = torch.from_numpy(np.ascontiguousarray(prompt, np.int32)).pin_memory()
        one = torch.empty(1, dtype=torch.int32, pin_memory=True)
        for _ in range(2):
            lib.call("mlb_session_generate", sess.handle, pbuf.data_ptr(), PROMPT, 0, 1, one.data_ptr())
        barrier()
        reps = 10
        t0 = time.perf_counter()
        for _ in range(reps):
            lib.call("mlb_session_generate", sess.handle, pbuf.data_ptr(), PROMPT, 0, 1, one.data_ptr())
        barrier()
        psecs = max_over_ranks(dist, (time.perf_counter() - t0) / reps, f"cuda:{dev}")
        prefill = {"value": world * PROMPT / psecs, "unit": "prompt tokens/s", "ms": psecs * 1e3,
                   "path": "mlb_session_generate(64-token host prompt -> 1 host token): tensor-core "
                           "prompt pass + first arg-max"}

    sess.close()
    model.close()
    tp = None
    if not args.no_tp:
        tp = tp_batch_leg(lib, dev, dist, world, rank)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        try:
            v, timed = reference_sample(threads, 3, 1)
            cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "reference",
                   "sample": reference_sample_text(threads, 3, timed)}
        except Exception as e:
            cpu = {"value": None, "unit": UNIT, "cores": threads, "kind": "reference",
                   "sample": f"unavailable: {e}"}
    dropin = None
    if world == 1 and not args.no_dropin:
        try:
            dropin = dropin_numbers()
        except Exception as e:
            dropin = {"value": None, "unit": UNIT, "unavailable": str(e)}
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 activations, Q8_0 weights",
        "data": "synthetic (seeded random-init weights and prompt ids)",
        "config": config_for(world),
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": 4 + 8 + 4,
                "d2h_bytes_per_step": NEW * 4 + 4,
                "path": "mlb_session_generate(host start token -> host 128 token ids)"},
        "decode_path": {2: "persistent kernel", 1: "graph, integer-MMA GEMV",
                        0: "graph, SIMT GEMV"}[path],
        "roofline": roof,
        "step_roofline": {"bytes_per_token_avg": step_bytes / new,
                          "achieved_gbs": step_gbs,
                          "frac": (step_gbs / peaks["hbm_gbs"]) if step_gbs else None},
        "cpu_baseline": cpu,
        "prefill": prefill,
        "dropin": dropin,
        "tp_batch": tp,
        "clocks": clk,
        "gpu_launches": gpu_launches,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-dropin", action="store_true",
                    help="skip the reference forward.cpp on this library (builds the model on the CPU)")
    ap.add_argument("--no-tp", action="store_true",
                    help="skip the tensor-parallel batched Llama-2-7B leg")
    ap.add_argument("--no-prefill", action="store_true",
                    help="profiling: skip the 64-token prefill (KV cache left empty)")
    ap.add_argument("--graph", action="store_true",
                    help="decode through the CUDA graph per token instead of the persistent kernel")
    ap.add_argument("--roofline-only", action="store_true",
                    help="time only the Q8_0 GEMV on the lm_head shape")
    ap.add_argument("--decode-tokens", type=int, default=NEW,
                    help="tokens per step (128 for the headline; fewer for profiling runs)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
