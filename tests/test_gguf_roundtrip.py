"""GGUF fixture round trip: a random model written as a GGUF v3 file
(tests/gguf_writer.py) and read by the reference's unchanged loader
(LoadGgufModel, src/gguf_loader.cpp:327-399: tensor-name map, MapShape's
reversed 2-D shapes, NeoX RoPE from general.architecture == "qwen2", a tied
lm_head as F32 when output.weight is absent), then decoded by the reference
CPU path and, on a GPU, by the same reference forward pass on this library.

CPU tests: the writer's blocks decode (oracle dequantizers) to the weights
they encode, and the reference CPU harness loads both files with the expected
configuration.  GPU tests: forward_on_b200 --gguf decodes the file on the
reference CPU path and on this library; greedy ids equal, logits within 1e-3
of the largest logit.
"""
import json
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT
from oracle.binding import Q40, Q41, Q80, Oracle
from tests.gguf_writer import GGML_Q4_0, GGML_Q4_1, GGML_Q8_0, quantize, random_model

REF = os.path.join(ROOT, "oracle", "_ref")

MODELS = {
    # Qwen2 layout: NeoX RoPE, q/k/v biases, GQA 4:2, tied (F32) lm_head, Q8_0 linears
    "qwen2_q8_0_tied": dict(arch="qwen2", dim=256, hidden=704, layers=2, heads=4, kv_heads=2, vocab=1000,
                            ctx=64, theta=1e6, eps=1e-6, types={"attn": GGML_Q8_0, "ffn": GGML_Q8_0},
                            seed=7, biases=True, tied=True, sigma=0.05),
    # Llama layout: normal RoPE, Q4_0 attention, Q4_1 FFN, Q8_0 embedding
    # (dequantized at load) and Q8_0 output.weight
    "llama_q4_mixed": dict(arch="llama", dim=256, hidden=512, layers=2, heads=4, kv_heads=4, vocab=512,
                           ctx=64, theta=1e4, eps=1e-5,
                           types={"attn": GGML_Q4_0, "ffn": GGML_Q4_1, "embd": GGML_Q8_0, "output": GGML_Q8_0},
                           seed=8, tied=False, sigma=0.05),
}
PROMPT, NEW, SEED = 12, 12, 5


def write(tmp_path, name):
    spec = dict(MODELS[name])
    path = str(tmp_path / f"{name}.gguf")
    random_model(path, spec.pop("arch"), **spec)
    return path


def run(exe, args, timeout=300):
    path = os.path.join(REF, exe)
    if not os.path.exists(path):
        pytest.fail(f"{path} missing: build with make -C oracle ref ref-b200 (needs the reference tree)")
    r = subprocess.run([path] + args, capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("ggml,qt,tol", [(GGML_Q8_0, Q80, 1 / 254), (GGML_Q4_0, Q40, 1 / 14), (GGML_Q4_1, Q41, 1 / 30)])
def test_writer_blocks_decode_to_their_weights(ggml, qt, tol):
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((8, 96)) * 0.05).astype(np.float32)
    w[0, :32] = 0.0  # an all-zero block (scale 0)
    blocks = np.frombuffer(quantize(w, ggml), dtype=np.uint8)
    back = Oracle().dequantize(qt, blocks, 8, 96)
    span = np.abs(w).reshape(-1, 32).max(axis=1).repeat(32).reshape(w.shape)
    if qt == Q41:
        b = w.reshape(-1, 32)
        span = (b.max(axis=1) - b.min(axis=1)).repeat(32).reshape(w.shape)
    assert np.all(np.abs(back - w) <= tol * span + 1e-3 * span + 1e-12)
    assert np.all(back[0, :32] == 0.0)


@pytest.mark.parametrize("name", sorted(MODELS))
def test_reference_loader_reads_the_file(tmp_path, name):
    spec = MODELS[name]
    out = run("ref_harness", ["gguf", write(tmp_path, name), str(PROMPT), str(NEW), str(SEED)])
    assert out["neox"] == (spec["arch"] == "qwen2")
    assert out["vocab"] == spec["vocab"] and out["dim"] == spec["dim"]
    assert out["head_dim"] == spec["dim"] // spec["heads"]
    assert out["lm_head_f32"] == int(spec["tied"])
    assert len(out["tokens"]) == NEW and len(set(out["tokens"])) > 3  # not a degenerate repeat
    again = run("ref_harness", ["gguf", write(tmp_path, name), str(PROMPT), str(NEW), str(SEED)])
    assert again["tokens"] == out["tokens"]


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(MODELS))
def test_gguf_model_decodes_on_this_library_as_on_the_reference_cpu(tmp_path, name):
    out = run("forward_on_b200", ["--gguf", write(tmp_path, name), str(PROMPT), str(NEW), str(SEED)])
    scale = max(1.0, out["logit_scale"])
    assert out["linear_calls"] > 0, "the device path did not run"
    assert out["logit_err"] <= 1e-3 * scale, out
    # the reference's top-2 margin exceeds twice the difference, so no arg-max can flip
    assert out["cpu_min_gap"] > 2 * out["logit_err"], f"near-tie in the reference logits: {out}"
    assert out["b200"] == out["cpu"], out
