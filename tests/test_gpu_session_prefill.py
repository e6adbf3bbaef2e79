"""The one-pass prompt path of mlb_session_generate (every layer on all prompt
tokens at once; tensor-core linears from 9 tokens) against the reference CPU
path and against the same session's token-by-token prompt path: greedy tokens
equal, the last prompt position's logits within 1e-3 relative (the usual
logits bound), the KV cache it writes within 1e-4 relative."""
import ctypes

import numpy as np
import pytest

from mini_llama_b200.device import Model, Session
from oracle.binding import MODEL_SPECS
from tests.test_gpu_model import assert_logits, oracle_loaded

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def qwen2(mlb, gpu):
    m = Model(mlb, gpu, MODEL_SPECS["qwen2"])
    m.synthesize(seed=MODEL_SPECS["qwen2"]["seed"], tied=True)
    yield m
    m.close()


def last_logits(mlb, gpu, s, vocab):
    out = np.empty(vocab, np.float32)
    mlb.call("mlb_memcpy_d2h", gpu, out.ctypes.data, s.logits_ptr(), out.nbytes)
    return out


def kv_rows(mlb, gpu, s, spec, n_pos):
    kc, vc = ctypes.c_void_p(), ctypes.c_void_p()
    mlb.call("mlb_session_kv_cache", s.handle, ctypes.byref(kc), ctypes.byref(vc))
    kd = spec["n_kv_heads"] * spec["head_dim"]
    total = spec["n_layers"] * spec["max_seq_len"] * kd
    out = []
    for ptr in (kc.value, vc.value):
        a = np.empty(total, np.float32)
        mlb.call("mlb_memcpy_d2h", gpu, a.ctypes.data, ptr, a.nbytes)
        out.append(a.reshape(spec["n_layers"], spec["max_seq_len"], kd)[:, :n_pos])
    return out


@pytest.mark.parametrize("persistent", [True, False], ids=["persistent", "graph"])
def test_qwen2_prompt_pass_matches_token_path(mlb, gpu, qwen2, golden_qwen2, persistent):
    spec = MODEL_SPECS["qwen2"]
    prompt = golden_qwen2["model_qwen2_prompt"]  # 64 tokens
    gen = golden_qwen2["model_qwen2_generated"][:24]
    s = Session(qwen2)
    try:
        s.use_persistent(persistent)
        s.prefill_min(16)
        got = s.generate(prompt, len(gen))
        assert np.array_equal(got, gen), f"first mismatch at {np.flatnonzero(got != gen)[:3]}"
        # the last prompt position through the prompt pass (generate of one token)
        s.reset()
        s.generate(prompt, 1)
        fast = last_logits(mlb, gpu, s, spec["vocab_size"])
        kf, vf = kv_rows(mlb, gpu, s, spec, len(prompt))
        s.reset()
        s.prefill_min(0)
        s.generate(prompt, 1)
        kt, vt = kv_rows(mlb, gpu, s, spec, len(prompt))
    finally:
        s.close()
    assert_logits(fast, golden_qwen2["model_qwen2_logits"], "prompt pass, last prompt position")
    for a, b, what in ((kf, kt, "keys"), (vf, vt, "values")):
        scale = max(1.0, float(np.abs(b).max()))
        err = float(np.abs(a.astype(np.float64) - b).max())
        assert err <= 1e-4 * scale, f"{what}: {err:.3e} (scale {scale:.2f})"


def test_qwen2_prompt_pass_from_a_later_position(mlb, gpu, qwen2):
    """A prompt continuing a cache that already holds 10 positions."""
    rng = np.random.default_rng(11)
    head = rng.integers(0, MODEL_SPECS["qwen2"]["vocab_size"], 10, dtype=np.int32)
    more = rng.integers(0, MODEL_SPECS["qwen2"]["vocab_size"], 40, dtype=np.int32)
    outs = []
    for pmin in (16, 0):
        s = Session(qwen2)
        try:
            s.prefill_min(pmin)
            s.generate(head, 1)  # positions 0..9 (token path: fewer than 16)
            outs.append(s.generate(more, 12, start_pos=10))
        finally:
            s.close()
    assert np.array_equal(outs[0], outs[1])


def test_tiny_prompt_pass_matches_oracle(mlb, gpu, oracle, golden_tiny):
    om, m = oracle_loaded(mlb, gpu, oracle, "tiny")
    s = Session(m)
    try:
        s.prefill_min(2)  # the 4-token prompt takes the prompt pass (GEMV rows)
        prompt = list(golden_tiny["model_tiny_prompt"])
        gen = list(golden_tiny["model_tiny_generated"])
        assert list(s.generate(prompt, len(gen))) == gen
    finally:
        s.close()
        m.close()
        om.close()


def test_llama2_q4_0_prompt_pass_matches_oracle(mlb, gpu, oracle, golden_llama):
    om, m = oracle_loaded(mlb, gpu, oracle, "llama2_l2")
    s = Session(m)
    try:
        s.prefill_min(2)
        prompt = list(golden_llama["model_llama2_l2_prompt"])
        gen = list(golden_llama["model_llama2_l2_generated"])
        assert list(s.generate(prompt, len(gen))) == gen
        s.reset()
        s.generate(prompt, 1)
        assert_logits(last_logits(mlb, gpu, s, 32000), golden_llama["model_llama2_l2_logits"],
                      "llama2 prompt pass, last prompt position")
    finally:
        s.close()
        m.close()
        om.close()
