"""The persistent decode kernel on small Q8_0 models against the oracle.

Shapes the kernel handles (every dimension a whole number of 32-blocks,
head_dim 32, 64 or 128) in three variants: Llama-style RoPE with
an untied head, Qwen2-style NeoX RoPE with q/k/v bias and a tied head at GQA
group 4, and a model whose dimension needs several tiles per CTA.  Greedy
tokens must equal the oracle's bit for bit and every step's logits must stay
within 1e-3 relative (|a - e| <= 1e-3 * max(1, max|e|)), through both
generate (one launch for the whole run) and single-token forwards.
"""
import numpy as np
import pytest

from mini_llama_b200 import capi
from mini_llama_b200.device import Model, Session
from oracle.binding import load_device_model

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3

VARIANTS = {
    "normal_untied": dict(hidden_dim=192, head_dim=32, n_heads=4, n_kv_heads=2, n_layers=2),
    "neox_bias_tied": dict(hidden_dim=256, head_dim=32, n_heads=8, n_kv_heads=2, n_layers=3,
                           rope_neox=1, qkv_bias=1, tied_embedding=1, seed=7, prompt_seed=9),
    "wide": dict(vocab_size=1000, dim=256, hidden_dim=640, head_dim=64, n_heads=4, n_kv_heads=4,
                 n_layers=2, max_seq_len=96, seed=11, prompt_seed=12),
}


def assert_logits(actual, expected, what):
    scale = max(1.0, float(np.abs(expected).max()))
    err = float(np.abs(actual.astype(np.float64) - expected).max())
    assert err <= LOGIT_TOL * scale, f"{what}: max error {err:.3e} (scale {scale:.3f})"


@pytest.fixture(params=sorted(VARIANTS), scope="module")
def variant(request, mlb, gpu, oracle):
    om = oracle.model("tiny", **VARIANTS[request.param])
    m = Model(mlb, gpu, om.spec)
    load_device_model(m, om)
    yield request.param, om, m
    m.close()
    om.close()


def test_persistent_matches_oracle(mlb, gpu, variant):
    name, om, m = variant
    prompt = om.prompt(6)
    n_new = 40
    gen_ref, logits_ref = om.greedy(prompt, n_new)
    s = Session(m)
    try:
        if s.path() != 2:
            s.use_persistent(True)  # raises with the reason the kernel was not selected
        assert s.path() == 2
        gen = s.generate(prompt, n_new)
        assert list(gen) == list(gen_ref), f"{name}: tokens"
        s.reset()
        tokens = list(prompt) + list(gen_ref)
        for step in range(len(tokens) - 1):
            logits, nxt = s.forward(tokens[step], step)
            assert_logits(logits, logits_ref[step], f"{name} step {step}")
            if step >= len(prompt) - 1:
                assert nxt == tokens[step + 1], f"{name}: token at step {step}"
    finally:
        s.close()


def test_persistent_runs_to_the_last_position(mlb, gpu, variant):
    """Generation that fills the cache up to max_seq_len - 1 (the arg-max of
    the last step lands in the history slot past the cache)."""
    name, om, m = variant
    max_seq = om.spec["max_seq_len"]
    prompt = om.prompt(3)
    n_new = max_seq - len(prompt) + 1
    gen_ref, _ = om.greedy(prompt, n_new)
    s = Session(m)
    try:
        gen = s.generate(prompt, n_new)
        assert list(gen) == list(gen_ref), f"{name}: tokens up to the last position"
        st = mlb.raw("mlb_session_generate", s.handle,
                     np.asarray(prompt, np.int32).ctypes.data, len(prompt), 0, n_new + 1,
                     np.zeros(n_new + 1, np.int32).ctypes.data)
        assert st == capi.MLB_ERR_OUT_OF_RANGE
    finally:
        s.close()


def test_persistent_matches_graph(mlb, gpu, variant):
    """Both decode paths of one session give the same greedy tokens, and
    switching between them mid-sequence keeps the KV cache coherent."""
    name, om, m = variant
    prompt = om.prompt(5)
    s = Session(m)
    try:
        a = s.generate(prompt, 24)
        s.reset()
        s.use_persistent(False)
        assert s.path() == 1
        b = s.generate(prompt, 24)
        assert list(a) == list(b), f"{name}: persistent vs graph"
        # first half on the graph, second half on the persistent kernel
        s.reset()
        s.generate(prompt, 12)
        s.use_persistent(True)
        tokens = list(prompt) + list(b)
        _, nxt = s.forward(tokens[len(prompt) + 11], len(prompt) + 11)
        assert nxt == b[12]
    finally:
        s.close()


def test_persistent_rejected_for_unsupported_shapes(mlb, gpu, oracle):
    """hidden_dim 176 is not a whole number of 32-blocks: the session keeps
    the graph path and refuses the persistent kernel."""
    om = oracle.model("tiny")
    m = Model(mlb, gpu, om.spec)
    try:
        load_device_model(m, om)
        s = Session(m)
        try:
            assert s.path() == 1
            st = mlb.raw("mlb_session_use_persistent", s.handle, 1)
            assert st == capi.MLB_ERR_UNSUPPORTED
            assert "multiples of 32" in mlb.last_error()
        finally:
            s.close()
    finally:
        m.close()
        om.close()


def test_bounded_wait_expires_and_device_recovers(mlb, gpu, variant):
    """A phase signal withheld by the host: every wait on it gives up after the
    session's wait limit, the call returns MLB_ERR_DEVICE_TIMEOUT (no fault,
    trap or hang: the waiting CTAs record the status and leave, the others
    see it and leave too), and the same session then decodes the oracle's
    tokens."""
    import time
    name, om, m = variant
    prompt = om.prompt(6)
    n_new = 12
    gen_ref, _ = om.greedy(prompt, n_new)
    s = Session(m)
    try:
        s.use_persistent(True)
        mlb.call("mlb_session_wait_limit", s.handle, 2_000_000)  # 2 ms
        mlb.call("mlb_session_test_withhold_signal", s.handle, 2)  # layer 0's FFN done
        p = np.asarray(prompt, np.int32)
        out = np.zeros(n_new, np.int32)
        t0 = time.perf_counter()
        st = mlb.raw("mlb_session_generate", s.handle, p.ctypes.data, len(p), 0, n_new, out.ctypes.data)
        elapsed = time.perf_counter() - t0
        assert st == capi.MLB_ERR_DEVICE_TIMEOUT, (name, st, mlb.last_error())
        assert "bounded device wait expired" in mlb.last_error()
        assert elapsed < 10.0, f"{name}: the expired wait took {elapsed:.1f} s to return"
        mlb.call("mlb_session_test_withhold_signal", s.handle, -1)
        mlb.call("mlb_session_wait_limit", s.handle, 2_000_000_000)
        s.reset()
        assert list(s.generate(prompt, n_new)) == list(gen_ref), f"{name}: tokens after the expired wait"
    finally:
        s.close()
