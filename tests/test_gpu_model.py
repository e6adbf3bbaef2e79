"""Whole-model parity of the decode session against the reference CPU path:
greedy tokens bit-exact, logits within 1e-3 relative (|a - e| <= 1e-3 *
max(1, max|e|) over the vocabulary).  The Qwen2 cases run through both decode
paths of a Q8_0 session: the persistent decode kernel (path 2) and the CUDA
graph per token (path 1)."""
import numpy as np
import pytest

from mini_llama_b200 import capi
from mini_llama_b200.device import DeviceArray, Model, Session
from oracle.binding import load_device_model
from oracle.binding import MODEL_SPECS

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3


def assert_logits(actual, expected, what):
    scale = max(1.0, float(np.abs(expected).max()))
    err = float(np.abs(actual.astype(np.float64) - expected).max())
    assert err <= LOGIT_TOL * scale, f"{what}: max error {err:.3e} (scale {scale:.3f})"


def oracle_loaded(mlb, gpu, oracle, name):
    om = oracle.model(name)
    m = Model(mlb, gpu, MODEL_SPECS[name])
    load_device_model(m, om)
    return om, m


def test_tiny_every_step(mlb, gpu, oracle, golden_tiny):
    om, m = oracle_loaded(mlb, gpu, oracle, "tiny")
    s = Session(m)
    try:
        prompt = list(golden_tiny["model_tiny_prompt"])
        gen = list(golden_tiny["model_tiny_generated"])
        ref_logits = golden_tiny["model_tiny_logits"].reshape(-1, 256)
        tokens = prompt + gen
        for step in range(len(prompt) + len(gen) - 1):
            logits, nxt = s.forward(tokens[step], step)
            assert_logits(logits, ref_logits[step], f"tiny step {step}")
            if step >= len(prompt) - 1:
                assert nxt == tokens[step + 1], f"tiny token at step {step}"
        # the same run through the device-side greedy loop
        s.reset()
        assert list(s.generate(prompt, len(gen))) == gen
    finally:
        s.close()
        m.close()
        om.close()


def test_llama2_q4_0_two_layers(mlb, gpu, oracle, golden_llama):
    om, m = oracle_loaded(mlb, gpu, oracle, "llama2_l2")
    s = Session(m)
    try:
        prompt = list(golden_llama["model_llama2_l2_prompt"])
        gen = list(golden_llama["model_llama2_l2_generated"])
        assert list(s.generate(prompt, len(gen))) == gen
        s.reset()
        for step, t in enumerate(prompt):
            logits, _ = s.forward(t, step)
        assert_logits(logits, golden_llama["model_llama2_l2_logits"], "llama2 last prompt step")
    finally:
        s.close()
        m.close()
        om.close()


@pytest.fixture(scope="module")
def qwen2(mlb, gpu):
    m = Model(mlb, gpu, MODEL_SPECS["qwen2"])
    m.synthesize(seed=MODEL_SPECS["qwen2"]["seed"], tied=True)
    yield m
    m.close()


@pytest.fixture(params=[2, 1], ids=["persistent", "graph"])
def qwen2_session(request, qwen2):
    s = Session(qwen2)
    if request.param == 1:
        s.use_persistent(False)
    assert s.path() == request.param
    yield s
    s.close()


def test_qwen2_device_weights_equal_oracle(mlb, gpu, oracle, qwen2):
    """Weights generated and quantized on the device equal the oracle's."""
    from oracle import binding as ob
    spec = MODEL_SPECS["qwen2"]
    D = spec["dim"]
    for layer, kind, rows, cols, stream in ((0, capi.W_WQ, 896, D, ob.stream_layer(0, 0)),
                                            (23, capi.W_DOWN, D, 4864, ob.stream_layer(23, 6))):
        w = oracle.normal(rows * cols, 3, stream, 0.02).reshape(rows, cols)
        ref = oracle.quantize(ob.Q80, w)
        ptr, nbytes = qwen2.weight(layer, kind)
        got = np.empty(nbytes, np.uint8)
        mlb.call("mlb_memcpy_d2h", gpu, got.ctypes.data, ptr, nbytes)
        assert np.array_equal(got, ref), (layer, kind)
    ptr, nbytes = qwen2.weight(5, capi.W_BK)
    got = np.empty(nbytes // 4, np.float32)
    mlb.call("mlb_memcpy_d2h", gpu, got.ctypes.data, ptr, nbytes)
    assert np.array_equal(got, oracle.normal(128, 3, ob.stream_layer(5, 8), 0.02))


def test_qwen2_greedy_128_tokens_bit_exact(mlb, gpu, qwen2_session, golden_qwen2):
    s = qwen2_session
    prompt = golden_qwen2["model_qwen2_prompt"]
    gen = golden_qwen2["model_qwen2_generated"]
    out = s.generate(prompt, len(gen))
    mismatch = np.flatnonzero(out != gen)
    assert mismatch.size == 0, f"first mismatch at generated token {mismatch[:3]}"
    # a second call on the same session (fresh counters, same cache layout)
    s.reset()
    assert np.array_equal(s.generate(prompt, 16), gen[:16])


def test_qwen2_logits_per_step(mlb, gpu, qwen2_session, golden_qwen2):
    """Per-step top-8 logits of the reference CPU path, and the full logits of
    the last prompt position, through single-token forwards."""
    s = qwen2_session
    prompt = list(golden_qwen2["model_qwen2_prompt"])
    gen = list(golden_qwen2["model_qwen2_generated"])
    tokens = prompt + gen
    top_idx = golden_qwen2["model_qwen2_top_idx"].reshape(-1, 8)
    top_val = golden_qwen2["model_qwen2_top_val"].reshape(-1, 8)
    scale = max(1.0, float(np.abs(top_val).max()))
    for step in range(len(tokens) - 1):
        logits, nxt = s.forward(tokens[step], step)
        err = float(np.abs(logits[top_idx[step]] - top_val[step]).max())
        assert err <= LOGIT_TOL * scale, f"step {step}: top-8 error {err:.3e}"
        if step == len(prompt) - 1:
            assert_logits(logits, golden_qwen2["model_qwen2_logits"], "last prompt step")
        if step >= len(prompt) - 1:
            assert nxt == tokens[step + 1], f"token at step {step}"


def test_session_device_decode_matches_generate(mlb, gpu, qwen2_session, golden_qwen2):
    """The measurement entry point (tokens on the device) produces the same
    greedy continuation as mlb_session_generate."""
    s = qwen2_session
    prompt = golden_qwen2["model_qwen2_prompt"]
    gen = golden_qwen2["model_qwen2_generated"]
    s.generate(prompt, 1)  # prefill positions 0..63, first token at 64
    toks = DeviceArray(mlb, gpu, 128, np.int32)
    first = np.zeros(128, np.int32)
    first[0] = gen[0]
    toks.upload(first)
    s.decode_device(toks.ptr, len(prompt), 127)
    assert np.array_equal(toks.download()[1:], gen[1:128])


def test_session_rejects_bad_inputs(mlb, gpu, qwen2):
    s = Session(qwen2)
    try:
        import ctypes
        st = mlb.raw("mlb_session_forward", s.handle, 151936, 0, None, None)
        assert st == capi.MLB_ERR_OUT_OF_RANGE and "token id out of range" in mlb.last_error()
        st = mlb.raw("mlb_session_forward", s.handle, 1, 256, None, None)
        assert st == capi.MLB_ERR_OUT_OF_RANGE and "position out of range" in mlb.last_error()
        p = np.array([1, 2], np.int32)
        out = np.zeros(300, np.int32)
        st = mlb.raw("mlb_session_generate", s.handle, p.ctypes.data, 2, 0, 300, out.ctypes.data)
        assert st == capi.MLB_ERR_OUT_OF_RANGE
    finally:
        s.close()



def test_q8_0_session_uses_integer_mma_path(mlb, gpu, qwen2):
    """A Q8_0 model decodes through the persistent kernel by default; the
    graph of integer-MMA GEMVs over R16 weights stays selectable."""
    import ctypes
    s = Session(qwen2)
    try:
        path = ctypes.c_int(-1)
        mlb.call("mlb_session_gemv_path", s.handle, ctypes.byref(path))
        assert path.value == 2
        s.use_persistent(False)
        assert s.path() == 1
        s.use_persistent(True)
        assert s.path() == 2
    finally:
        s.close()
