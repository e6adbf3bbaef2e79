"""Pins the C oracle to the reference: every oracle function must reproduce the
golden vectors that the reference CPU implementation itself produced
(tests/golden/make_golden.py over oracle/_ref/ref_harness) bit for bit.

The oracle restates the reference's fp32 operation order exactly, so the bar
here is bit equality, not a tolerance.
"""
import numpy as np
import pytest

from oracle.binding import Q40, Q41, Q80, STREAM_W, STREAM_X, Oracle

LINEAR_SHAPES = [(5, 13), (5, 32), (5, 33), (5, 64), (5, 129), (7, 176), (16, 896), (3, 4864)]


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def assert_bits_equal(actual, expected, what):
    a, e = bits(actual).ravel(), bits(expected).ravel()
    assert a.shape == e.shape, what
    bad = np.flatnonzero(a != e)
    assert bad.size == 0, f"{what}: {bad.size} mismatches, first at {bad[:5]}"


def test_fp16_to_f32_every_pattern(oracle, golden_ops):
    ref = golden_ops["fp16_to_f32"]
    ours = np.array([oracle.f16_to_f32(i) for i in range(65536)], np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(ours), nan)
    assert_bits_equal(ours[~nan], ref[~nan], "Fp16ToFloat")


def test_fp16_scale_probes(oracle, golden_ops):
    probes = golden_ops["fp16_probes"]
    d80, d40 = golden_ops["fp16_q80_d"], golden_ops["fp16_q40_d"]
    for i, p in enumerate(probes):
        blk = np.zeros(32, np.float32)
        blk[0] = p
        blk[7] = np.float32(p) * np.float32(0.25)
        q8 = oracle.quantize(Q80, blk)
        q4 = oracle.quantize(Q40, blk)
        assert int(q8[:2].view(np.uint16)[0]) == int(d80[i]), (i, p)
        assert int(q4[:2].view(np.uint16)[0]) == int(d40[i]), (i, p)


def test_fp16_known_answers(oracle):
    # test/core_cpu_test.cpp:198-216 of the reference
    def d_of(qtype, v):
        blk = np.zeros(32, np.float32)
        blk[0] = v
        return int(oracle.quantize(qtype, blk)[:2].view(np.uint16)[0])
    assert d_of(Q80, np.float32(127.0) / np.float32(65536.0)) == 0x0100
    assert d_of(Q40, np.float32(7.0) / np.float32(65536.0)) == 0x0100
    assert d_of(Q80, 190.5) == 0x3E00
    assert d_of(Q40, 10.5) == 0x3E00


def test_zero_blocks(oracle, golden_ops):
    z = np.zeros((2, 64), np.float32)
    assert np.array_equal(oracle.quantize(Q80, z), golden_ops["zero_q80"])
    assert np.array_equal(oracle.quantize(Q40, z), golden_ops["zero_q40"])
    assert not oracle.quantize(Q80, z).any() and not oracle.quantize(Q40, z).any()


@pytest.mark.parametrize("idx,shape", list(enumerate(LINEAR_SHAPES)))
def test_quantize_dequantize_linear(oracle, golden_ops, idx, shape):
    n, k = shape
    tag = f"{n}x{k}"
    w = oracle.normal(n * k, 2, STREAM_W + 16 * idx, 0.02).reshape(n, k)
    x = oracle.normal(3 * k, 2, STREAM_X + 16 * idx, 1.0).reshape(3, k)
    x1 = oracle.normal(k, 2, STREAM_X + 16 * idx + 1, 1.0)
    for qt, name in ((Q80, "80"), (Q40, "40"), (Q41, "41")):
        blocks = oracle.quantize(qt, w)
        assert np.array_equal(blocks, golden_ops[f"q{name}_{tag}"]), f"quantize q{name} {tag}"
        assert_bits_equal(oracle.dequantize(qt, blocks, n, k), golden_ops[f"deq{name}_{tag}"],
                          f"dequantize q{name} {tag}")
        assert_bits_equal(oracle.linear(qt, x, blocks, n), golden_ops[f"lin{name}_{tag}"],
                          f"linear q{name} {tag}")
        assert_bits_equal(oracle.linear(qt, x1, blocks, n), golden_ops[f"lin{name}v_{tag}"],
                          f"linear 1-D q{name} {tag}")


def test_rmsnorm(oracle, golden_ops):
    for idx, n in enumerate((129, 896, 4096)):
        x = oracle.normal(n, 2, 100 + idx, 1.0)
        w = (np.float32(1.0) + oracle.normal(n, 2, 200 + idx, 0.1)).astype(np.float32)
        for eps, tag in ((1e-5, "e5"), (1e-6, "e6")):
            assert_bits_equal(oracle.rmsnorm(x, w, np.float32(eps)),
                              golden_ops[f"rmsnorm_{n}_{tag}"], f"rmsnorm {n} {tag}")


def test_activations_and_argmax(oracle, golden_ops):
    g = oracle.normal(4864, 2, 300, 2.0)
    u = oracle.normal(4864, 2, 301, 1.0)
    assert_bits_equal(oracle.silu(g), golden_ops["silu"], "silu")
    assert_bits_equal(oracle.swiglu(g, u), golden_ops["swiglu"], "swiglu")
    assert_bits_equal(oracle.softmax(g), golden_ops["softmax"], "softmax")
    ties = np.array([0.5, 2.0, -1.0, 2.0, 1.0, 2.0, 0.0, -3.0, 1.5], np.float32)
    assert [oracle.argmax(ties), oracle.argmax(g), oracle.argmax(u)] == \
        list(golden_ops["argmax"])


ROPE_CASES = [
    ("qwen2", 64, 14, 2, 32768, 1e6, 1, [0, 1, 63, 191, 8191, 32767]),
    ("llama", 128, 32, 8, 768, 1e4, 0, [0, 5, 511, 767]),
    ("tiny", 16, 4, 2, 128, 1e4, 0, [0, 3, 11, 127]),
    ("gputest_normal", 14, 4, 2, 64, 1e4, 0, [3, 11]),
    ("gputest_neox", 14, 4, 2, 64, 1e4, 1, [3, 11]),
]


def test_rope(oracle, golden_ops):
    idx = 0
    for tag, hd, nh, nkv, max_seq, theta, neox, positions in ROPE_CASES:
        tables = oracle.rope_tables(max_seq, hd, theta)
        for pos in positions:
            q = oracle.normal(nh * hd, 4, 400 + idx, 1.0).reshape(nh, hd)
            k = oracle.normal(nkv * hd, 4, 500 + idx, 1.0).reshape(nkv, hd)
            assert_bits_equal(oracle.rope(q, pos, theta, neox, tables),
                              golden_ops[f"rope_q_{tag}_p{pos}"], f"rope q {tag} {pos}")
            assert_bits_equal(oracle.rope(k, pos, theta, neox, tables),
                              golden_ops[f"rope_k_{tag}_p{pos}"], f"rope k {tag} {pos}")
            # the direct form (freq and angle per call) is the same arithmetic
            assert_bits_equal(oracle.rope(q, pos, theta, neox),
                              golden_ops[f"rope_q_{tag}_p{pos}"], f"rope direct {tag} {pos}")
            idx += 1


def attention_case(oracle, layers, layer, pos, nh, nkv, hd, stream):
    max_seq = pos + 1
    per_layer = max_seq * nkv * hd
    kc = np.zeros((layers, max_seq, nkv, hd), np.float32)
    vc = np.zeros_like(kc)
    kc[layer] = oracle.normal(per_layer, 4, stream + 1, 1.0).reshape(max_seq, nkv, hd)
    vc[layer] = oracle.normal(per_layer, 4, stream + 2, 1.0).reshape(max_seq, nkv, hd)
    q = oracle.normal(nh * hd, 4, stream, 1.0).reshape(nh, hd)
    return q, kc, vc


ATTN_GRID = [(hd, pos) for hd in (7, 128, 129) for pos in (0, 4, 126, 127, 128, 256)]
ATTN_SWEEP = [(nh, nkv, hd, pos) for (nh, nkv, hd) in ((14, 2, 64), (32, 8, 128))
              for pos in (127, 1023, 8191, 32767)]
# shapes that exercise every tile geometry of the device kernel
ATTN_GEO = [(32, 1, 64, 300), (12, 4, 96, 257), (8, 8, 256, 100), (6, 2, 20, 70), (4, 1, 8, 40),
            (7, 7, 30, 33)]


def test_attention(oracle, golden_ops):
    stream = 1000
    for hd, pos in ATTN_GRID:
        q, kc, vc = attention_case(oracle, 2, 1, pos, 4, 2, hd, stream)
        assert_bits_equal(oracle.attention(q, kc, vc, 1, pos, 4, 2, hd),
                          golden_ops[f"attn_grid_hd{hd}_p{pos}"], f"attention {hd} {pos}")
        stream += 8
    for nh, nkv, hd, pos in ATTN_SWEEP:
        q, kc, vc = attention_case(oracle, 1, 0, pos, nh, nkv, hd, stream)
        assert_bits_equal(oracle.attention(q, kc, vc, 0, pos, nh, nkv, hd),
                          golden_ops[f"attn_sweep_{nh}x{hd}_p{pos}"], f"sweep {nh} {hd} {pos}")
        stream += 8
    for nh, nkv, hd, pos in ATTN_GEO:
        q, kc, vc = attention_case(oracle, 2, 1, pos, nh, nkv, hd, 5000 + 16 * nh + hd)
        assert_bits_equal(oracle.attention(q, kc, vc, 1, pos, nh, nkv, hd),
                          golden_ops[f"attn_geo_{nh}x{nkv}x{hd}_p{pos}"], f"geometry {nh} {nkv} {hd} {pos}")


def check_model(oracle, golden, name, prompt_len, n_new, full_logits, max_steps=None):
    m = oracle.model(name)
    try:
        prompt = m.prompt(prompt_len)
        assert np.array_equal(prompt, golden[f"model_{name}_prompt"])
        steps = prompt_len + n_new - 1
        if max_steps is not None:
            steps = min(steps, max_steps)
        top_idx = golden[f"model_{name}_top_idx"].reshape(-1, 8)
        top_val = golden[f"model_{name}_top_val"].reshape(-1, 8)
        gen_ref = golden[f"model_{name}_generated"]
        vocab = m.spec["vocab_size"]
        logits_ref = golden[f"model_{name}_logits"].reshape(-1, vocab)
        tokens = list(prompt)
        m.reset()
        for step in range(steps):
            logits = m.forward(tokens[step], step)
            assert np.array_equal(logits[top_idx[step]], top_val[step]), f"step {step} top-8"
            if full_logits:
                assert_bits_equal(logits, logits_ref[step], f"{name} logits step {step}")
            elif step == prompt_len - 1:
                assert_bits_equal(logits, logits_ref[0], f"{name} logits step {step}")
            if step >= prompt_len - 1:
                nxt = oracle.argmax(logits)
                assert nxt == gen_ref[step - prompt_len + 1], f"{name} token at step {step}"
                if len(tokens) == step + 1:
                    tokens.append(nxt)
    finally:
        m.close()


def test_model_tiny(oracle, golden_tiny):
    check_model(oracle, golden_tiny, "tiny", 4, 8, True)


def test_model_llama2_two_layers_q4_0(oracle, golden_llama):
    check_model(oracle, golden_llama, "llama2_l2", 6, 6, False)


@pytest.mark.slow
def test_model_qwen2_prefix(oracle, golden_qwen2):
    # 64 prompt positions plus the first 3 greedy steps; the complete 191-step
    # run is exercised by the GPU parity tests against the same fixture.
    check_model(oracle, golden_qwen2, "qwen2", 64, 128, False, max_steps=67)


def test_bench_prompt_ids_match_oracle_generator():
    """bench.py draws its prompt ids with the package's host generator; they
    are the oracle's seeded prompt stream."""
    from mini_llama_b200 import synth
    for n, seed, vocab in ((64, 3, 151936), (17, 1, 32000), (5, 42, 256)):
        assert np.array_equal(synth.tokens(n, seed, vocab), np.asarray(Oracle().tokens(n, seed, vocab)))
