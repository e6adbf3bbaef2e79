"""GPU parity of the op-level C ABI against the oracle and the reference's own
golden vectors.

Tolerances (mixed absolute/relative as in the reference's RequireClose,
test/gpu_core_test.cpp:35-53: |a - e| <= tol * max(1, |e|)):
  - quantized linear: 1e-4 (the target for quantized linear outputs)
  - attention, RMSNorm, SiLU, softmax: 1e-4
  - RoPE, quantization, dequantization, KV write, embedding, arg-max and the
    synthetic generator: bit-exact
"""
import ctypes

import numpy as np
import pytest

from mini_llama_b200 import capi
from mini_llama_b200.device import DeviceArray
from oracle.binding import BLOCK_BYTES, Q40, Q41, Q80, STREAM_W, STREAM_X

pytestmark = pytest.mark.gpu

LIN_TOL = 1e-4
OP_TOL = 1e-4
# Quantized linears, per output: |a - e| <= LIN_TOL * |e| + LIN_FLOOR * sum_k |x_k w_k|.
# 1e-4 relative to the output itself, with a floor at the rounding noise of a
# fp32 dot product of K terms: the reference's own result (sequential fp32
# sums) differs from the exact value by up to 4e-7 * sum_k |x_k w_k| on the
# benchmark shapes, so no computation can be held closer to it than that.
LIN_FLOOR = 2.0 ** -20
QNAME = {Q80: "q8_0", Q40: "q4_0", Q41: "q4_1"}
LINEAR_SHAPES = [(5, 13), (5, 32), (5, 33), (5, 64), (5, 129), (7, 176), (16, 896), (3, 4864)]


def assert_close(actual, expected, tol, what):
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    assert a.shape == e.shape, what
    assert np.all(np.isfinite(a)), f"{what}: non-finite output"
    err = np.abs(a - e)
    bound = tol * np.maximum(1.0, np.abs(e))
    bad = np.flatnonzero(err > bound)
    assert bad.size == 0, (f"{what}: {bad.size} of {a.size} outside {tol}, worst "
                           f"{float((err / np.maximum(1.0, np.abs(e))).max()):.3e} at {bad[:4]}")


def linear_terms(x, wdq, bias=None):
    """sum_k |x_k w_k| (+ |bias|) per output, from the dequantized weights."""
    x = np.asarray(x, np.float32)
    t = np.abs(x) @ np.abs(np.asarray(wdq, np.float32)).T
    return t + np.abs(bias) if bias is not None else t


def assert_linear_close(actual, expected, terms, what):
    """Every output within LIN_TOL of itself, or within the fp32 rounding floor
    of its terms."""
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    t = np.asarray(terms, np.float64).ravel()
    assert a.shape == e.shape == t.shape, what
    assert np.all(np.isfinite(a)), f"{what}: non-finite output"
    err = np.abs(a - e)
    bound = LIN_TOL * np.abs(e) + LIN_FLOOR * t
    bad = np.flatnonzero(err > bound)
    worst = int(np.argmax(err / bound))
    assert bad.size == 0, (f"{what}: {bad.size} of {a.size} outside 1e-4 |e| + 2^-20 sum|x w|; worst "
                           f"{err[worst]:.3e} (|e| {abs(e[worst]):.3e}, sum|x w| {t[worst]:.3e}) at {bad[:4]}")


def linear_gpu(mlb, dev, qtype, x, blocks, n, bias=None):
    x = np.ascontiguousarray(x, np.float32)
    rows, k = (1, x.shape[0]) if x.ndim == 1 else x.shape
    xd = DeviceArray.from_host(mlb, dev, x)
    wd = DeviceArray.from_host(mlb, dev, blocks)
    bd = DeviceArray.from_host(mlb, dev, bias) if bias is not None else None
    yd = DeviceArray(mlb, dev, (rows, n))
    nb = (k + 31) // 32
    mlb.call("mlb_quant_linear", dev, qtype, xd.ptr, wd.ptr, n * nb, rows, k, n,
             bd.ptr if bd else None, yd.ptr)
    return yd.download().reshape((n,) if x.ndim == 1 else (rows, n))


@pytest.mark.parametrize("qtype", [Q80, Q40, Q41])
@pytest.mark.parametrize("idx,shape", list(enumerate(LINEAR_SHAPES)))
def test_linear_matches_reference_golden(mlb, gpu, oracle, golden_ops, qtype, idx, shape):
    n, k = shape
    tag = f"{n}x{k}"
    name = {Q80: "80", Q40: "40", Q41: "41"}[qtype]
    blocks = golden_ops[f"q{name}_{tag}"]
    x = oracle.normal(3 * k, 2, STREAM_X + 16 * idx, 1.0).reshape(3, k)
    x1 = oracle.normal(k, 2, STREAM_X + 16 * idx + 1, 1.0)
    wdq = oracle.dequantize(qtype, blocks, n, k)
    assert_linear_close(linear_gpu(mlb, gpu, qtype, x, blocks, n), golden_ops[f"lin{name}_{tag}"],
                        linear_terms(x, wdq), f"{QNAME[qtype]} batch {tag}")
    assert_linear_close(linear_gpu(mlb, gpu, qtype, x1, blocks, n), golden_ops[f"lin{name}v_{tag}"],
                        linear_terms(x1[None, :], wdq), f"{QNAME[qtype]} 1-D {tag}")
    bias = oracle.normal(n, 2, 999, 0.1)
    assert_linear_close(linear_gpu(mlb, gpu, qtype, x1, blocks, n, bias),
                        golden_ops[f"lin{name}v_{tag}"] + bias, linear_terms(x1[None, :], wdq, bias),
                        f"{QNAME[qtype]} bias {tag}")


BENCH_SHAPES = [(896, 896), (4864, 896), (896, 4864), (151936, 896)]
_WEIGHTS = {}
_DEQUANT = {}


def bench_blocks(oracle, qtype, n, k):
    key = (qtype, n, k)
    if key not in _WEIGHTS:
        w = oracle.normal(n * k, 2, STREAM_W + 1000 + n + k, 0.02).reshape(n, k)
        _WEIGHTS[key] = oracle.quantize(qtype, w)
    return _WEIGHTS[key]


def bench_dequant(oracle, qtype, n, k):
    """The dequantized benchmark weights (the last shape asked for is kept)."""
    key = (qtype, n, k)
    if key not in _DEQUANT:
        _DEQUANT.clear()
        _DEQUANT[key] = oracle.dequantize(qtype, bench_blocks(oracle, qtype, n, k), n, k)
    return _DEQUANT[key]


@pytest.mark.parametrize("qtype", [Q80, Q40, Q41])
@pytest.mark.parametrize("n,k", BENCH_SHAPES)
@pytest.mark.parametrize("m", [1, 8])
def test_linear_microbench_shapes(mlb, gpu, oracle, qtype, n, k, m):
    blocks = bench_blocks(oracle, qtype, n, k)
    x = oracle.normal(m * k, 2, STREAM_X + 1000 + n + k, 1.0).reshape(m, k)
    expect = oracle.linear(qtype, x, blocks, n)
    assert_linear_close(linear_gpu(mlb, gpu, qtype, x, blocks, n), expect,
                        linear_terms(x, bench_dequant(oracle, qtype, n, k)), f"{QNAME[qtype]} [{n},{k}] M={m}")


# Shapes with enough 16-row tiles per SM (4) to take the tensor-core GEMV over
# the blocks for 1..8 rows, covering its unit and bank layouts: K = 4864 (rows
# split into 8-block pieces copied row by row; at 8 rows of x its digit tables
# leave too little room, so the call runs two launches of 4 rows), 1024 (16
# whole rows per copy, row pitch 0 mod 8 words), 576 (odd pitch in words), 896
# (pitch 2 mod 4 words: interleaved rows), 800 (odd block count: Q4_1 here,
# the other GEMV for Q8_0 / Q4_0); every N ends on a partial tile (3 or 4
# rows).
BLOCK_MMA_SHAPES = [(9475, 4864), (9475, 1024), (9475, 576), (9475, 896), (9492, 896), (9475, 800)]


@pytest.mark.parametrize("qtype", [Q80, Q40, Q41])
@pytest.mark.parametrize("n,k", BLOCK_MMA_SHAPES)
def test_linear_block_mma_layouts(mlb, gpu, oracle, qtype, n, k):
    w = oracle.normal(n * k, 2, STREAM_W + 3000 + k, 0.02).reshape(n, k)
    blocks = oracle.quantize(qtype, w)
    wdq = np.abs(np.asarray(oracle.dequantize(qtype, blocks, n, k), np.float32))  # |w| for the terms
    bias = oracle.normal(n, 2, 3001, 0.1)
    for m in (1, 2, 3, 8):
        x = oracle.normal(m * k, 2, STREAM_X + 3000 + k + m, 1.0).reshape(m, k)
        expect = oracle.linear(qtype, x, blocks, n)
        assert_linear_close(linear_gpu(mlb, gpu, qtype, x, blocks, n), expect, linear_terms(x, wdq),
                            f"{QNAME[qtype]} [{n},{k}] M={m}")
        assert_linear_close(linear_gpu(mlb, gpu, qtype, x, blocks, n, bias), expect + bias,
                            linear_terms(x, wdq, bias), f"{QNAME[qtype]} [{n},{k}] M={m} bias")


def test_linear_block_mma_repeated_calls(mlb, gpu, oracle):
    """The GEMV's tile scheduler resets itself at the end of every launch:
    calls in a row, of different shapes, each give the full result."""
    cases = [(151936 // 8, 896, 1), (9475, 4864, 8), (9475, 896, 5)]
    for rep in range(2):
        for (n, k, m) in cases:
            blocks = bench_blocks(oracle, Q80, n, k)
            x = oracle.normal(m * k, 2, STREAM_X + 4000 + n + m + rep, 1.0).reshape(m, k)
            got = linear_gpu(mlb, gpu, Q80, x, blocks, n)
            assert_linear_close(got, oracle.linear(Q80, x, blocks, n),
                                linear_terms(x, bench_dequant(oracle, Q80, n, k)), f"[{n},{k}] M={m} call {rep}")


def test_linear_misaligned_weight_pointer(mlb, gpu, oracle):
    """A weight pointer off the 16-byte grid takes the direct-load kernel."""
    n, k = 33, 96
    w = oracle.normal(n * k, 2, 77, 0.02).reshape(n, k)
    blocks = oracle.quantize(Q80, w)
    x = oracle.normal(2 * k, 2, 78, 1.0).reshape(2, k)
    buf = DeviceArray(mlb, gpu, blocks.nbytes + 16, np.uint8)
    shifted = np.zeros(blocks.nbytes + 16, np.uint8)
    shifted[2:2 + blocks.nbytes] = blocks
    buf.upload(shifted)
    xd = DeviceArray.from_host(mlb, gpu, x)
    yd = DeviceArray(mlb, gpu, (2, n))
    mlb.call("mlb_q80_linear", gpu, xd.ptr, buf.ptr + 2, blocks.nbytes // 34, 2, k, n, None,
             yd.ptr)
    assert_linear_close(yd.download(), oracle.linear(Q80, x, blocks, n),
                        linear_terms(x, oracle.dequantize(Q80, blocks, n, k)), "misaligned")


def test_linear_rejects_bad_block_count(mlb, gpu):
    xd = DeviceArray(mlb, gpu, 32)
    wd = DeviceArray(mlb, gpu, 34 * 4, np.uint8)
    yd = DeviceArray(mlb, gpu, 4)
    st = mlb.raw("mlb_q80_linear", gpu, xd.ptr, wd.ptr, 3, 1, 32, 4, None, yd.ptr)
    assert st == capi.MLB_ERR_INVALID_ARGUMENT
    assert "block count mismatch: expected 4, got 3" in mlb.last_error()
    assert mlb.raw("mlb_q80_linear", gpu, xd.ptr, None, 4, 1, 32, 4, None, yd.ptr) != 0
    assert "null" in mlb.last_error()


@pytest.mark.parametrize("qtype", [Q80, Q40, Q41])
def test_device_quantizer_bit_exact(mlb, gpu, oracle, golden_ops, qtype):
    name = {Q80: "80", Q40: "40", Q41: "41"}[qtype]
    for idx, (n, k) in enumerate(LINEAR_SHAPES):
        w = oracle.normal(n * k, 2, STREAM_W + 16 * idx, 0.02).reshape(n, k)
        wd = DeviceArray.from_host(mlb, gpu, w)
        nb = (k + 31) // 32
        qd = DeviceArray(mlb, gpu, n * nb * BLOCK_BYTES[qtype], np.uint8)
        mlb.call("mlb_quantize", gpu, qtype, wd.ptr, n, k, qd.ptr)
        got = qd.download()
        assert np.array_equal(got, golden_ops[f"q{name}_{n}x{k}"]), f"quantize {qtype} {n}x{k}"
        yd = DeviceArray(mlb, gpu, (n, k))
        mlb.call("mlb_dequantize", gpu, qtype, qd.ptr, n, k, yd.ptr)
        ref = golden_ops[f"deq{name}_{n}x{k}"]
        assert np.array_equal(yd.download().view(np.uint32).ravel(), ref.view(np.uint32)), \
            f"dequantize {qtype} {n}x{k}"


def test_device_quantizer_fp16_probes(mlb, gpu, golden_ops):
    probes = golden_ops["fp16_probes"]
    blocks = np.zeros((len(probes), 32), np.float32)
    blocks[:, 0] = probes
    blocks[:, 7] = probes * np.float32(0.25)
    xd = DeviceArray.from_host(mlb, gpu, blocks)
    for qtype, key, bb in ((Q80, "fp16_q80_d", 34), (Q40, "fp16_q40_d", 18)):
        qd = DeviceArray(mlb, gpu, len(probes) * bb, np.uint8)
        mlb.call("mlb_quantize", gpu, qtype, xd.ptr, len(probes), 32, qd.ptr)
        d = qd.download().reshape(len(probes), bb)[:, :2].copy().view(np.uint16).ravel()
        assert np.array_equal(d, golden_ops[key]), key


def test_synth_device_matches_host(mlb, gpu, oracle):
    for seed, stream, sigma, n in ((3, 1, 0.02, 100003), (4, 1005, 1.0, 4096), (2, 8, 0.02, 17)):
        d = DeviceArray(mlb, gpu, n)
        mlb.call("mlb_synth_normal", gpu, d.ptr, n, seed, stream, sigma)
        host = oracle.normal(n, seed, stream, sigma)
        assert np.array_equal(d.download().view(np.uint32), host.view(np.uint32))


def test_rmsnorm(mlb, gpu, oracle, golden_ops):
    for idx, n in enumerate((129, 896, 4096)):
        x = oracle.normal(n, 2, 100 + idx, 1.0)
        w = (np.float32(1.0) + oracle.normal(n, 2, 200 + idx, 0.1)).astype(np.float32)
        xd, wd, yd = (DeviceArray.from_host(mlb, gpu, x), DeviceArray.from_host(mlb, gpu, w),
                      DeviceArray(mlb, gpu, n))
        for eps, tag in ((1e-5, "e5"), (1e-6, "e6")):
            mlb.call("mlb_rmsnorm", gpu, xd.ptr, wd.ptr, n, eps, yd.ptr)
            assert_close(yd.download(), golden_ops[f"rmsnorm_{n}_{tag}"], OP_TOL, f"rmsnorm {n}")


def test_activations_softmax_argmax(mlb, gpu, oracle, golden_ops):
    g = oracle.normal(4864, 2, 300, 2.0)
    u = oracle.normal(4864, 2, 301, 1.0)
    gd, ud, yd = (DeviceArray.from_host(mlb, gpu, g), DeviceArray.from_host(mlb, gpu, u),
                  DeviceArray(mlb, gpu, 4864))
    mlb.call("mlb_silu", gpu, gd.ptr, 4864, yd.ptr)
    assert_close(yd.download(), golden_ops["silu"], OP_TOL, "silu")
    mlb.call("mlb_mul", gpu, gd.ptr, ud.ptr, 4864, yd.ptr)
    assert np.array_equal(yd.download(), g * u)
    mlb.call("mlb_add", gpu, gd.ptr, ud.ptr, 4864, yd.ptr)
    assert np.array_equal(yd.download(), g + u)
    mlb.call("mlb_softmax", gpu, gd.ptr, 4864, yd.ptr)
    assert_close(yd.download(), golden_ops["softmax"], OP_TOL, "softmax")
    out = DeviceArray(mlb, gpu, 1, np.int32)
    ties = np.array([0.5, 2.0, -1.0, 2.0, 1.0, 2.0, 0.0, -3.0, 1.5], np.float32)
    got = []
    for v in (ties, g, u):
        vd = DeviceArray.from_host(mlb, gpu, v)
        mlb.call("mlb_argmax", gpu, vd.ptr, len(v), out.ptr)
        got.append(int(out.download()[0]))
    assert got == list(golden_ops["argmax"])


ROPE_CASES = [
    ("qwen2", 64, 14, 2, 1e6, 1, [0, 1, 63, 191, 8191, 32767]),
    ("llama", 128, 32, 8, 1e4, 0, [0, 5, 511, 767]),
    ("tiny", 16, 4, 2, 1e4, 0, [0, 3, 11, 127]),
    ("gputest_normal", 14, 4, 2, 1e4, 0, [3, 11]),
    ("gputest_neox", 14, 4, 2, 1e4, 1, [3, 11]),
]


def test_rope_bit_exact(mlb, gpu, oracle, golden_ops):
    idx = 0
    for tag, hd, nh, nkv, theta, neox, positions in ROPE_CASES:
        for pos in positions:
            q = oracle.normal(nh * hd, 4, 400 + idx, 1.0)
            k = oracle.normal(nkv * hd, 4, 500 + idx, 1.0)
            qd, kd = DeviceArray.from_host(mlb, gpu, q), DeviceArray.from_host(mlb, gpu, k)
            mlb.call("mlb_rope", gpu, qd.ptr, kd.ptr, nh, nkv, hd, pos, theta,
                     capi.ROPE_NEOX if neox else capi.ROPE_NORMAL)
            for got, key in ((qd.download(), f"rope_q_{tag}_p{pos}"),
                             (kd.download(), f"rope_k_{tag}_p{pos}")):
                assert np.array_equal(got.view(np.uint32), golden_ops[key].view(np.uint32)), key
            idx += 1


def test_embedding_and_kv_write(mlb, gpu, oracle):
    table = oracle.normal(50 * 24, 9, 1, 1.0).reshape(50, 24)
    td, yd = DeviceArray.from_host(mlb, gpu, table), DeviceArray(mlb, gpu, 24)
    mlb.call("mlb_embedding", gpu, td.ptr, 50, 24, 37, yd.ptr)
    assert np.array_equal(yd.download(), table[37])
    assert mlb.raw("mlb_embedding", gpu, td.ptr, 50, 24, 50, yd.ptr) == capi.MLB_ERR_INVALID_ARGUMENT
    layers, seq, nkv, hd = 3, 9, 2, 8
    kc = DeviceArray(mlb, gpu, (layers, seq, nkv, hd))
    vc = DeviceArray(mlb, gpu, (layers, seq, nkv, hd))
    mlb.call("mlb_memset", gpu, kc.ptr, 0, kc.nbytes)
    mlb.call("mlb_memset", gpu, vc.ptr, 0, vc.nbytes)
    k = oracle.normal(nkv * hd, 9, 2, 1.0)
    v = oracle.normal(nkv * hd, 9, 3, 1.0)
    kd, vd = DeviceArray.from_host(mlb, gpu, k), DeviceArray.from_host(mlb, gpu, v)
    mlb.call("mlb_kv_write", gpu, kc.ptr, vc.ptr, layers, seq, nkv, hd, 2, 5, kd.ptr, vd.ptr)
    K, V = kc.download(), vc.download()
    assert np.array_equal(K[2, 5].ravel(), k) and np.array_equal(V[2, 5].ravel(), v)
    K[2, 5] = 0
    V[2, 5] = 0
    assert not K.any() and not V.any()
    st = mlb.raw("mlb_kv_write", gpu, kc.ptr, vc.ptr, layers, seq, nkv, hd, 2, seq, kd.ptr, vd.ptr)
    assert st == capi.MLB_ERR_OUT_OF_RANGE and "position out of range" in mlb.last_error()


def attention_inputs(oracle, layers, layer, pos, nh, nkv, hd, stream, max_seq=None):
    max_seq = max_seq or pos + 1
    per_layer = (pos + 1) * nkv * hd
    kc = np.zeros((layers, max_seq, nkv, hd), np.float32)
    vc = np.zeros_like(kc)
    kc[layer, :pos + 1] = oracle.normal(per_layer, 4, stream + 1, 1.0).reshape(pos + 1, nkv, hd)
    vc[layer, :pos + 1] = oracle.normal(per_layer, 4, stream + 2, 1.0).reshape(pos + 1, nkv, hd)
    q = oracle.normal(nh * hd, 4, stream, 1.0).reshape(nh, hd)
    return q, kc, vc


def attention_gpu(mlb, dev, q, kc, vc, layer, pos, nh, nkv, hd):
    qd, kd, vd = (DeviceArray.from_host(mlb, dev, q), DeviceArray.from_host(mlb, dev, kc),
                  DeviceArray.from_host(mlb, dev, vc))
    od = DeviceArray(mlb, dev, (nh, hd))
    mlb.call("mlb_attention_decode", dev, qd.ptr, kd.ptr, vd.ptr, kc.shape[0], kc.shape[1],
             layer, pos, nh, nkv, hd, od.ptr)
    return od.download()


def test_attention_reference_grid(mlb, gpu, oracle, golden_ops):
    stream = 1000
    for hd in (7, 128, 129):
        for pos in (0, 4, 126, 127, 128, 256):
            q, kc, vc = attention_inputs(oracle, 2, 1, pos, 4, 2, hd, stream)
            got = attention_gpu(mlb, gpu, q, kc, vc, 1, pos, 4, 2, hd)
            assert_close(got, golden_ops[f"attn_grid_hd{hd}_p{pos}"], OP_TOL,
                         f"attention hd={hd} pos={pos}")
            stream += 8


@pytest.mark.parametrize("shape", [(14, 2, 64), (32, 8, 128)])
def test_attention_sweep(mlb, gpu, oracle, golden_ops, shape):
    nh, nkv, hd = shape
    stream = 1000 + 18 * 8 + (0 if nh == 14 else 4 * 8)
    for pos in (127, 1023, 8191, 32767):
        q, kc, vc = attention_inputs(oracle, 1, 0, pos, nh, nkv, hd, stream)
        got = attention_gpu(mlb, gpu, q, kc, vc, 0, pos, nh, nkv, hd)
        assert_close(got, golden_ops[f"attn_sweep_{nh}x{hd}_p{pos}"], OP_TOL,
                     f"sweep {nh}x{hd} pos={pos}")
        stream += 8


@pytest.mark.parametrize("shape", [
    (32, 1, 64, 300),   # 32 query heads on one KV head: two head groups of 16 per KV head
    (12, 4, 96, 257),   # head_dim 96: rows of 24 pieces, strided value rows
    (8, 8, 256, 100),   # head_dim 256: 16-row tiles
    (6, 2, 20, 70),     # head_dim 20: five pieces per row, two score threads per position
    (4, 1, 8, 40),      # head_dim 8: 256-row tiles, a thread per position
    (7, 7, 30, 33),     # head_dim 30: single-float copies, padded rows
])
def test_attention_tile_geometries(mlb, gpu, oracle, shape):
    """Every tile geometry of the split-K kernel (rows per tile, threads per
    position, value-row layout, head groups) against the oracle."""
    nh, nkv, hd, pos = shape
    q, kc, vc = attention_inputs(oracle, 2, 1, pos, nh, nkv, hd, 5000 + nh * 16 + hd, max_seq=pos + 9)
    got = attention_gpu(mlb, gpu, q, kc, vc, 1, pos, nh, nkv, hd)
    ref = oracle.attention(q, kc, vc, 1, pos, nh, nkv, hd)
    assert_close(got, ref, OP_TOL, f"attention {nh}/{nkv}x{hd} pos={pos}")


def test_attention_batched_independent_sequences(mlb, gpu, oracle):
    """32 sequences with different lengths in one call equal 32 single calls."""
    batch, nh, nkv, hd, max_seq, layers = 32, 14, 2, 64, 300, 2
    rng = np.random.default_rng(4)
    positions = rng.integers(0, max_seq, batch).astype(np.int32)
    positions[0], positions[1] = 0, max_seq - 1
    kc = oracle.normal(batch * layers * max_seq * nkv * hd, 4, 7000, 1.0).reshape(
        batch, layers, max_seq, nkv, hd)
    vc = oracle.normal(batch * layers * max_seq * nkv * hd, 4, 7001, 1.0).reshape(kc.shape)
    q = oracle.normal(batch * nh * hd, 4, 7002, 1.0).reshape(batch, nh, hd)
    qd, kd, vd = (DeviceArray.from_host(mlb, gpu, q), DeviceArray.from_host(mlb, gpu, kc),
                  DeviceArray.from_host(mlb, gpu, vc))
    pd = DeviceArray.from_host(mlb, gpu, positions)
    od = DeviceArray(mlb, gpu, (batch, nh, hd))
    mlb.call("mlb_attention_decode_batched", gpu, batch, qd.ptr, kd.ptr, vd.ptr, layers, max_seq,
             1, pd.ptr, int(positions.max()), nh, nkv, hd, od.ptr)
    got = od.download()
    for b in range(batch):
        ref = oracle.attention(q[b], kc[b], vc[b], 1, int(positions[b]), nh, nkv, hd)
        assert_close(got[b], ref, OP_TOL, f"sequence {b} pos={positions[b]}")


def test_attention_validation(mlb, gpu):
    q = DeviceArray(mlb, gpu, 64)
    kc = DeviceArray(mlb, gpu, 2 * 4 * 64)
    st = mlb.raw("mlb_attention_decode", gpu, q.ptr, kc.ptr, kc.ptr, 1, 4, 0, 4, 1, 1, 64, q.ptr)
    assert st == capi.MLB_ERR_OUT_OF_RANGE
    st = mlb.raw("mlb_attention_decode", gpu, q.ptr, kc.ptr, kc.ptr, 1, 4, 0, 1, 3, 2, 64, q.ptr)
    assert st == capi.MLB_ERR_INVALID_ARGUMENT and "divisible" in mlb.last_error()


R16_SHAPES = [(5, 13), (16, 32), (33, 33), (7, 176), (896, 896), (4864, 896), (896, 4864),
              (151936, 896)]


@pytest.mark.parametrize("n,k", R16_SHAPES)
@pytest.mark.parametrize("m", [1, 2, 3, 8])
def test_q80_r16_integer_mma_linear(mlb, gpu, oracle, n, k, m):
    """Prepared (R16) Q8_0 weights through the integer tensor-core GEMV."""
    if n == 151936 and m not in (1, 8):
        pytest.skip("lm_head shape covered at M = 1 and 8")
    blocks = bench_blocks(oracle, Q80, n, k) if (n, k) in BENCH_SHAPES else oracle.quantize(
        Q80, oracle.normal(n * k, 2, STREAM_W + 3000 + n + k, 0.02).reshape(n, k))
    x = oracle.normal(m * k, 2, STREAM_X + 3000 + n + k, 1.0).reshape(m, k)
    x[0, :7] *= np.float32(1e-3)   # blocks with a wide dynamic range
    if k > 40:
        x[-1, 32:64] = 0.0         # an all-zero block
    expect = oracle.linear(Q80, x, blocks, n)
    wd = DeviceArray.from_host(mlb, gpu, blocks)
    r16 = DeviceArray(mlb, gpu, mlb.dll.mlb_r16_bytes(n, k), np.uint8)
    mlb.call("mlb_q80_repack_r16", gpu, wd.ptr, n, k, r16.ptr)
    xd = DeviceArray.from_host(mlb, gpu, x)
    yd = DeviceArray(mlb, gpu, (m, n))
    bias = oracle.normal(n, 2, 4000 + n, 0.1)
    bd = DeviceArray.from_host(mlb, gpu, bias)
    mlb.call("mlb_q80_linear_r16", gpu, xd.ptr, r16.ptr, m, k, n, bd.ptr, yd.ptr)
    wdq = bench_dequant(oracle, Q80, n, k) if (n, k) in BENCH_SHAPES else oracle.dequantize(Q80, blocks, n, k)
    assert_linear_close(yd.download(), expect + bias, linear_terms(x, wdq, bias), f"R16 [{n},{k}] M={m}")


def test_q80_r16_layout(mlb, gpu, oracle):
    """The R16 copy holds the same quants and scales, regrouped."""
    n, k = 20, 70
    blocks = oracle.quantize(Q80, oracle.normal(n * k, 2, 5000, 0.02).reshape(n, k))
    nb = 3
    wd = DeviceArray.from_host(mlb, gpu, blocks)
    size = mlb.dll.mlb_r16_bytes(n, k)
    assert size == 2 * nb * 544
    r16 = DeviceArray(mlb, gpu, size, np.uint8)
    mlb.call("mlb_q80_repack_r16", gpu, wd.ptr, n, k, r16.ptr)
    got = r16.download().reshape(2, nb, 544)
    g = blocks.reshape(n, nb, 34)
    for r in range(32):
        t, i = divmod(r, 16)
        for b in range(nb):
            chunk = got[t, b]
            swz = (i >> 2) & 1
            q = np.concatenate([chunk[32 * i + 16 * (0 ^ swz):32 * i + 16 * (0 ^ swz) + 16],
                                chunk[32 * i + 16 * (1 ^ swz):32 * i + 16 * (1 ^ swz) + 16]])
            d = chunk[512 + 2 * i:514 + 2 * i]
            if r < n:
                assert np.array_equal(q, g[r, b, 2:]) and np.array_equal(d, g[r, b, :2])
            else:
                assert not q.any() and not d.any()


@pytest.mark.parametrize("m,k,n", [(1, 33, 7), (3, 33, 7), (1, 896, 4864), (8, 896, 1000),
                                   (2, 4864, 896), (1, 896, 151936)])
def test_f32_linear(mlb, gpu, oracle, m, k, n):
    w = oracle.normal(n * k, 6, 100 + k, 0.02).reshape(n, k)
    x = oracle.normal(m * k, 6, 200 + k, 1.0).reshape(m, k)
    bias = oracle.normal(n, 6, 300, 0.1)
    wd, xd, bd = (DeviceArray.from_host(mlb, gpu, w), DeviceArray.from_host(mlb, gpu, x),
                  DeviceArray.from_host(mlb, gpu, bias))
    yd = DeviceArray(mlb, gpu, (m, n))
    mlb.call("mlb_f32_linear", gpu, xd.ptr, wd.ptr, m, k, n, bd.ptr, yd.ptr)
    ref = (x.astype(np.float64) @ w.astype(np.float64).T) + bias
    assert_close(yd.download(), ref, 2e-4, f"f32 linear {m}x{k}x{n}")


@pytest.mark.parametrize("m,k,n", [(3, 17, 9), (65, 130, 70), (128, 64, 128)])
def test_f32_matmul(mlb, gpu, oracle, m, k, n):
    a = oracle.normal(m * k, 6, 400 + k, 0.5).reshape(m, k)
    b = oracle.normal(k * n, 6, 500 + k, 0.5).reshape(k, n)
    ad, bd = DeviceArray.from_host(mlb, gpu, a), DeviceArray.from_host(mlb, gpu, b)
    cd = DeviceArray(mlb, gpu, (m, n))
    mlb.call("mlb_f32_matmul", gpu, ad.ptr, bd.ptr, m, k, n, cd.ptr)
    assert_close(cd.download(), a.astype(np.float64) @ b.astype(np.float64), 2e-4, "f32 matmul")
