"""Quantized linears for 9 rows and more (prefill batches), which run on the
tcgen05 tensor cores (csrc/tc05.cu), against the oracle's fp32 linear
(the reference CPU algorithm).  Tolerance as for every quantized linear, per
output: |a - e| <= 1e-4 |e| + 2^-20 sum_k |x_k w_k| (tests/test_gpu_kernels.py)."""
import numpy as np
import pytest

from oracle.binding import Q40, Q41, Q80, STREAM_W, STREAM_X
from tests.test_gpu_kernels import (LIN_TOL, QNAME, assert_close, assert_linear_close, bench_blocks, bench_dequant,
                                    linear_gpu, linear_terms)

pytestmark = pytest.mark.gpu

SMALL_SHAPES = [(896, 896), (4864, 896), (896, 4864)]


@pytest.mark.parametrize("qtype", [Q80, Q40, Q41])
@pytest.mark.parametrize("n,k", SMALL_SHAPES)
@pytest.mark.parametrize("m", [16, 64, 512])
def test_prefill_linear_microbench_shapes(mlb, gpu, oracle, qtype, n, k, m):
    blocks = bench_blocks(oracle, qtype, n, k)
    x = oracle.normal(m * k, 2, STREAM_X + 2000 + n + k + m, 1.0).reshape(m, k)
    expect = oracle.linear(qtype, x, blocks, n)
    assert_linear_close(linear_gpu(mlb, gpu, qtype, x, blocks, n), expect,
                        linear_terms(x, bench_dequant(oracle, qtype, n, k)), f"{QNAME[qtype]} [{n},{k}] M={m}")


@pytest.mark.parametrize("qtype", [Q80, Q40, Q41])
@pytest.mark.parametrize("m", [16, 32, 64, 512])
def test_prefill_linear_lm_head(mlb, gpu, oracle, qtype, m):
    """The lm_head shape: 16 and 32 rows on the integer-MMA linear (1187 row
    groups), 64 and more on the tcgen05 kernel; at 512 rows every 16th row is
    checked against the oracle (the full fp32 CPU product is 70 G
    multiply-adds)."""
    n, k = 151936, 896
    blocks = bench_blocks(oracle, qtype, n, k)
    x = oracle.normal(m * k, 2, STREAM_X + 3000 + m, 1.0).reshape(m, k)
    got = linear_gpu(mlb, gpu, qtype, x, blocks, n)
    rows = np.arange(0, m, 16) if m > 64 else np.arange(m)
    expect = oracle.linear(qtype, np.ascontiguousarray(x[rows]), blocks, n)
    assert_linear_close(got[rows], expect, linear_terms(x[rows], bench_dequant(oracle, qtype, n, k)),
                        f"{QNAME[qtype]} lm_head M={m}")


@pytest.mark.parametrize("qtype", [Q80, Q40, Q41])
@pytest.mark.parametrize("m,k,n", [(64, 33, 7), (100, 129, 200), (130, 896, 131), (63, 64, 96), (9, 896, 300),
                                   (8, 64, 96), (37, 4864, 129)])
def test_prefill_linear_ragged_with_bias(mlb, gpu, oracle, qtype, m, k, n):
    """Partial row and column tiles, K not a multiple of 32 or 64, bias; 8
    rows take the GEMV, 9 and more the tensor cores."""
    w = oracle.normal(n * k, 2, STREAM_W + 4000 + n + k, 0.02).reshape(n, k)
    blocks = oracle.quantize(qtype, w)
    x = oracle.normal(m * k, 2, STREAM_X + 4000 + m + k, 1.0).reshape(m, k)
    bias = oracle.normal(n, 2, 4999, 0.1)
    expect = oracle.linear(qtype, x, blocks, n) + bias[None, :]
    assert_linear_close(linear_gpu(mlb, gpu, qtype, x, blocks, n, bias), expect,
                        linear_terms(x, oracle.dequantize(qtype, blocks, n, k), bias), f"{QNAME[qtype]} M={m} K={k} N={n}")


# Shapes for the integer-MMA linear of 9..64 rows (csrc/wide.cu): x rows that
# fill 8-row groups partly (17, 24, 40), block counts not a multiple of a
# stage's four (Q4_1 only with an odd count: Q8_0 / Q4_0 then take the
# tcgen05 kernel), output rows not a multiple of a CTA's 128, weight rows
# viewed 1, 2 or 4 at a time by the tensor map, and N % 4 != 0 with 4 rows per
# view (the per-row bulk-copy fallback), with bias, and the same call twice
# (x's tables rebuilt, the split sums rewritten).
@pytest.mark.parametrize("qtype", [Q80, Q40, Q41])
@pytest.mark.parametrize("m,k,n", [(24, 1024, 262), (40, 896, 262), (17, 800, 262), (64, 96, 1000),
                                   (32, 4864, 384)])
def test_prefill_linear_int_mma_layouts(mlb, gpu, oracle, qtype, m, k, n):
    w = oracle.normal(n * k, 2, STREAM_W + 5000 + n + k, 0.02).reshape(n, k)
    blocks = oracle.quantize(qtype, w)
    x = oracle.normal(m * k, 2, STREAM_X + 5000 + m + k, 1.0).reshape(m, k)
    bias = oracle.normal(n, 2, 5999, 0.1)
    expect = oracle.linear(qtype, x, blocks, n) + bias[None, :]
    terms = linear_terms(x, oracle.dequantize(qtype, blocks, n, k), bias)
    for rep in range(2):
        assert_linear_close(linear_gpu(mlb, gpu, qtype, x, blocks, n, bias), expect, terms,
                            f"{QNAME[qtype]} M={m} K={k} N={n} call {rep}")


def test_prefill_linear_row_scales(mlb, gpu, oracle):
    """Rows of very different magnitude (1e-6 .. 1e4) keep their relative
    accuracy: each x row and W row has its own power-of-two scale."""
    n, k, m = 256, 896, 128
    w = oracle.normal(n * k, 2, STREAM_W + 5000, 0.02).reshape(n, k)
    w[::7] *= 1e-3
    blocks = oracle.quantize(Q80, w)
    x = oracle.normal(m * k, 2, STREAM_X + 5000, 1.0).reshape(m, k)
    x *= np.logspace(-6, 4, m, dtype=np.float64)[:, None].astype(np.float32)
    x = x.astype(np.float32)
    expect = oracle.linear(Q80, x, blocks, n)
    got = linear_gpu(mlb, gpu, Q80, x, blocks, n)
    # relative to each row's own scale
    scale = np.maximum(np.abs(expect).max(axis=1, keepdims=True), 1e-30)
    err = np.abs(got.astype(np.float64) - expect) / scale
    assert float(err.max()) <= 1e-5, float(err.max())


@pytest.mark.parametrize("qtype", [Q80, Q40, Q41])
def test_prefill_linear_large_blocks_rescaled(mlb, gpu, oracle, qtype):
    """Weights around 1e4: block scales whose |w| bound reaches 2^15 would
    overflow fp16 unscaled, so those tiles are recomputed with per-row
    power-of-two scales.  Tolerance 2e-6 of sum_k |x_k w_nk| per output."""
    n, k, m = 300, 896, 96
    w = oracle.normal(n * k, 2, STREAM_W + 6000, 1e4).reshape(n, k)
    blocks = oracle.quantize(qtype, w)
    x = oracle.normal(m * k, 2, STREAM_X + 6000, 1.0).reshape(m, k)
    expect = oracle.linear(qtype, x, blocks, n)
    got = linear_gpu(mlb, gpu, qtype, x, blocks, n).astype(np.float64)
    # error against each output's own scale sum_k |x_k w_nk| (outputs near
    # zero come from cancellation between terms of ~1e4, where any two fp32
    # summation orders differ by ~1e-7 of that sum)
    wd = oracle.dequantize(qtype, blocks, n, k).astype(np.float64)
    scale = np.abs(x.astype(np.float64)) @ np.abs(wd).T
    err = float((np.abs(got - expect) / scale).max())
    assert err <= 2e-6, f"{QNAME[qtype]} |w|~1e4: {err:.3e}"


@pytest.mark.parametrize("qtype", [Q80, Q40, Q41])
def test_prefill_linear_subnormal_halves(mlb, gpu, oracle, qtype):
    """Weights around 1e-4: fp16 block scales and many hi / lo halves are
    subnormal; the products stay exact (relative error against the largest
    output, which is ~1e-3, so the absolute floor of the usual tolerance
    cannot hide a loss)."""
    n, k, m = 256, 896, 64
    w = oracle.normal(n * k, 2, STREAM_W + 7000, 1e-4).reshape(n, k)
    blocks = oracle.quantize(qtype, w)
    x = oracle.normal(m * k, 2, STREAM_X + 7000, 1.0).reshape(m, k)
    expect = oracle.linear(qtype, x, blocks, n)
    got = linear_gpu(mlb, gpu, qtype, x, blocks, n).astype(np.float64)
    scale = float(np.abs(expect).max())
    assert scale > 0
    err = float(np.abs(got - expect).max()) / scale
    assert err <= 1e-5, err
