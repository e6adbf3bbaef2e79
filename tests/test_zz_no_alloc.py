"""The allocation-free decode attention (mlb_attention_decode_noalloc).

Callers that cannot allocate device memory while decoding (another framework
holds the free memory, or the thread must not take the allocator's locks or
risk the synchronisation a free can cause) use this entry point; its split-K
scratch is a fixed array in the library image.  It must give the same result
as mlb_attention_decode, call after call.  This file is collected last so that
a failure here never hides the other tests; it also passes on its own in a
fresh process.
"""
import numpy as np
import pytest

from mini_llama_b200 import capi
from mini_llama_b200.device import DeviceArray

pytestmark = pytest.mark.gpu

TOL = 1e-4  # the attention tolerance of the other GPU tests


def _case(mlb, dev, oracle, nh, nkv, hd, pos, stream):
    max_seq = pos + 1
    kc = oracle.normal(max_seq * nkv * hd, 4, stream + 1, 1.0).reshape(1, max_seq, nkv, hd)
    vc = oracle.normal(max_seq * nkv * hd, 4, stream + 2, 1.0).reshape(1, max_seq, nkv, hd)
    q = oracle.normal(nh * hd, 4, stream, 1.0).reshape(nh, hd)
    return (DeviceArray.from_host(mlb, dev, q), DeviceArray.from_host(mlb, dev, kc),
            DeviceArray.from_host(mlb, dev, vc), max_seq)


def _run(mlb, dev, name, qd, kd, vd, max_seq, pos, nh, nkv, hd):
    od = DeviceArray(mlb, dev, (nh, hd))
    mlb.call(name, dev, qd.ptr, kd.ptr, vd.ptr, 1, max_seq, 0, pos, nh, nkv, hd, od.ptr)
    return od.download()


def test_noalloc_attention_matches_allocating_entry_point(mlb, gpu, oracle):
    # two calls in a row with different shapes: the second must not see
    # anything the first left in the shared array
    for (nh, nkv, hd, pos, stream) in ((14, 2, 64, 1023, 9100), (32, 8, 128, 8191, 9200)):
        qd, kd, vd, max_seq = _case(mlb, gpu, oracle, nh, nkv, hd, pos, stream)
        got = _run(mlb, gpu, "mlb_attention_decode_noalloc", qd, kd, vd, max_seq, pos, nh, nkv, hd)
        ref = _run(mlb, gpu, "mlb_attention_decode", qd, kd, vd, max_seq, pos, nh, nkv, hd)
        err = np.abs(got.astype(np.float64) - ref) / np.maximum(1.0, np.abs(ref))
        assert np.all(np.isfinite(got)) and float(err.max()) <= TOL, (nh, hd, pos, err.max())


def test_noalloc_attention_rejects_oversized_scratch(mlb, gpu):
    # 64 heads of 256 over 4 KV heads at 32768 positions split into 74 chunks:
    # 64 x 74 x 258 partial floats, more than the array's 1 Mi; the shape
    # check happens before any device work
    q = DeviceArray(mlb, gpu, 64)
    st = mlb.raw("mlb_attention_decode_noalloc", gpu, q.ptr, q.ptr, q.ptr, 1, 32768, 0, 32767,
                 64, 4, 256, q.ptr)
    assert st == capi.MLB_ERR_UNSUPPORTED
    assert "split-K scratch" in mlb.last_error()
