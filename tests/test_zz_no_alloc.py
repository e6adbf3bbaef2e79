"""The allocation-free decode attention (mlb_attention_decode_noalloc).

Callers that cannot allocate device memory while decoding (another framework
holds the free memory, or the thread must not take the allocator's locks or
risk the synchronisation a free can cause) use this entry point; its split-K
scratch is a fixed array in the library image.  It must give the same result
as mlb_attention_decode (and the oracle), call after call, without taking any
device memory.  This file is collected last so that a failure here never
hides the other tests; it also passes on its own in a fresh process.
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
    return q, kc, vc, max_seq


def _run(mlb, dev, name, qd, kd, vd, max_seq, pos, nh, nkv, hd):
    od = DeviceArray(mlb, dev, (nh, hd))
    mlb.call(name, dev, qd.ptr, kd.ptr, vd.ptr, 1, max_seq, 0, pos, nh, nkv, hd, od.ptr)
    return od.download()


def _free_bytes(dev):
    import torch
    torch.cuda.synchronize(dev)
    return torch.cuda.mem_get_info(dev)[0]


def test_noalloc_attention_matches_allocating_entry_point(mlb, gpu, oracle):
    # two calls in a row with different shapes: the second must not see
    # anything the first left in the shared array
    cases = ((14, 2, 64, 1023, 9100), (32, 8, 128, 8191, 9200))
    inputs = []
    for (nh, nkv, hd, pos, stream) in cases:
        q, kc, vc, max_seq = _case(mlb, gpu, oracle, nh, nkv, hd, pos, stream)
        inputs.append((q, kc, vc, max_seq, DeviceArray.from_host(mlb, gpu, q),
                       DeviceArray.from_host(mlb, gpu, kc), DeviceArray.from_host(mlb, gpu, vc)))
    # the first call sets the entry point up on this device (the array's
    # device address); every later call must leave device memory untouched
    q, kc, vc, max_seq, qd, kd, vd = inputs[0]
    nh, nkv, hd, pos, _ = cases[0]
    _run(mlb, gpu, "mlb_attention_decode_noalloc", qd, kd, vd, max_seq, pos, nh, nkv, hd)
    got = []
    free0 = _free_bytes(gpu)
    for (nh, nkv, hd, pos, _), (q, kc, vc, max_seq, qd, kd, vd) in zip(cases, inputs):
        got.append(_run(mlb, gpu, "mlb_attention_decode_noalloc", qd, kd, vd, max_seq, pos, nh, nkv, hd))
    assert _free_bytes(gpu) == free0, "the allocation-free entry point took device memory"
    for (nh, nkv, hd, pos, _), (q, kc, vc, max_seq, qd, kd, vd), a in zip(cases, inputs, got):
        ref = _run(mlb, gpu, "mlb_attention_decode", qd, kd, vd, max_seq, pos, nh, nkv, hd)
        orc = oracle.attention(q, kc, vc, 0, pos, nh, nkv, hd)
        for name, e in (("mlb_attention_decode", ref), ("oracle", orc)):
            err = np.abs(a.astype(np.float64) - e) / np.maximum(1.0, np.abs(e))
            assert np.all(np.isfinite(a)) and float(err.max()) <= TOL, (name, nh, hd, pos, err.max())


def test_noalloc_attention_rejects_oversized_scratch(mlb, gpu):
    # 64 heads of 256 over 4 KV heads at 32768 positions: on a B200 the split
    # needs more partial floats than the array's 1 Mi, so the call must fail
    # before any device work.  The buffers are sized to the full shape, so
    # even a planner that fits this shape on some other part launches nothing
    # out of bounds (the call then succeeds instead).
    nh, nkv, hd, max_seq = 64, 4, 256, 32768
    q = DeviceArray(mlb, gpu, nh * hd)
    kc = DeviceArray(mlb, gpu, max_seq * nkv * hd)
    vc = DeviceArray(mlb, gpu, max_seq * nkv * hd)
    out = DeviceArray(mlb, gpu, nh * hd)
    for buf in (q, kc, vc):
        mlb.call("mlb_memset", gpu, buf.ptr, 0, buf.nbytes)
    sms = mlb.device_info(gpu).sm_count
    st = mlb.raw("mlb_attention_decode_noalloc", gpu, q.ptr, kc.ptr, vc.ptr, 1, max_seq, 0, max_seq - 1,
                 nh, nkv, hd, out.ptr)
    msg = mlb.last_error()  # before any other call replaces it
    if sms >= 100:
        assert st == capi.MLB_ERR_UNSUPPORTED
        assert "split-K scratch" in msg
    else:
        assert st in (capi.MLB_OK, capi.MLB_ERR_UNSUPPORTED)
