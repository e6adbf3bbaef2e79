"""CPU-side checks of the C ABI: the CUDA library loads here (no GPU needed to
load it) and exports every entry point include/mlb.h declares, with the
signatures the Python binding uses.  No compute call is made."""
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "mlb.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mlb_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib_path():
    from mini_llama_b200 import build
    return build.build()


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "mlb_q80_linear" in syms and "mlb_attention_decode" in syms
    assert len(syms) >= 40


def test_library_exports_every_declared_symbol(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (mlb_[a-z0-9_]+)$", out, flags=re.M))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_covers_header(lib_path):
    from mini_llama_b200 import capi
    assert sorted(capi.SIGNATURES) == declared_symbols()
    lib = capi.load(lib_path)
    assert lib.dll.mlb_abi_version() == 1


def test_no_device_reports_cleanly(lib_path):
    """On a host without a GPU the library loads and reports zero devices;
    a device call then fails with a status, not a crash."""
    from mini_llama_b200 import capi
    lib = capi.load(lib_path)
    if lib.device_count() > 0:
        pytest.skip("a GPU is visible")
    import ctypes
    p = ctypes.c_void_p()
    status = lib.raw("mlb_malloc", 0, 16, ctypes.byref(p))
    assert status != capi.MLB_OK
    assert "device" in lib.last_error().lower() or "cuda" in lib.last_error().lower()


def test_null_argument_errors_without_device(lib_path):
    from mini_llama_b200 import capi
    lib = capi.load(lib_path)
    assert lib.raw("mlb_device_count", None) == capi.MLB_ERR_INVALID_ARGUMENT
    assert "null" in lib.last_error()


def test_timeline_summary_of_synthetic_stamps():
    """The phase-timeline summary (host side of mlb_session_trace) on hand-made
    stamps: one layer, two CTAs, phases 1 us apart."""
    import numpy as np
    from mini_llama_b200 import timeline
    steps, L, E, G = 3, 1, timeline.EVENTS, 2
    t = np.zeros((steps, L + 1, E, G), np.int64)
    for st in range(steps):
        base = 100000 * (st + 1)
        for ev, us in ((0, 0), (11, 1), (10, 2), (1, 3), (2, 4), (8, 5), (9, 6), (3, 7),
                       (4, 8), (7, 9), (6, 10), (5, 13)):
            t[st, 0, ev, :] = base + 1000 * us
        t[st, 0, 1, 1] = base + 3500  # the second CTA signals QKV later
        t[st, 1, 0, :] = base + 14000
        t[st, 1, 1, :] = base + 20000
    out = timeline.summarise(t)
    assert out["span_us"]["qkv"] == 3.5
    assert out["handover_us"]["qkv_to_att"] == 0.5
    assert out["span_us"]["ffn"] == 5.0
    assert out["handover_us"]["ffn_to_next"] == 1.0  # last layer: to the lm_head wait
    assert out["per_cta_us"]["ffn_products"] == 1.0
    assert out["span_us"]["lm_head"] == 6.0
    assert out["span_us"]["step"] == 100.0
    assert out["per_cta_us"]["att_softmax_v"] == 1.0
