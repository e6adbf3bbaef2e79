"""ctypes binding of the mini_llama_b200 C ABI (include/mlb.h).

This is plumbing for tests and benchmarks; the product is the shared library
mini_llama_b200/_build/libmlb.so.  Loading fails loudly when the library is
missing: there is no CPU or Python fallback for any entry point.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libmlb.so")

MLB_OK = 0
MLB_ERR_INVALID_ARGUMENT = 1
MLB_ERR_OUT_OF_RANGE = 2
MLB_ERR_CUDA = 3
MLB_ERR_UNSUPPORTED = 4
MLB_ERR_DEVICE_TIMEOUT = 5

F32, Q8_0, Q4_0, Q4_1 = 0, 1, 2, 3
ROPE_NORMAL, ROPE_NEOX = 0, 1

W_EMBEDDING, W_FINAL_NORM, W_LM_HEAD, W_ATTN_NORM = 0, 1, 2, 3
W_WQ, W_WK, W_WV, W_BQ, W_BK, W_BV, W_WO = 4, 5, 6, 7, 8, 9, 10
W_FFN_NORM, W_GATE, W_UP, W_DOWN = 11, 12, 13, 14

# Every symbol include/mlb.h declares, with (restype, argtypes).
_vp, _i, _f, _sz, _u64, _d = (ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t,
                              ctypes.c_uint64, ctypes.c_double)
_pp = ctypes.POINTER(ctypes.c_void_p)
_pi = ctypes.POINTER(ctypes.c_int)
_psz = ctypes.POINTER(ctypes.c_size_t)


class DeviceInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 256), ("compute_major", ctypes.c_int),
                ("compute_minor", ctypes.c_int), ("total_memory_bytes", ctypes.c_size_t),
                ("sm_count", ctypes.c_int), ("driver_version", ctypes.c_int),
                ("runtime_version", ctypes.c_int)]


class ModelConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "vocab_size", "dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "head_dim",
        "max_seq_len")] + [("rope_theta", ctypes.c_float), ("rms_norm_eps", ctypes.c_float)] + [
        (n, ctypes.c_int) for n in ("rope_type", "weight_type", "qkv_bias")]


SIGNATURES = {
    "mlb_last_error": (ctypes.c_char_p, []),
    "mlb_abi_version": (_i, []),
    "mlb_device_count": (_i, [_pi]),
    "mlb_set_device": (_i, [_i]),
    "mlb_get_device_info": (_i, [_i, ctypes.POINTER(DeviceInfo)]),
    "mlb_get_stream": (_i, [_i, _pp]),
    "mlb_malloc": (_i, [_i, _sz, _pp]),
    "mlb_free": (_i, [_i, _vp]),
    "mlb_memcpy_h2d": (_i, [_i, _vp, _vp, _sz]),
    "mlb_memcpy_d2h": (_i, [_i, _vp, _vp, _sz]),
    "mlb_memcpy_d2d": (_i, [_i, _vp, _vp, _sz]),
    "mlb_memset": (_i, [_i, _vp, _i, _sz]),
    "mlb_synchronize": (_i, [_i]),
    "mlb_q80_linear": (_i, [_i, _vp, _vp, _sz, _i, _i, _i, _vp, _vp]),
    "mlb_q40_linear": (_i, [_i, _vp, _vp, _sz, _i, _i, _i, _vp, _vp]),
    "mlb_q41_linear": (_i, [_i, _vp, _vp, _sz, _i, _i, _i, _vp, _vp]),
    "mlb_quant_linear": (_i, [_i, _i, _vp, _vp, _sz, _i, _i, _i, _vp, _vp]),
    "mlb_f32_linear": (_i, [_i, _vp, _vp, _i, _i, _i, _vp, _vp]),
    "mlb_f32_matmul": (_i, [_i, _vp, _vp, _i, _i, _i, _vp]),
    "mlb_r16_bytes": (_sz, [_i, _i]),
    "mlb_q80_repack_r16": (_i, [_i, _vp, _i, _i, _vp]),
    "mlb_q80_linear_r16": (_i, [_i, _vp, _vp, _i, _i, _i, _vp, _vp]),
    "mlb_quantize": (_i, [_i, _i, _vp, _i, _i, _vp]),
    "mlb_dequantize": (_i, [_i, _i, _vp, _i, _i, _vp]),
    "mlb_rmsnorm": (_i, [_i, _vp, _vp, _i, _f, _vp]),
    "mlb_rope": (_i, [_i, _vp, _vp, _i, _i, _i, _i, _f, _i]),
    "mlb_silu": (_i, [_i, _vp, _sz, _vp]),
    "mlb_mul": (_i, [_i, _vp, _vp, _sz, _vp]),
    "mlb_add": (_i, [_i, _vp, _vp, _sz, _vp]),
    "mlb_softmax": (_i, [_i, _vp, _i, _vp]),
    "mlb_embedding": (_i, [_i, _vp, _i, _i, _i, _vp]),
    "mlb_argmax": (_i, [_i, _vp, _i, _vp]),
    "mlb_kv_write": (_i, [_i, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp]),
    "mlb_attention_decode": (_i, [_i, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "mlb_attention_decode_batched": (_i, [_i, _i, _vp, _vp, _vp, _i, _i, _i, _vp, _i, _i, _i,
                                          _i, _vp]),
    "mlb_attention_decode_noalloc": (_i, [_i, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "mlb_synth_normal": (_i, [_i, _vp, _sz, _u64, _u64, _d]),
    "mlb_model_create": (_i, [_i, ctypes.POINTER(ModelConfig), _pp]),
    "mlb_model_destroy": (_i, [_vp]),
    "mlb_model_weight": (_i, [_vp, _i, _i, _pp, _psz]),
    "mlb_model_set_weight": (_i, [_vp, _i, _i, _vp, _sz, _i]),
    "mlb_model_bytes": (_i, [_vp, _psz]),
    "mlb_session_create": (_i, [_vp, _pp]),
    "mlb_session_destroy": (_i, [_vp]),
    "mlb_session_reset": (_i, [_vp]),
    "mlb_session_forward": (_i, [_vp, _i, _i, _vp, _pi]),
    "mlb_session_generate": (_i, [_vp, _vp, _i, _i, _i, _vp]),
    "mlb_session_decode_device": (_i, [_vp, _vp, _i, _i]),
    "mlb_session_logits": (_i, [_vp, _pp]),
    "mlb_session_gemv_path": (_i, [_vp, _pi]),
    "mlb_session_use_persistent": (_i, [_vp, _i]),
    "mlb_session_trace": (_i, [_vp, _vp, _sz]),
    "mlb_session_wait_limit": (_i, [_vp, ctypes.c_ulonglong]),
    "mlb_session_test_withhold_signal": (_i, [_vp, _i]),
    "mlb_session_kv_cache": (_i, [_vp, _pp, _pp]),
    "mlb_session_prefill_min": (_i, [_vp, _i]),
    "mlb_nccl_unique_id": (_i, [_vp]),
    "mlb_batch_shard": (_i, [ctypes.POINTER(ModelConfig), _i, _i, _pi]),
    "mlb_batch_create": (_i, [_vp, _i, _i, _i, _vp, _pp]),
    "mlb_batch_destroy": (_i, [_vp]),
    "mlb_batch_generate": (_i, [_vp, _vp, _i, _i, _vp, ctypes.POINTER(ctypes.c_float),
                                ctypes.POINTER(ctypes.c_float)]),
    "mlb_batch_logits": (_i, [_vp, _pp, _pi, _pi]),
}

NCCL_ID_BYTES = 128


class MlbError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


class Lib:
    """Thin checked wrapper: every call raises MlbError on a nonzero status."""

    def __init__(self, path: str = LIB_PATH):
        if not os.path.exists(path):
            raise RuntimeError(f"mini_llama_b200 CUDA library missing: {path} "
                               "(build it with python -m mini_llama_b200.build)")
        self.path = path
        self.dll = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(self.dll, name)
            fn.restype = res
            fn.argtypes = args

    def _check(self, status: int):
        if status != MLB_OK:
            raise MlbError(status, self.dll.mlb_last_error().decode())

    def call(self, name: str, *args):
        self._check(getattr(self.dll, name)(*args))

    def raw(self, name: str, *args) -> int:
        """Call returning the status instead of raising (for error-path tests)."""
        return getattr(self.dll, name)(*args)

    def last_error(self) -> str:
        return self.dll.mlb_last_error().decode()

    # ---- runtime helpers ----
    def device_count(self) -> int:
        n = ctypes.c_int(0)
        self.call("mlb_device_count", ctypes.byref(n))
        return n.value

    def device_info(self, device: int = 0) -> DeviceInfo:
        info = DeviceInfo()
        self.call("mlb_get_device_info", device, ctypes.byref(info))
        return info

    def stream(self, device: int = 0) -> int:
        s = ctypes.c_void_p()
        self.call("mlb_get_stream", device, ctypes.byref(s))
        return s.value or 0

    def malloc(self, device: int, nbytes: int) -> int:
        p = ctypes.c_void_p()
        self.call("mlb_malloc", device, nbytes, ctypes.byref(p))
        return p.value or 0

    def free(self, device: int, ptr: int):
        self.call("mlb_free", device, ptr)

    def sync(self, device: int = 0):
        self.call("mlb_synchronize", device)


_LIB = None


def load(path: str = LIB_PATH) -> Lib:
    global _LIB
    if _LIB is None or _LIB.path != path:
        _LIB = Lib(path)
    return _LIB
