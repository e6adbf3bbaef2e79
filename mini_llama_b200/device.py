"""Device arrays and a decode-session wrapper over the C ABI (test/bench plumbing)."""
from __future__ import annotations

import ctypes

import numpy as np

from . import capi


class DeviceArray:
    """A device allocation from the library pool holding a numpy-typed array."""

    def __init__(self, lib: capi.Lib, device: int, shape, dtype=np.float32):
        self.lib, self.device = lib, device
        self.shape = tuple(int(s) for s in (shape if isinstance(shape, (tuple, list)) else (shape,)))
        self.dtype = np.dtype(dtype)
        self.nbytes = int(np.prod(self.shape, dtype=np.int64)) * self.dtype.itemsize
        self.ptr = lib.malloc(device, max(self.nbytes, 1))

    @classmethod
    def from_host(cls, lib, device, array: np.ndarray) -> "DeviceArray":
        a = np.ascontiguousarray(array)
        d = cls(lib, device, a.shape, a.dtype)
        d.upload(a)
        return d

    def upload(self, array: np.ndarray):
        a = np.ascontiguousarray(array, dtype=self.dtype)
        assert a.nbytes == self.nbytes
        self.lib.call("mlb_memcpy_h2d", self.device, self.ptr, a.ctypes.data, self.nbytes)

    def download(self) -> np.ndarray:
        out = np.empty(self.shape, dtype=self.dtype)
        self.lib.call("mlb_memcpy_d2h", self.device, out.ctypes.data, self.ptr, self.nbytes)
        return out

    def free(self):
        if self.ptr:
            self.lib.free(self.device, self.ptr)
            self.ptr = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def model_config(spec: dict) -> capi.ModelConfig:
    """mlb_model_config from a synthetic model spec (keys of oracle MODEL_SPECS)."""
    return capi.ModelConfig(
        vocab_size=spec["vocab_size"], dim=spec["dim"], hidden_dim=spec["hidden_dim"],
        n_layers=spec["n_layers"], n_heads=spec["n_heads"], n_kv_heads=spec["n_kv_heads"],
        head_dim=spec["head_dim"], max_seq_len=spec["max_seq_len"],
        rope_theta=spec["rope_theta"], rms_norm_eps=spec["rms_norm_eps"],
        rope_type=capi.ROPE_NEOX if spec["rope_neox"] else capi.ROPE_NORMAL,
        weight_type=spec["qtype"], qkv_bias=spec["qkv_bias"])


# Stream ids of the synthetic generator (oracle/synth.h): layer tensors use
# ((layer + 1) << 8) | kind.
_SYNTH_KIND = {capi.W_WQ: 0, capi.W_WK: 1, capi.W_WV: 2, capi.W_WO: 3, capi.W_GATE: 4,
               capi.W_UP: 5, capi.W_DOWN: 6, capi.W_BQ: 7, capi.W_BK: 8, capi.W_BV: 9}
_STREAM_EMBEDDING, _STREAM_LM_HEAD = 1, 2


class Model:
    """A model on the device (mlb_model) with its weights."""

    def __init__(self, lib: capi.Lib, device: int, spec: dict):
        self.lib, self.device, self.spec = lib, device, spec
        self.cfg = model_config(spec)
        h = ctypes.c_void_p()
        lib.call("mlb_model_create", device, ctypes.byref(self.cfg), ctypes.byref(h))
        self.handle = h.value

    def weight(self, layer: int, kind: int):
        p, n = ctypes.c_void_p(), ctypes.c_size_t()
        self.lib.call("mlb_model_weight", self.handle, layer, kind, ctypes.byref(p), ctypes.byref(n))
        return p.value or 0, n.value

    def set_weight(self, layer: int, kind: int, data: np.ndarray):
        a = np.ascontiguousarray(data)
        self.lib.call("mlb_model_set_weight", self.handle, layer, kind, a.ctypes.data, a.nbytes, 1)

    def synthesize(self, seed: int, tied: bool):
        """Generates the synthetic weights on the device: N(0, 0.02) linears
        quantized by the device quantizer, norms = 1, as the oracle does."""
        s = self.spec
        qd, kd = s["n_heads"] * s["head_dim"], s["n_kv_heads"] * s["head_dim"]
        D, F, V = s["dim"], s["hidden_dim"], s["vocab_size"]
        shapes = {capi.W_WQ: (qd, D), capi.W_WK: (kd, D), capi.W_WV: (kd, D),
                  capi.W_WO: (D, qd), capi.W_GATE: (F, D), capi.W_UP: (F, D),
                  capi.W_DOWN: (D, F)}
        scratch = self.lib.malloc(self.device, 4 * max(V * D, F * D, qd * D))
        try:
            emb, _ = self.weight(-1, capi.W_EMBEDDING)
            self.lib.call("mlb_synth_normal", self.device, emb, V * D, seed, _STREAM_EMBEDDING, 0.02)
            lm, _ = self.weight(-1, capi.W_LM_HEAD)
            if tied:
                self.lib.call("mlb_quantize", self.device, s["qtype"], emb, V, D, lm)
            else:
                self.lib.call("mlb_synth_normal", self.device, scratch, V * D, seed,
                              _STREAM_LM_HEAD, 0.02)
                self.lib.call("mlb_quantize", self.device, s["qtype"], scratch, V, D, lm)
            ones = np.ones(D, np.float32)
            self.set_weight(-1, capi.W_FINAL_NORM, ones)
            for l in range(s["n_layers"]):
                self.set_weight(l, capi.W_ATTN_NORM, ones)
                self.set_weight(l, capi.W_FFN_NORM, ones)
                for kind, (r, c) in shapes.items():
                    dst, _ = self.weight(l, kind)
                    stream = ((l + 1) << 8) | _SYNTH_KIND[kind]
                    self.lib.call("mlb_synth_normal", self.device, scratch, r * c, seed, stream, 0.02)
                    self.lib.call("mlb_quantize", self.device, s["qtype"], scratch, r, c, dst)
                if s["qkv_bias"]:
                    for kind, n in ((capi.W_BQ, qd), (capi.W_BK, kd), (capi.W_BV, kd)):
                        dst, _ = self.weight(l, kind)
                        stream = ((l + 1) << 8) | _SYNTH_KIND[kind]
                        self.lib.call("mlb_synth_normal", self.device, dst, n, seed, stream, 0.02)
            self.lib.sync(self.device)
        finally:
            self.lib.free(self.device, scratch)

    def bytes(self) -> int:
        n = ctypes.c_size_t()
        self.lib.call("mlb_model_bytes", self.handle, ctypes.byref(n))
        return n.value

    def close(self):
        if self.handle:
            self.lib.call("mlb_model_destroy", self.handle)
            self.handle = None


class Session:
    def __init__(self, model: Model):
        self.model, self.lib = model, model.lib
        h = ctypes.c_void_p()
        self.lib.call("mlb_session_create", model.handle, ctypes.byref(h))
        self.handle = h.value

    def reset(self):
        self.lib.call("mlb_session_reset", self.handle)

    def forward(self, token: int, pos: int, want_logits: bool = True):
        logits = np.empty(self.model.spec["vocab_size"], np.float32) if want_logits else None
        nxt = ctypes.c_int(-1)
        self.lib.call("mlb_session_forward", self.handle, int(token), int(pos),
                      logits.ctypes.data if want_logits else None, ctypes.byref(nxt))
        return logits, nxt.value

    def generate(self, prompt, n_new: int, start_pos: int = 0) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(n_new, np.int32)
        self.lib.call("mlb_session_generate", self.handle, p.ctypes.data, len(p), start_pos, n_new,
                      out.ctypes.data)
        return out

    def decode_device(self, tokens_ptr: int, start_pos: int, n_steps: int):
        self.lib.call("mlb_session_decode_device", self.handle, tokens_ptr, start_pos, n_steps)

    def path(self) -> int:
        """2 persistent kernel, 1 graph with integer-MMA GEMV, 0 graph with SIMT GEMV."""
        v = ctypes.c_int(-1)
        self.lib.call("mlb_session_gemv_path", self.handle, ctypes.byref(v))
        return v.value

    def use_persistent(self, enable: bool):
        self.lib.call("mlb_session_use_persistent", self.handle, 1 if enable else 0)

    def prefill_min(self, min_tokens: int):
        """Prompts of at least min_tokens tokens take the one-pass prompt path (0: never)."""
        self.lib.call("mlb_session_prefill_min", self.handle, int(min_tokens))

    def logits_ptr(self) -> int:
        p = ctypes.c_void_p()
        self.lib.call("mlb_session_logits", self.handle, ctypes.byref(p))
        return p.value

    def close(self):
        if self.handle:
            self.lib.call("mlb_session_destroy", self.handle)
            self.handle = None


def nccl_unique_id(lib: capi.Lib) -> bytes:
    """A fresh NCCL id for one tensor-parallel group (mlb_nccl_unique_id)."""
    buf = (ctypes.c_char * capi.NCCL_ID_BYTES)()
    lib.call("mlb_nccl_unique_id", buf)
    return bytes(buf)


def batch_shard(lib: capi.Lib, spec: dict, tp_rank: int, tp_size: int) -> dict:
    """The slices a tensor-parallel rank owns (mlb_batch_shard), as half-open
    (begin, end) pairs: q heads, KV heads, dim rows, hidden rows, vocab rows."""
    cfg = model_config(spec)
    r = (ctypes.c_int * 10)()
    lib.call("mlb_batch_shard", ctypes.byref(cfg), tp_rank, tp_size, r)
    v = list(r)
    return {"heads": (v[0], v[1]), "kv_heads": (v[2], v[3]), "dim": (v[4], v[5]),
            "hidden": (v[6], v[7]), "vocab": (v[8], v[9])}


class BatchSession:
    """Lockstep greedy decoding of `batch` sequences (mlb_batch), optionally
    tensor-parallel: every rank passes the same NCCL id (nccl_unique_id on one
    rank, shared by the caller) and its own rank."""

    def __init__(self, model: Model, batch: int, tp_rank: int = 0, tp_size: int = 1,
                 nccl_id: bytes | None = None):
        self.model, self.lib, self.batch = model, model.lib, batch
        h = ctypes.c_void_p()
        idbuf = ctypes.create_string_buffer(nccl_id, capi.NCCL_ID_BYTES) if nccl_id else None
        self.lib.call("mlb_batch_create", model.handle, batch, tp_rank, tp_size, idbuf, ctypes.byref(h))
        self.handle = h.value

    def generate(self, prompts, n_new: int):
        """prompts [batch, n_prompt] -> (tokens [batch, n_new], prefill_ms, decode_ms)."""
        p = np.ascontiguousarray(prompts, dtype=np.int32)
        assert p.ndim == 2 and p.shape[0] == self.batch
        out = np.empty((self.batch, n_new), np.int32)
        pre, dec = ctypes.c_float(), ctypes.c_float()
        self.lib.call("mlb_batch_generate", self.handle, p.ctypes.data, p.shape[1], n_new, out.ctypes.data,
                      ctypes.byref(pre), ctypes.byref(dec))
        return out, pre.value, dec.value

    def logits(self) -> np.ndarray:
        """This rank's logits slice of the last step, [batch, cols]."""
        ptr, cols, col0 = ctypes.c_void_p(), ctypes.c_int(), ctypes.c_int()
        self.lib.call("mlb_batch_logits", self.handle, ctypes.byref(ptr), ctypes.byref(cols), ctypes.byref(col0))
        out = np.empty((self.batch, cols.value), np.float32)
        self.lib.call("mlb_memcpy_d2h", self.model.device, out.ctypes.data, ptr.value, out.nbytes)
        return out

    def close(self):
        if self.handle:
            self.lib.call("mlb_batch_destroy", self.handle)
            self.handle = None
