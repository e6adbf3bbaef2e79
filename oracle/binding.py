"""ctypes binding of the C oracle (oracle/oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py, always as the checker, never as the measured path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
REF_HARNESS = os.path.join(HERE, "_ref", "ref_harness")

F32, Q80, Q40, Q41 = 0, 1, 2, 3
BLOCK_BYTES = {Q80: 34, Q40: 18, Q41: 20}
QTYPE_NAMES = {"q8_0": Q80, "q4_0": Q40, "q4_1": Q41}

T_EMBEDDING, T_FINAL_NORM, T_LM_HEAD, T_ATTN_NORM = 0, 1, 2, 3
T_WQ, T_WK, T_WV, T_BQ, T_BK, T_BV, T_WO = 4, 5, 6, 7, 8, 9, 10
T_FFN_NORM, T_GATE, T_UP, T_DOWN = 11, 12, 13, 14

# Stream ids of oracle/synth.h
STREAM_EMBEDDING, STREAM_LM_HEAD, STREAM_PROMPT = 1, 2, 3
STREAM_X, STREAM_Q, STREAM_K, STREAM_V, STREAM_W = 4, 5, 6, 7, 8
KIND = dict(wq=0, wk=1, wv=2, wo=3, gate=4, up=5, down=6, bq=7, bk=8, bv=9)


def stream_layer(layer: int, kind: int) -> int:
    return ((layer + 1) << 8) | kind


class OrcConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "vocab_size", "dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads",
        "head_dim", "max_seq_len")] + [
        ("rope_theta", ctypes.c_float), ("rms_norm_eps", ctypes.c_float)] + [
        (n, ctypes.c_int) for n in ("rope_neox", "qkv_bias", "tied_embedding", "qtype")]


# Synthetic model configurations (same shapes as oracle/ref_harness.cpp GetSpec).
MODEL_SPECS = {
    "tiny": dict(vocab_size=256, dim=64, hidden_dim=176, n_layers=2, n_heads=4, n_kv_heads=2,
                 head_dim=16, max_seq_len=128, rope_theta=1e4, rms_norm_eps=1e-5, rope_neox=0,
                 qkv_bias=0, tied_embedding=0, qtype=Q80, seed=0, prompt_seed=1),
    "qwen2": dict(vocab_size=151936, dim=896, hidden_dim=4864, n_layers=24, n_heads=14,
                  n_kv_heads=2, head_dim=64, max_seq_len=256, rope_theta=1e6, rms_norm_eps=1e-6,
                  rope_neox=1, qkv_bias=1, tied_embedding=1, qtype=Q80, seed=3, prompt_seed=3),
    "llama2_l2": dict(vocab_size=32000, dim=4096, hidden_dim=11008, n_layers=2, n_heads=32,
                      n_kv_heads=32, head_dim=128, max_seq_len=64, rope_theta=1e4,
                      rms_norm_eps=1e-5, rope_neox=0, qkv_bias=0, tied_embedding=0, qtype=Q40,
                      seed=5, prompt_seed=5),
}


def _fp(a):
    return a.ctypes.data_as(ctypes.c_void_p)


class Oracle:
    def __init__(self, path: str = LIB_PATH):
        if not os.path.exists(path):
            raise RuntimeError(f"oracle library missing: {path} (run make -C oracle oracle)")
        self.lib = ctypes.CDLL(path)
        L = self.lib
        vp, i, f, sz, u64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t, \
            ctypes.c_uint64
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f32_to_f16.argtypes = [f]
        L.orc_f16_to_f32.restype = f
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_quantize.argtypes = [i, vp, i, i, vp]
        L.orc_dequantize.argtypes = [i, vp, i, i, vp]
        L.orc_linear.argtypes = [i, vp, i, i, vp, i, vp, i]
        L.orc_rmsnorm.argtypes = [vp, vp, i, f, vp]
        L.orc_rope_tables.argtypes = [i, i, f, vp, vp]
        L.orc_rope_apply.argtypes = [vp, i, i, i, vp, vp, i]
        L.orc_rope_direct.argtypes = [vp, i, i, i, f, i]
        L.orc_attention.argtypes = [vp, vp, vp, i, i, i, i, i, i, vp, vp]
        L.orc_softmax.argtypes = [vp, i, vp]
        L.orc_silu.argtypes = [vp, i, vp]
        L.orc_swiglu.argtypes = [vp, vp, i, vp]
        L.orc_argmax.argtypes = [vp, i]
        L.orc_argmax.restype = i
        L.orc_model_create_synth.argtypes = [ctypes.POINTER(OrcConfig), u64, i]
        L.orc_model_create_synth.restype = vp
        L.orc_model_free.argtypes = [vp]
        L.orc_model_tensor.argtypes = [vp, i, i, ctypes.POINTER(sz)]
        L.orc_model_tensor.restype = vp
        L.orc_model_reset.argtypes = [vp]
        L.orc_model_forward.argtypes = [vp, i, i, vp]
        L.orc_model_forward.restype = i
        L.orc_synth_normal.argtypes = [vp, sz, u64, u64, ctypes.c_double, i]
        L.orc_synth_tokens.argtypes = [vp, i, u64, i]

    # ---- primitives ----
    def f32_to_f16(self, v: float) -> int:
        return int(self.lib.orc_f32_to_f16(float(v)))

    def f16_to_f32(self, bits: int) -> float:
        return float(self.lib.orc_f16_to_f32(int(bits)))

    def normal(self, n: int, seed: int, stream: int, sigma: float, threads: int = 8) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        self.lib.orc_synth_normal(_fp(out), n, seed, stream, sigma, threads)
        return out

    def tokens(self, n: int, seed: int, vocab: int) -> np.ndarray:
        out = np.empty(n, dtype=np.int32)
        self.lib.orc_synth_tokens(_fp(out), n, seed, vocab)
        return out

    def quantize(self, qtype: int, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.float32)
        rows, cols = (1, w.shape[0]) if w.ndim == 1 else w.shape
        nb = (cols + 31) // 32
        out = np.zeros(rows * nb * BLOCK_BYTES[qtype], dtype=np.uint8)
        self.lib.orc_quantize(qtype, _fp(w), rows, cols, _fp(out))
        return out

    def dequantize(self, qtype: int, blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
        out = np.empty((rows, cols), dtype=np.float32)
        self.lib.orc_dequantize(qtype, _fp(np.ascontiguousarray(blocks)), rows, cols, _fp(out))
        return out

    def linear(self, qtype: int, x: np.ndarray, blocks: np.ndarray, n: int,
               threads: int = 8) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        m, k = (1, x.shape[0]) if x.ndim == 1 else x.shape
        y = np.empty((m, n), dtype=np.float32)
        self.lib.orc_linear(qtype, _fp(x), m, k, _fp(np.ascontiguousarray(blocks)), n, _fp(y),
                            threads)
        return y.reshape(n) if x.ndim == 1 else y

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self.lib.orc_rmsnorm(_fp(x), _fp(np.ascontiguousarray(w, np.float32)), x.size,
                             float(eps), _fp(y))
        return y

    def rope_tables(self, max_seq_len, head_dim, theta):
        half = head_dim // 2
        c = np.empty((max_seq_len, half), np.float32)
        s = np.empty((max_seq_len, half), np.float32)
        self.lib.orc_rope_tables(max_seq_len, head_dim, float(theta), _fp(c), _fp(s))
        return c, s

    def rope(self, x, pos, theta, neox, tables=None):
        x = np.array(x, dtype=np.float32, copy=True)
        rows, hd = x.shape
        if tables is None:
            self.lib.orc_rope_direct(_fp(x), rows, hd, pos, float(theta), int(neox))
        else:
            c, s = tables
            self.lib.orc_rope_apply(_fp(x), rows, hd, pos, _fp(c), _fp(s), int(neox))
        return x

    def attention(self, q, kcache, vcache, layer, pos, n_heads, n_kv_heads, head_dim):
        """kcache/vcache: [n_layers, max_seq_len, n_kv_heads, head_dim] fp32."""
        max_seq_len = kcache.shape[1]
        out = np.empty((n_heads, head_dim), np.float32)
        scratch = np.empty(pos + 1, np.float32)
        self.lib.orc_attention(_fp(np.ascontiguousarray(q, np.float32)),
                               _fp(np.ascontiguousarray(kcache)), _fp(np.ascontiguousarray(vcache)),
                               layer, pos, max_seq_len, n_heads, n_kv_heads, head_dim, _fp(out),
                               _fp(scratch))
        return out

    def softmax(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self.lib.orc_softmax(_fp(x), x.size, _fp(y))
        return y

    def silu(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self.lib.orc_silu(_fp(x), x.size, _fp(y))
        return y

    def swiglu(self, g, u):
        g = np.ascontiguousarray(g, np.float32)
        y = np.empty_like(g)
        self.lib.orc_swiglu(_fp(g), _fp(np.ascontiguousarray(u, np.float32)), g.size, _fp(y))
        return y

    def argmax(self, x):
        x = np.ascontiguousarray(x, np.float32)
        return int(self.lib.orc_argmax(_fp(x), x.size))

    # ---- models ----
    def model(self, name: str, threads: int = 8, **overrides) -> "OracleModel":
        spec = dict(MODEL_SPECS[name])
        spec.update(overrides)
        return OracleModel(self, spec, threads)


class OracleModel:
    def __init__(self, orc: Oracle, spec: dict, threads: int):
        self.orc = orc
        self.spec = spec
        cfg = OrcConfig(**{k: spec[k] for k, _ in OrcConfig._fields_})
        self.cfg = cfg
        self.handle = orc.lib.orc_model_create_synth(ctypes.byref(cfg), spec["seed"], threads)
        if not self.handle:
            raise RuntimeError("orc_model_create_synth failed")

    def close(self):
        if self.handle:
            self.orc.lib.orc_model_free(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    def tensor(self, layer: int, kind: int) -> np.ndarray | None:
        n = ctypes.c_size_t(0)
        p = self.orc.lib.orc_model_tensor(self.handle, layer, kind, ctypes.byref(n))
        if not p or n.value == 0:
            return None
        buf = (ctypes.c_uint8 * n.value).from_address(p)
        return np.frombuffer(buf, dtype=np.uint8).copy()

    def reset(self):
        self.orc.lib.orc_model_reset(self.handle)

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.empty(self.spec["vocab_size"], np.float32)
        rc = self.orc.lib.orc_model_forward(self.handle, int(token), int(pos), _fp(out))
        if rc != 0:
            raise ValueError("orc_model_forward: token or position out of range")
        return out

    def prompt(self, n: int) -> np.ndarray:
        return self.orc.tokens(n, self.spec["prompt_seed"], self.spec["vocab_size"])

    def greedy(self, prompt, n_new):
        """Returns (generated tokens, list of per-step logits)."""
        self.reset()
        tokens = list(int(t) for t in prompt)
        gen, all_logits = [], []
        for step in range(len(prompt) + n_new - 1):
            logits = self.forward(tokens[step], step)
            all_logits.append(logits)
            if step >= len(prompt) - 1:
                nxt = self.orc.argmax(logits)
                gen.append(nxt)
                if len(tokens) == step + 1:
                    tokens.append(nxt)
        return gen, all_logits


def run_ref_bench(model: str, threads: int, prompt_len: int, n_predict: int, steps: int,
                  warmup: int, timeout: float = 900.0):
    """Runs the reference RunBenchmark through oracle/_ref/ref_harness; returns step records."""
    import json
    if not os.path.exists(REF_HARNESS):
        raise RuntimeError(f"reference harness missing: {REF_HARNESS}")
    out = subprocess.run([REF_HARNESS, "bench", model, str(threads), str(prompt_len),
                          str(n_predict), str(steps), str(warmup)], capture_output=True,
                         text=True, timeout=timeout, check=True)
    return [json.loads(line) for line in out.stdout.splitlines() if line.startswith("{")]


def run_ref_decode(model: str, threads: int, prompt_len: int, tokens: int, steps: int, warmup: int,
                   timeout: float = 900.0):
    """The reference's decode loop in timed steps (oracle/_ref/ref_harness
    decode); returns the JSON records."""
    import json
    if not os.path.exists(REF_HARNESS):
        raise RuntimeError(f"reference harness missing: {REF_HARNESS}")
    out = subprocess.run([REF_HARNESS, "decode", model, str(threads), str(prompt_len), str(tokens),
                          str(steps), str(warmup)], capture_output=True, text=True, timeout=timeout,
                         check=True)
    return [json.loads(line) for line in out.stdout.splitlines() if line.startswith("{")]


def load_device_model(model, om) -> None:
    """Copies every tensor of an oracle model (host) into a device model
    (mini_llama_b200.device.Model) through mlb_model_set_weight; test and
    smoke-check input plumbing only."""
    from mini_llama_b200 import capi
    globals_ = [(capi.W_EMBEDDING, T_EMBEDDING), (capi.W_FINAL_NORM, T_FINAL_NORM),
                (capi.W_LM_HEAD, T_LM_HEAD)]
    for k, ok in globals_:
        model.set_weight(-1, k, om.tensor(-1, ok))
    for layer in range(model.spec["n_layers"]):
        for k in range(capi.W_ATTN_NORM, capi.W_DOWN + 1):
            t = om.tensor(layer, k)  # oracle kinds use the same numbering
            if t is not None:
                model.set_weight(layer, k, t)
