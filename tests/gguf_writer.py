"""Test fixture writer: a small random model as a GGUF v3 file, in the tensor
names, metadata keys and shape order that the reference loader reads
(src/gguf_loader.cpp:25-83 names, :90-104 shape order, :257-286 metadata;
src/gguf.cpp:380-520 header, tensor infos and the aligned data section).

GGUF v3 layout written here: "GGUF", version 3 (u32), tensor count and
metadata count (u64); metadata as (string key, u32 type, value); tensor infos
as (string name, u32 n_dims, u64 ne[n_dims] with ne[0] the row length, u32
ggml type, u64 offset into the data section); zero padding to the alignment
(32); the tensors, each at an aligned offset.  Strings are a u64 length and
the bytes.  Block encodings: Q8_0 = fp16 d + 32 int8 (w = d q); Q4_0 = fp16 d
+ 16 bytes, element j in the low nibble of byte j, element j + 16 in the high
nibble (w = d (q - 8)); Q4_1 = fp16 d, fp16 m + 16 bytes (w = d q + m).
"""
from __future__ import annotations

import struct

import numpy as np

GGML_F32, GGML_Q4_0, GGML_Q4_1, GGML_Q8_0 = 0, 2, 3, 8
_T_U32, _T_F32, _T_STRING, _T_ARRAY = 4, 6, 8, 9
ALIGN = 32


def _s(text: str) -> bytes:
    b = text.encode()
    return struct.pack("<Q", len(b)) + b


def _blocks(w: np.ndarray) -> np.ndarray:
    rows, cols = w.shape
    assert cols % 32 == 0
    return w.astype(np.float32).reshape(rows * cols // 32, 32)


def quantize(w: np.ndarray, ggml_type: int) -> bytes:
    """Row-major blocks of 32 along each row (the row is ne[0])."""
    if ggml_type == GGML_F32:
        return np.ascontiguousarray(w, dtype="<f4").tobytes()
    b = _blocks(w)
    if ggml_type == GGML_Q8_0:
        d = np.abs(b).max(axis=1) / 127.0
        d16 = d.astype(np.float16)
        inv = np.where(d16 > 0, 1.0 / np.maximum(d16.astype(np.float32), 1e-30), 0.0)
        q = np.clip(np.rint(b * inv[:, None]), -127, 127).astype(np.int8)
        out = np.zeros(len(b), dtype=[("d", "<f2"), ("q", "i1", 32)])
        out["d"], out["q"] = d16, q
        return out.tobytes()
    if ggml_type == GGML_Q4_0:
        d16 = (np.abs(b).max(axis=1) / 7.0).astype(np.float16)
        inv = np.where(d16 > 0, 1.0 / np.maximum(d16.astype(np.float32), 1e-30), 0.0)
        q = np.clip(np.rint(b * inv[:, None]) + 8, 0, 15).astype(np.uint8)
        out = np.zeros(len(b), dtype=[("d", "<f2"), ("q", "u1", 16)])
        out["d"], out["q"] = d16, q[:, :16] | (q[:, 16:] << 4)
        return out.tobytes()
    if ggml_type == GGML_Q4_1:
        mn, mx = b.min(axis=1), b.max(axis=1)
        d16, m16 = ((mx - mn) / 15.0).astype(np.float16), mn.astype(np.float16)
        inv = np.where(d16 > 0, 1.0 / np.maximum(d16.astype(np.float32), 1e-30), 0.0)
        q = np.clip(np.rint((b - m16.astype(np.float32)[:, None]) * inv[:, None]), 0, 15).astype(np.uint8)
        out = np.zeros(len(b), dtype=[("d", "<f2"), ("m", "<f2"), ("q", "u1", 16)])
        out["d"], out["m"], out["q"] = d16, m16, q[:, :16] | (q[:, 16:] << 4)
        return out.tobytes()
    raise ValueError(f"ggml type {ggml_type}")


def write_gguf(path: str, arch: str, meta: dict, tensors: list) -> None:
    """tensors: (name, array [rows, cols] or [n], ggml type)."""
    kv = [("general.architecture", _T_STRING, arch), ("general.alignment", _T_U32, ALIGN)]
    for k, v in meta.items():
        if k != "vocab":
            kv.append((f"{arch}.{k}", _T_F32 if isinstance(v, float) else _T_U32, v))
    kv.append(("tokenizer.ggml.tokens", _T_ARRAY, [f"<t{i}>" for i in range(meta["vocab"])]))
    head = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv)))
    for key, t, v in kv:
        head += _s(key) + struct.pack("<I", t)
        if t == _T_STRING:
            head += _s(v)
        elif t == _T_U32:
            head += struct.pack("<I", v)
        elif t == _T_F32:
            head += struct.pack("<f", v)
        else:
            head += struct.pack("<IQ", _T_STRING, len(v)) + b"".join(_s(x) for x in v)
    blobs, offset = [], 0
    for name, arr, gt in tensors:
        data = quantize(arr if arr.ndim == 2 else arr.reshape(1, -1), gt)
        ne = [arr.shape[-1]] + ([arr.shape[0]] if arr.ndim == 2 else [])
        head += _s(name) + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}Q", *ne)
        head += struct.pack("<IQ", gt, offset)
        pad = (-len(data)) % ALIGN
        blobs.append(data + b"\0" * pad)
        offset += len(data) + pad
    head += b"\0" * ((-len(head)) % ALIGN)
    with open(path, "wb") as f:
        f.write(bytes(head))
        for b in blobs:
            f.write(b)


def random_model(path: str, arch: str, *, dim: int, hidden: int, layers: int, heads: int, kv_heads: int,
                 vocab: int, ctx: int, theta: float, eps: float, types: dict, seed: int,
                 biases: bool = False, tied: bool = True, sigma: float = 0.02) -> None:
    """A random model (embedding N(0, 0.02), layer weights N(0, sigma), norms
    1 + N(0, 0.1)) in `path`.
    types maps attn / ffn / embd / output to ggml types; tied leaves output.weight
    out (the loader then uses the embedding as an F32 lm_head)."""
    rng = np.random.default_rng(seed)
    hd = dim // heads
    w = lambda r, c, sd=sigma: (rng.standard_normal((r, c)) * sd).astype(np.float32)  # noqa: E731
    norm = lambda n: (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)  # noqa: E731
    t = [("token_embd.weight", w(vocab, dim, 0.02), types.get("embd", GGML_F32))]
    for l in range(layers):
        p = f"blk.{l}."
        t += [(p + "attn_norm.weight", norm(dim), GGML_F32),
              (p + "attn_q.weight", w(heads * hd, dim), types["attn"]),
              (p + "attn_k.weight", w(kv_heads * hd, dim), types["attn"]),
              (p + "attn_v.weight", w(kv_heads * hd, dim), types["attn"])]
        if biases:
            t += [(p + "attn_q.bias", w(1, heads * hd)[0], GGML_F32),
                  (p + "attn_k.bias", w(1, kv_heads * hd)[0], GGML_F32),
                  (p + "attn_v.bias", w(1, kv_heads * hd)[0], GGML_F32)]
        t += [(p + "attn_output.weight", w(dim, heads * hd), types["attn"]),
              (p + "ffn_norm.weight", norm(dim), GGML_F32),
              (p + "ffn_gate.weight", w(hidden, dim), types["ffn"]),
              (p + "ffn_up.weight", w(hidden, dim), types["ffn"]),
              (p + "ffn_down.weight", w(dim, hidden), types["ffn"])]
    t.append(("output_norm.weight", norm(dim), GGML_F32))
    if not tied:
        t.append(("output.weight", w(vocab, dim), types["output"]))
    meta = {"block_count": layers, "embedding_length": dim, "feed_forward_length": hidden,
            "attention.head_count": heads, "attention.head_count_kv": kv_heads, "context_length": ctx,
            "rope.freq_base": float(theta), "attention.layer_norm_rms_epsilon": float(eps), "vocab": vocab}
    write_gguf(path, arch, meta, t)
