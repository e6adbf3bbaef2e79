"""Regenerates the golden fixtures of this directory from the reference itself.

Runs oracle/_ref/ref_harness (the reference mini_llama CPU sources compiled by
oracle/Makefile) on the seeded inputs of oracle/synth.h and packs its raw
outputs into .npz files:

    ops.npz            fp16 tables, Q8_0/Q4_0/Q4_1 blocks, dequantized weights,
                       LinearQ80/Q40/Q41, RmsNorm, Silu/Swiglu/Softmax, GetArgMax,
                       RoPE (MiniLlamaContext tables), GQA attention
    model_tiny.npz     tiny Llama Q8_0: prompt, greedy tokens, logits every step
    model_llama2_l2.npz  Llama-2-7B shapes, 2 layers, Q4_0
    model_qwen2.npz    Qwen2-0.5B shapes Q8_0: 64-token prompt + 128 greedy tokens

Usage: python tests/golden/make_golden.py [case ...]   (needs the reference tree)
"""
from __future__ import annotations

import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
HARNESS = os.path.join(ROOT, "oracle", "_ref", "ref_harness")

DTYPES = {".f32": np.float32, ".u16": np.uint16, ".i32": np.int32, ".u8": np.uint8}
GROUPS = {
    "ops": ["fp16", "quant", "normact", "rope", "attention"],
    "model_tiny": ["tiny"],
    "model_llama2_l2": ["llama2_l2"],
    "model_qwen2": ["qwen2"],
}


def load_dir(path: str) -> dict:
    out = {}
    for name in sorted(os.listdir(path)):
        stem, ext = os.path.splitext(name)
        if ext in DTYPES:
            out[stem] = np.fromfile(os.path.join(path, name), dtype=DTYPES[ext])
    return out


def main(argv):
    want = argv or list(GROUPS)
    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "-j8"], check=True)
    for group in want:
        with tempfile.TemporaryDirectory() as tmp:
            subprocess.run([HARNESS, "golden", tmp] + GROUPS[group], check=True)
            arrays = load_dir(tmp)
        dst = os.path.join(HERE, group + ".npz")
        np.savez_compressed(dst, **arrays)
        print(f"{dst}: {len(arrays)} arrays, {os.path.getsize(dst) / 1e6:.2f} MB")


if __name__ == "__main__":
    main(sys.argv[1:])
