"""Seeded prompt ids for benchmarks: the counter-based splitmix64 generator of
the library's synthetic inputs (mlb_synth_normal draws the weights from the
same streams), here for uniform token ids on the host.

    key   = mix64(seed * GAMMA + stream * 0xD1B54A32D192ED03 + 1)
    u64_k = mix64(key + (k + 1) * GAMMA)
    id_i  = ((u64_i >> 32) * vocab) >> 32          (stream 3: prompts)
"""
from __future__ import annotations

import numpy as np

_M64 = (1 << 64) - 1
_GAMMA = 0x9E3779B97F4A7C15
STREAM_PROMPT = 3


def _mix64(z: int) -> int:
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def tokens(n: int, seed: int, vocab: int, stream: int = STREAM_PROMPT) -> np.ndarray:
    """n token ids uniform over [0, vocab) for (seed, stream)."""
    key = _mix64((seed * _GAMMA + stream * 0xD1B54A32D192ED03 + 1) & _M64)
    out = np.empty(n, np.int32)
    for i in range(n):
        r = _mix64((key + (i + 1) * _GAMMA) & _M64) >> 32
        out[i] = (r * vocab) >> 32
    return out
