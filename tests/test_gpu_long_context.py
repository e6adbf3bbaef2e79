"""Long contexts on both decode paths, greedy tokens bit-exact against the
oracle (the reference CPU path).

The model has the Qwen2-0.5B attention shape (14 query heads over 2 KV heads,
head_dim 64, NeoX RoPE with theta 1e6, q/k/v bias, tied head) with small
linears, and a cache of 8192 positions, so that the reference accepts every
position below it (src/cuda_kv_cache.cpp:63-80, src/cuda_attention.cu:221-235).
Prompts of 290, 1010 and 4100 tokens are followed by 24 greedy tokens:

* persistent decode kernel: attention over the cache in passes of 256
  positions with a running max and sum (positions past 256 take the later
  passes, reading K and V rows from the cache);
* per-token graph: split-K attention whose partials no longer fit the
  O-projection's prologue at this cache length, so a merge kernel runs
  before a plain O-projection.

The 290-token prompt also runs token by token through the persistent kernel
(no prompt pass), so the kernel itself writes and reads the cache past 256.
"""
import numpy as np
import pytest

from mini_llama_b200.device import Model, Session
from oracle.binding import load_device_model

pytestmark = pytest.mark.gpu

LONG = dict(vocab_size=512, dim=256, hidden_dim=512, n_layers=2, n_heads=14, n_kv_heads=2, head_dim=64,
            max_seq_len=8192, rope_theta=1e6, rms_norm_eps=1e-6, rope_neox=1, qkv_bias=1, tied_embedding=1,
            seed=21, prompt_seed=22)
N_NEW = 24


@pytest.fixture(scope="module")
def long_model(mlb, gpu, oracle):
    om = oracle.model("tiny", **LONG)
    m = Model(mlb, gpu, om.spec)
    load_device_model(m, om)
    yield om, m
    m.close()
    om.close()


@pytest.mark.parametrize("n_prompt", [290, 1010, 4100])
def test_long_context_greedy_both_paths(mlb, gpu, long_model, n_prompt):
    om, m = long_model
    prompt = om.prompt(n_prompt)
    gen_ref, _ = om.greedy(prompt, N_NEW)
    runs = [("persistent kernel", True, 16), ("graph", False, 16)]
    if n_prompt == 290:
        runs.append(("persistent kernel, token by token", True, 0))
    for name, persistent, prefill_min in runs:
        s = Session(m)
        try:
            s.use_persistent(persistent)
            assert s.path() == (2 if persistent else 1), name
            s.prefill_min(prefill_min)
            gen = s.generate(prompt, N_NEW)
            assert list(gen) == list(gen_ref), f"{name}, prompt {n_prompt}: {list(gen)} != {list(gen_ref)}"
        finally:
            s.close()


def test_qwen2_shape_8192_cache_paths_agree(mlb, gpu):
    """The full Qwen2-0.5B-architecture Q8_0 model with an 8192-position
    cache: both decode paths accept it, and past position 4096 they agree on
    the greedy tokens (the oracle, at 0.1 s a token on the CPU, is left to
    the model above)."""
    from mini_llama_b200 import synth
    cfg = dict(vocab_size=151936, dim=896, hidden_dim=4864, n_layers=24, n_heads=14, n_kv_heads=2,
               head_dim=64, max_seq_len=8192, rope_theta=1e6, rms_norm_eps=1e-6, rope_neox=1,
               qkv_bias=1, tied_embedding=1, qtype=1, seed=3, prompt_seed=3)
    m = Model(mlb, gpu, cfg)
    try:
        m.synthesize(seed=cfg["seed"], tied=True)
        prompt = synth.tokens(4100, cfg["prompt_seed"], cfg["vocab_size"])
        out = {}
        for persistent in (True, False):
            s = Session(m)
            try:
                s.use_persistent(persistent)
                out[persistent] = list(s.generate(prompt, 16))
            finally:
                s.close()
        assert out[True] == out[False], out
    finally:
        m.close()
