"""Batched lockstep decoding (mlb_batch) on one GPU: every sequence's greedy
tokens equal those of the single-sequence path for the same prompt -- the
oracle (the reference CPU algorithm) for the tiny model, the decode session
(itself pinned to the reference) for the larger ones.  Batches of up to 8
rows run their linears on the GEMV, larger ones on the tcgen05 tensor
cores."""
import numpy as np
import pytest

from mini_llama_b200 import capi
from mini_llama_b200.device import BatchSession, Model, Session
from oracle.binding import load_device_model
from oracle.binding import MODEL_SPECS

pytestmark = pytest.mark.gpu


def prompts(seed, batch, n, vocab):
    rng = np.random.default_rng(seed)
    return rng.integers(0, vocab, size=(batch, n), dtype=np.int32)


@pytest.fixture(scope="module")
def tiny(mlb, gpu, oracle):
    om = oracle.model("tiny")
    m = Model(mlb, gpu, MODEL_SPECS["tiny"])
    load_device_model(m, om)
    yield om, m
    m.close()
    om.close()


@pytest.mark.parametrize("batch", [1, 5, 12])
def test_tiny_batch_matches_oracle(tiny, batch):
    om, m = tiny
    p = prompts(100 + batch, batch, 4, 256)
    b = BatchSession(m, batch)
    try:
        toks, _, _ = b.generate(p, 8)
    finally:
        b.close()
    for i in range(batch):
        gen, _ = om.greedy(p[i], 8)
        assert list(toks[i]) == gen, f"sequence {i}"


def test_tiny_batch_logits_match_oracle(tiny):
    om, m = tiny
    p = prompts(7, 3, 5, 256)
    b = BatchSession(m, 3)
    try:
        b.generate(p, 1)  # the last step is the last prompt position
        got = b.logits()
    finally:
        b.close()
    for i in range(3):
        _, logits = om.greedy(p[i], 1)
        e = np.asarray(logits[-1], np.float64)
        assert float(np.abs(got[i] - e).max()) <= 1e-3 * max(1.0, float(np.abs(e).max())), f"sequence {i}"


@pytest.fixture(scope="module")
def qwen2(mlb, gpu):
    m = Model(mlb, gpu, MODEL_SPECS["qwen2"])
    m.synthesize(seed=MODEL_SPECS["qwen2"]["seed"], tied=True)
    yield m
    m.close()


@pytest.mark.parametrize("batch", [3, 10])
def test_qwen2_batch_matches_session(qwen2, batch):
    p = prompts(200 + batch, batch, 6, MODEL_SPECS["qwen2"]["vocab_size"])
    b = BatchSession(qwen2, batch)
    try:
        toks, pre, dec = b.generate(p, 8)
    finally:
        b.close()
    assert pre > 0 and dec > 0
    s = Session(qwen2)
    try:
        for i in range(batch):
            s.reset()
            assert list(toks[i]) == list(s.generate(p[i], 8)), f"sequence {i}"
    finally:
        s.close()


def test_llama2_q4_0_batch_matches_session(mlb, gpu):
    spec = MODEL_SPECS["llama2_l2"]
    m = Model(mlb, gpu, spec)
    try:
        m.synthesize(seed=spec["seed"], tied=False)
        p = prompts(300, 9, 5, spec["vocab_size"])
        b = BatchSession(m, 9)
        try:
            toks, _, _ = b.generate(p, 6)
        finally:
            b.close()
        s = Session(m)
        try:
            for i in range(9):
                s.reset()
                assert list(toks[i]) == list(s.generate(p[i], 6)), f"sequence {i}"
        finally:
            s.close()
    finally:
        m.close()


def test_batch_rejects_bad_prompt(tiny):
    _, m = tiny
    b = BatchSession(m, 2)
    try:
        p = prompts(1, 2, 3, 256)
        p[1, 2] = 256
        with pytest.raises(capi.MlbError) as e:
            b.generate(p, 2)
        assert e.value.status == capi.MLB_ERR_OUT_OF_RANGE
        with pytest.raises(capi.MlbError):
            b.generate(prompts(1, 2, 100, 256), 40)  # past max_seq_len
        toks, _, _ = b.generate(prompts(2, 2, 3, 256), 2)  # still usable
        assert toks.shape == (2, 2)
    finally:
        b.close()
