"""Tensor-parallel batched decoding on 2 GPUs (one process each, NCCL inside
the library): the greedy tokens equal the single-GPU batch's and each rank's
logits slice matches the single-GPU logits.  Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from mini_llama_b200 import capi
from mini_llama_b200.device import BatchSession, Model, nccl_unique_id
from mini_llama_b200.tp import share_nccl_id
from oracle.binding import MODEL_SPECS

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, name, batch, n_prompt, n_new, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lib = capi.load()
        spec = MODEL_SPECS[name]
        m = Model(lib, rank, spec)
        try:
            m.synthesize(seed=spec["seed"], tied=bool(spec["tied_embedding"]))
            rng = np.random.default_rng(42)
            p = rng.integers(0, spec["vocab_size"], size=(batch, n_prompt), dtype=np.int32)
            nid = share_nccl_id(dist, lambda: nccl_unique_id(lib))
            b = BatchSession(m, batch, rank, world, nid)
            try:
                toks, _, _ = b.generate(p, n_new)
                logits = b.logits()
            finally:
                dist.barrier()
                b.close()
            res = {"tokens": toks.tolist(), "logits": logits}
            if rank == 0:
                b1 = BatchSession(m, batch)
                try:
                    t1, _, _ = b1.generate(p, n_new)
                    res["ref_tokens"] = t1.tolist()
                    res["ref_logits"] = b1.logits()
                finally:
                    b1.close()
            out[rank] = res
        finally:
            m.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name,batch", [("qwen2", 4), ("qwen2", 12), ("llama2_l2", 10)])
def test_two_gpu_batch_matches_one_gpu(mlb, name, batch):
    if mlb.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with mp.get_context("spawn").Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_worker, args=(2, _free_port(), name, batch, 5, 6, out), nprocs=2, join=True)
        res = dict(out)
    ref = np.asarray(res[0]["ref_tokens"])
    for r in (0, 1):
        assert np.array_equal(np.asarray(res[r]["tokens"]), ref), f"rank {r} tokens"
    full = np.concatenate([res[0]["logits"], res[1]["logits"]], axis=1)
    e = res[0]["ref_logits"].astype(np.float64)
    err = float(np.abs(full - e).max())
    assert err <= 1e-4 * max(1.0, float(np.abs(e).max())), err
