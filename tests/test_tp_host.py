"""Host-side logic of the tensor-parallel batch driver, on the CPU: the shard
ranges (mlb_batch_shard, no device needed) and the NCCL id exchange and timing
reduction over a world-size-2 gloo group."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from mini_llama_b200 import capi
from mini_llama_b200.device import batch_shard
from mini_llama_b200.tp import max_over_ranks, share_nccl_id
from oracle.binding import MODEL_SPECS

LLAMA7B = dict(vocab_size=32000, dim=4096, hidden_dim=11008, n_layers=32, n_heads=32, n_kv_heads=32,
               head_dim=128, max_seq_len=768, rope_theta=1e4, rms_norm_eps=1e-5, rope_neox=0,
               qkv_bias=0, tied_embedding=0, qtype=capi.Q4_0)


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_llama7b_shards_cover_everything(tp):
    lib = capi.load()
    seen = {k: [] for k in ("heads", "kv_heads", "dim", "hidden", "vocab")}
    for r in range(tp):
        s = batch_shard(lib, LLAMA7B, r, tp)
        for k, (a, b) in s.items():
            seen[k].append((a, b))
        # q heads are the query heads of the rank's KV heads
        group = LLAMA7B["n_heads"] // LLAMA7B["n_kv_heads"]
        assert s["heads"] == (s["kv_heads"][0] * group, s["kv_heads"][1] * group)
    full = {"heads": 32, "kv_heads": 32, "dim": 4096, "hidden": 11008, "vocab": 32000}
    for k, ranges in seen.items():
        assert ranges[0][0] == 0 and ranges[-1][1] == full[k]
        assert all(ranges[i][1] == ranges[i + 1][0] for i in range(tp - 1))
        assert len({b - a for a, b in ranges}) == 1  # equal slices (NCCL all-gather)


def test_qwen2_splits_at_most_two_ways():
    lib = capi.load()
    spec = MODEL_SPECS["qwen2"]
    assert batch_shard(lib, spec, 1, 2)["kv_heads"] == (1, 2)
    with pytest.raises(capi.MlbError) as e:
        batch_shard(lib, spec, 0, 4)  # 2 KV heads
    assert e.value.status == capi.MLB_ERR_UNSUPPORTED
    with pytest.raises(capi.MlbError):
        batch_shard(lib, spec, 2, 2)  # rank out of range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        nid = share_nccl_id(dist, lambda: bytes(range(128)))
        t = max_over_ranks(dist, [float(rank + 1), float(10 - rank)])
        out[rank] = (nid == bytes(range(128)), t)
    finally:
        dist.destroy_process_group()


def test_nccl_id_exchange_and_timing_max_over_gloo():
    port = _free_port()
    with mp.get_context("spawn").Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
        res = dict(out)
    assert res[0][0] and res[1][0]
    assert res[0][1] == res[1][1] == [2.0, 10.0]


def test_library_loaded_before_torch_leaves_torch_importable():
    """NCCL is opened lazily: loading the library first must not bind a system
    NCCL that PyTorch's own build cannot use."""
    import subprocess
    import sys
    code = (f"import ctypes; ctypes.CDLL({capi.LIB_PATH!r}); import torch; "
            "import torch.distributed; print('ok')")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-2000:]
