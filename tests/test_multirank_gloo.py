"""Multi-rank host logic on CPU (gloo, world size 2): KV-head sharding is
exact, and a rank that leaves early ends the others' next collective with
an error instead of a hang."""

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _sharded_worker(rank, world, port, result_path):
    sys.path.insert(0, str(REPO))
    import oracle
    import workloads
    from my_vllm_b200 import sharding

    _init(rank, world, port)
    w = workloads.config1(device="cpu")
    shard = sharding.kv_head_shard(w.num_q_heads, w.num_kv_heads, rank, world)
    q, key, value, kc, vc = sharding.shard_tensors(shard, w.q, w.key, w.value, w.k_cache,
                                                   w.v_cache)

    def bits(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    kc_b, vc_b = bits(kc).copy(), bits(vc).copy()
    oracle.kv_append(bits(key), bits(value), kc_b, vc_b, w.slot_mapping.numpy())
    out = oracle.paged_attention_from_tables(bits(q), kc_b, vc_b, w.block_tables.numpy(),
                                             w.seq_lens.numpy(), w.query_start_loc.numpy(),
                                             w.block_size, out_dtype="float32")
    parts = [torch.empty_like(torch.from_numpy(out)) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(out))
    if rank == 0:
        np.save(result_path, torch.cat(parts, dim=1).numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_kv_head_sharding_matches_unsharded(tmp_path):
    sys.path.insert(0, str(REPO))
    import oracle
    import workloads

    result = tmp_path / "sharded.npy"
    mp.start_processes(_sharded_worker, args=(2, _free_port(), str(result)), nprocs=2,
                       join=True, start_method="spawn")
    w = workloads.config1(device="cpu")

    def bits(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    kc, vc = bits(w.k_cache).copy(), bits(w.v_cache).copy()
    oracle.kv_append(bits(w.key), bits(w.value), kc, vc, w.slot_mapping.numpy())
    full = oracle.paged_attention_from_tables(bits(w.q), kc, vc, w.block_tables.numpy(),
                                              w.seq_lens.numpy(), w.query_start_loc.numpy(),
                                              w.block_size, out_dtype="float32")
    np.testing.assert_allclose(np.load(result), full, rtol=0, atol=1e-6)


def _leaver_worker(rank, world, port, flag_path):
    _init(rank, world, port, timeout_s=5)
    dist.barrier()
    if rank == 1:
        # leaves between steps, with nothing in flight
        os._exit(0)
    try:
        t = torch.ones(1)
        dist.all_reduce(t)
        dist.barrier()
    except Exception as exc:  # noqa: BLE001 - any error proves no hang
        Path(flag_path).write_text(type(exc).__name__)
        os._exit(0)
    os._exit(3)


def test_rank_that_leaves_ends_peers_collective_with_error(tmp_path):
    flag = tmp_path / "error.txt"
    ctx = mp.start_processes(_leaver_worker, args=(2, _free_port(), str(flag)), nprocs=2,
                             join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
        assert not p.is_alive(), "a rank hung"
    assert flag.exists(), "rank 0 did not observe its peer leaving"


def test_shard_ranges():
    from my_vllm_b200 import sharding

    s = sharding.kv_head_shard(64, 8, 3, 8)
    assert (s.q_heads, s.kv_heads) == (slice(24, 32), slice(3, 4))
    with pytest.raises(ValueError):
        sharding.kv_head_shard(32, 8, 0, 3)
    with pytest.raises(ValueError):
        sharding.kv_head_shard(32, 8, 2, 2)
