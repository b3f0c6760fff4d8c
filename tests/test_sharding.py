"""KV-head sharding across ranks (the multi-GPU path), on CPU with gloo.

Each of 2 ranks owns half of the kv heads (and their query heads) of every
page; the block table is the same on every rank. Each rank computes its
heads' attention with the CPU oracle on its slice of the pages, the outputs
are all-gathered with the same helper bench.py uses, and the result must
equal the single-device oracle bit for bit (the per-head arithmetic is
identical)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from genllm_b200.synth import fragmented_case
from genllm_b200.workload import allgather_heads, shard_heads


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.oracle import Oracle, run_oracle_case
        case = fragmented_case(9, 16, 8, 128, 300, 30)
        qb, qe, kb, ke = shard_heads(16, 8, world, rank)
        # This rank's slice: its kv heads of every page, its query heads.
        case.k_pool = np.ascontiguousarray(case.k_pool[:, :, kb:ke])
        case.v_pool = np.ascontiguousarray(case.v_pool[:, :, kb:ke])
        case.k_new = np.ascontiguousarray(case.k_new[kb:ke])
        case.v_new = np.ascontiguousarray(case.v_new[kb:ke])
        case.q = np.ascontiguousarray(case.q[qb:qe])
        case.n_q_heads, case.n_kv_heads = qe - qb, ke - kb
        out, _, _, k_ids, v_ids, _ = run_oracle_case(case, Oracle())
        full = torch.empty((16, 1, 128), dtype=torch.float32)
        allgather_heads(torch.from_numpy(out), full)
        ids = torch.from_numpy(np.concatenate([k_ids, v_ids]))
        same = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(same, ids)
        if rank == 0:
            np.savez(result_path, full=full.numpy(), tables_equal=all(torch.equal(same[0], x) for x in same))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_kv_head_sharding_matches_single_device(tmp_path, world):
    from oracle.oracle import Oracle, run_oracle_case
    path = str(tmp_path / "res.npz")
    mp.spawn(_worker, args=(world, _free_port(), path), nprocs=world, join=True)
    r = np.load(path)
    want = run_oracle_case(fragmented_case(9, 16, 8, 128, 300, 30), Oracle())[0]
    assert bool(r["tables_equal"])
    assert np.array_equal(r["full"], want)


def test_shard_heads_partition():
    for world in (1, 2, 4, 8):
        seen_q, seen_k = [], []
        for rank in range(world):
            qb, qe, kb, ke = shard_heads(32, 8, world, rank)
            assert qe - qb == 32 // world and ke - kb == 8 // world
            assert qb == kb * 4 and qe == ke * 4  # query heads follow their kv head
            seen_q += list(range(qb, qe))
            seen_k += list(range(kb, ke))
        assert seen_q == list(range(32)) and seen_k == list(range(8))
    with pytest.raises(ValueError):
        shard_heads(32, 8, 3, 0)
