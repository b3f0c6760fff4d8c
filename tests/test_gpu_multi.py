"""KV-head sharding on 2 GPUs with the head all-gather fused into the decode
step (genllm_b200.gather.HeadGather over the C ABI, NVLink peer stores).

Each rank holds half of the kv heads of a fragmented cache; three decode
steps run in a row on two layers; after each step every rank's gathered
[Hq, 128] output must match the CPU oracle of the full-head cache within the
path's tolerance. Needs 2 GPUs (skipped otherwise)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        import sys
        here = os.path.dirname(os.path.abspath(__file__))
        sys.path.insert(0, os.path.dirname(here))
        sys.path.insert(0, here)
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from genllm_b200.gather import HeadGather
        from genllm_b200.synth import bf16_to_f32, fragmented_case, randn_bf16
        from genllm_b200.workload import shard_heads
        from gpu_util import assert_close, build_state, to_dev_bf16
        from oracle.oracle import Oracle, OraclePool
        hq, hkv, d = 16, 8, 128
        qb, qe, kb, ke = shard_heads(hq, hkv, world, rank)
        hg = HeadGather(rank, n_layers=2, n_q_heads=hq)
        orc = Oracle()
        mgrs_cases = []
        from genllm_b200.paged_attention import PagedAttentionManager
        m = PagedAttentionManager(rank)
        for layer in range(2):
            full = fragmented_case(70 + layer, hq, hkv, d, 200 + 17 * layer, 24)
            mine = fragmented_case(70 + layer, hq, hkv, d, 200 + 17 * layer, 24)
            mine.k_pool = np.ascontiguousarray(full.k_pool[:, :, kb:ke])
            mine.v_pool = np.ascontiguousarray(full.v_pool[:, :, kb:ke])
            mine.n_kv_heads, mine.n_q_heads = ke - kb, qe - qb
            build_state(mine, rank, layer, m)
            op = OraclePool(full.pool_pages, orc)
            for w, order in ((0, full.k_free_order), (1, full.v_free_order)):
                for _ in range(full.pool_pages):
                    op.alloc(w)
                for i in order:
                    op.free(w, int(i))
            op.set_table(full.k_ids, full.v_ids, full.n_prior)
            mgrs_cases.append((full, op, full.k_pool.copy(), full.v_pool.copy()))
        rng = np.random.default_rng(5)
        for step in range(3):
            for layer in range(2):
                full, op, kp, vp = mgrs_cases[layer]
                qf = randn_bf16(rng, (hq, 1, d))
                kf = randn_bf16(rng, (hkv, 1, d))
                vf = randn_bf16(rng, (hkv, 1, d))
                Q = to_dev_bf16(np.ascontiguousarray(qf[qb:qe]), "cuda").view(1, qe - qb, 1, d)
                K = to_dev_bf16(np.ascontiguousarray(kf[kb:ke]), "cuda").view(1, ke - kb, 1, d)
                V = to_dev_bf16(np.ascontiguousarray(vf[kb:ke]), "cuda").view(1, ke - kb, 1, d)
                out = hg.decode(m, layer, Q, K, V, full.scale)
                torch.cuda.synchronize()
                op.append_kv(kp, vp, kf, vf, hkv, 1, d)
                k_ids, v_ids = op.table()
                want = orc.paged_attention_f32(qf, kp, vp, k_ids, v_ids, op.num_cached, hq, hkv, 1, d, full.scale)
                got = out.float().cpu().numpy()
                # bf16 output: compare against the oracle rounded to bf16 as well.
                assert_close(got, bf16_to_f32(orc.round_bf16(want[:, 0])), f"rank {rank} step {step} layer {layer}")
        assert m.check_device_errors(0) == 0 and m.check_device_errors(1) == 0
        dist.barrier()
        hg.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent
        import traceback
        q.put((rank, traceback.format_exc()))


def _stress_worker(rank, world, port, q):
    """40 back-to-back steps on 2 layers with no host synchronisation: every
    step's gathered output is snapshotted on the stream right after the call
    (stream order puts the copy after the call's completion, i.e. after the
    peers' blocks were flagged as landed). Each rank's snapshot of the peer's
    heads must equal the peer's own snapshot of them, bit for bit."""
    try:
        import sys
        here = os.path.dirname(os.path.abspath(__file__))
        sys.path.insert(0, os.path.dirname(here))
        sys.path.insert(0, here)
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from genllm_b200.gather import HeadGather
        from genllm_b200.paged_attention import PagedAttentionManager
        from genllm_b200.synth import fragmented_case, randn_bf16
        from genllm_b200.workload import shard_heads
        from gpu_util import build_state, to_dev_bf16
        hq, hkv, d, steps = 16, 8, 128, 40
        qb, qe, kb, ke = shard_heads(hq, hkv, world, rank)
        hg = HeadGather(rank, n_layers=2, n_q_heads=hq)
        m = PagedAttentionManager(rank)
        for layer in range(2):
            c = fragmented_case(90 + layer, hq, hkv, d, 3000 + 17 * layer, 260)
            c.k_pool = np.ascontiguousarray(c.k_pool[:, :, kb:ke])
            c.v_pool = np.ascontiguousarray(c.v_pool[:, :, kb:ke])
            c.n_kv_heads, c.n_q_heads = ke - kb, qe - qb
            build_state(c, rank, layer, m)
        rng = np.random.default_rng(11)
        ins = []
        for step in range(steps):
            for layer in range(2):
                qf = randn_bf16(rng, (hq, 1, d))
                kf = randn_bf16(rng, (hkv, 1, d))
                vf = randn_bf16(rng, (hkv, 1, d))
                ins.append(tuple(to_dev_bf16(np.ascontiguousarray(a), "cuda").view(1, e - b, 1, d)
                                 for a, b, e in ((qf[qb:qe], qb, qe), (kf[kb:ke], kb, ke), (vf[kb:ke], kb, ke))))
        torch.cuda.synchronize()
        dist.barrier()
        snaps = []
        for step in range(steps):
            for layer in range(2):
                Q, K, V = ins[step * 2 + layer]
                out = hg.decode(m, layer, Q, K, V, 1.0 / np.sqrt(d))
                snaps.append(out.clone())
        torch.cuda.synchronize()
        got = torch.stack(snaps).view(steps * 2, hq, d).cpu()
        allv = [None] * world
        dist.all_gather_object(allv, got)
        for r in range(world):
            pb, pe, _, _ = shard_heads(hq, hkv, world, r)
            assert torch.equal(got[:, pb:pe], allv[r][:, pb:pe]), f"rank {rank}: heads of rank {r} differ"
        assert m.check_device_errors(0) == 0 and m.check_device_errors(1) == 0
        dist.barrier()
        hg.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:  # report to the parent
        import traceback
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_head_allgather_back_to_back_steps():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_stress_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_head_allgather_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res
