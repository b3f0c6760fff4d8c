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


def _worker(rank, world, port, q, mode="p2p"):
    """mode "p2p": the gather fused into the decode (HeadGather); "nccl": a
    plain decode of the rank's heads, then gkv_allgather_heads over a NCCL
    communicator made through the C ABI (gkv_nccl_unique_id / comm_create)."""
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
        import ctypes as C
        from genllm_b200 import _lib
        from genllm_b200.paged_attention import paged_attention
        L = _lib.lib()
        if mode == "p2p":
            hg = HeadGather(rank, n_layers=2, n_q_heads=hq)
        else:
            uid = (C.c_char * 128)()
            if rank == 0:
                assert L.gkv_nccl_unique_id(uid) == 0, L.gkv_last_error()
            box = [bytes(uid)]
            dist.broadcast_object_list(box, src=0)
            comm = C.c_void_p()
            assert L.gkv_nccl_comm_create(rank, world, rank, box[0], C.byref(comm)) == 0, L.gkv_last_error()
            full_out = torch.empty(hq, d, dtype=torch.bfloat16, device="cuda")
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
                if mode == "p2p":
                    out = hg.decode(m, layer, Q, K, V, full.scale)
                else:
                    mine = paged_attention(m, layer, Q, K, V, scale=full.scale)  # [1, Hq/N, 1, D] bf16
                    st = L.gkv_allgather_heads(comm, C.c_void_p(mine.data_ptr()), C.c_void_p(full_out.data_ptr()),
                                               mine.numel() * 2, C.c_void_p(torch.cuda.current_stream().cuda_stream))
                    assert st == 0, L.gkv_last_error()
                    out = full_out
                torch.cuda.synchronize()
                op.append_kv(kp, vp, kf, vf, hkv, 1, d)
                k_ids, v_ids = op.table()
                want = orc.paged_attention_f32(qf, kp, vp, k_ids, v_ids, op.num_cached, hq, hkv, 1, d, full.scale)
                got = out.float().cpu().numpy()
                # bf16 output: compare against the oracle rounded to bf16 as well.
                assert_close(got, bf16_to_f32(orc.round_bf16(want[:, 0])), f"rank {rank} step {step} layer {layer}")
        assert m.check_device_errors(0) == 0 and m.check_device_errors(1) == 0
        dist.barrier()
        if mode == "p2p":
            hg.close()
        else:
            assert L.gkv_nccl_comm_destroy(comm) == 0
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
@pytest.mark.parametrize("mode", ["p2p", "nccl"])
def test_head_allgather_two_gpus(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res


def test_gather_wait_runs_out_and_stream_stays_usable():
    """The fused gather's wait for its peers is bounded. One GPU, a world-2
    gather whose 'peer' never runs: both regions are local buffers, so this
    rank's combine stores its block into both and publishes its flag, but the
    peer's flag slot is never written. With a 2 ms limit the combine gives up,
    sets the timeout bit of the error word and finishes; the stream keeps
    working, and this rank's own block is still correct."""
    import ctypes as C

    from genllm_b200 import _lib
    from genllm_b200.synth import fragmented_case, randn_bf16
    from gpu_util import assert_close, build_state, to_dev_bf16

    L = _lib.lib()
    hq, hkv, d = 8, 4, 128
    case = fragmented_case(91, hq, hkv, d, 300, 40)
    m = build_state(case)
    ref = build_state(case)  # the same cache, decoded without the gather
    bases, flags = (C.c_void_p * 2)(), (C.c_void_p * 2)()
    for r in range(2):
        b, f = C.c_void_p(), C.c_void_p()
        assert L.gkv_device_alloc(0, hq * d * 2 * 2, C.byref(b)) == 0
        assert L.gkv_device_alloc(0, 4 * 2, C.byref(f)) == 0
        bases[r], flags[r] = b, f
    g = C.c_void_p()
    assert L.gkv_gather_create(0, 2, 0, 1, bases, flags, C.byref(g)) == 0, L.gkv_last_error()
    assert L.gkv_gather_set_wait_limit(g, 2_000_000) == 0
    assert L.gkv_gather_set_wait_limit(g, 10) == _lib.GKV_ERR_INVALID
    rng = np.random.default_rng(2)
    q = to_dev_bf16(randn_bf16(rng, (hq, 1, d)), "cuda")
    k = to_dev_bf16(randn_bf16(rng, (hkv, 1, d)), "cuda")
    v = to_dev_bf16(randn_bf16(rng, (hkv, 1, d)), "cuda")
    s = torch.cuda.current_stream()
    st = L.gkv_paged_attention_gather(m.handle, 0, C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()),
                                      C.c_void_p(v.data_ptr()), g, 0, hq, C.c_float(case.scale), _lib.GKV_F32,
                                      C.c_void_p(s.cuda_stream))
    assert st == 0, L.gkv_last_error()
    torch.cuda.synchronize()
    assert m.check_device_errors(0) & 2, "the wait for the silent peer did not report a timeout"
    # The stream and the context are fine: a regular decode and a torch op run after it.
    from genllm_b200.paged_attention import paged_attention
    want = torch.empty(1, hq, 1, d, device="cuda")
    paged_attention(ref, 0, q.view(1, hq, 1, d), k.view(1, hkv, 1, d), v.view(1, hkv, 1, d), out=want,
                    scale=case.scale)
    torch.cuda.synchronize()
    # Rank 0's block sits at offset 0 of its own region (bases[0]).
    got = torch.as_tensor(_CudaView(bases[0], hq * d), device="cuda").clone()  # ctypes array items are ints
    torch.cuda.synchronize()
    assert_close(got.view(hq, d).cpu().numpy(), want[0, :, 0].cpu().numpy(), "own block after timeout")
    assert ref.check_device_errors(0) == 0
    assert L.gkv_gather_destroy(g) == 0
    for r in range(2):
        L.gkv_device_free(0, bases[r])
        L.gkv_device_free(0, flags[r])


class _CudaView:
    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": (n,), "typestr": "<f4", "version": 3,
                                         "strides": None}
