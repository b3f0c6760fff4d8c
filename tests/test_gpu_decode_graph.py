"""Captured decode steps (gkv_decode_graph_*): a CUDA graph replayed per
token gives exactly what gkv_decode_layers gives (same kernels, same split
geometry; outputs, pages and tables bit-identical) over many tokens, page
boundaries, host-only table growth, QK-norm + RoPE and pool exhaustion;
and one replayed step against the oracle."""
import os

import numpy as np
import pytest
import torch

from genllm_b200._lib import GKV_ERR_NO_PAGES, GkvError
from genllm_b200.paged_attention import (DecodeGraph, DecodeStep, PagedAttentionManager, QkNorm,
                                         paged_attention_qknorm)
from genllm_b200.synth import fragmented_case, qk_rope_case
from gpu_util import assert_close, build_state, to_dev_bf16
from oracle.oracle import Oracle, run_oracle_case

pytestmark = pytest.mark.gpu
HQ, HKV = 16, 8


def twin_managers(priors, pool_pages, seed=0):
    cases = [fragmented_case(seed + 40 * l, HQ, HKV, 128, n, pool_pages) for l, n in enumerate(priors)]
    ma, mb = PagedAttentionManager(0), PagedAttentionManager(0)
    for l, c in enumerate(cases):
        build_state(c, mgr=ma, layer=l)
        build_state(c, mgr=mb, layer=l)
    return cases, ma, mb


def bound_tensors(n, dev, out_dtype=torch.bfloat16):
    Q = [torch.empty((HQ, 128), dtype=torch.bfloat16, device=dev) for _ in range(n)]
    K = [torch.empty((HKV, 128), dtype=torch.bfloat16, device=dev) for _ in range(n)]
    V = [torch.empty((HKV, 128), dtype=torch.bfloat16, device=dev) for _ in range(n)]
    O = [torch.empty((HQ, 128), dtype=out_dtype, device=dev) for _ in range(n)]
    return Q, K, V, O


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_graph_matches_decode_step_over_many_tokens(out_dtype):
    priors = [14, 301, 2357]  # a page boundary on step 2; 147 splits on the last layer
    cases, ma, mb = twin_managers(priors, 2357 // 16 + 8)
    dev = ma.device
    qa, ka, va, oa = bound_tensors(3, dev, out_dtype)
    qb, kb, vb, ob = bound_tensors(3, dev, out_dtype)
    graph = DecodeGraph(ma, [0, 1, 2], qa, ka, va, oa, HQ, cases[0].scale)
    step = DecodeStep(mb, [0, 1, 2], qb, kb, vb, ob, HQ, cases[0].scale)
    g = torch.Generator(device=dev).manual_seed(3)
    for t in range(24):
        for l in range(3):
            for a, b in ((qa[l], qb[l]), (ka[l], kb[l]), (va[l], vb[l])):
                a.copy_(torch.randn(a.shape, generator=g, device=dev).to(torch.bfloat16))
                b.copy_(a)
        graph.run()
        step.run()
        torch.cuda.synchronize()
        for l in range(3):
            assert torch.equal(oa[l], ob[l]), f"token {t}, layer {l}: outputs differ"
    for l in range(3):
        kpa, vpa = ma.pool_tensors(l)
        kpb, vpb = mb.pool_tensors(l)
        assert torch.equal(kpa, kpb) and torch.equal(vpa, vpb)
        assert ma.get_layer(l).num_cached == mb.get_layer(l).num_cached == priors[l] + 24
        assert ma.device_table(l) == mb.device_table(l) == ma.page_table(l)
        assert ma.check_device_errors(l) == 0
    graph.close()


def test_graph_step_against_the_oracle():
    c = fragmented_case(77, HQ, HKV, 128, 1000, 80, page_order="desc")
    o_out, o_kp, o_vp, _, _, _ = run_oracle_case(c, Oracle(), True, threads=min(os.cpu_count() or 1, 16))
    m = build_state(c)
    Q, K, V, O = bound_tensors(1, m.device, torch.float32)
    Q[0].copy_(to_dev_bf16(c.q, m.device).view(HQ, 128))
    K[0].copy_(to_dev_bf16(c.k_new, m.device).view(HKV, 128))
    V[0].copy_(to_dev_bf16(c.v_new, m.device).view(HKV, 128))
    graph = DecodeGraph(m, [0], Q, K, V, O, HQ, c.scale)
    graph.run()
    torch.cuda.synchronize()
    assert_close(O[0].cpu().numpy(), o_out.reshape(HQ, 128), "captured decode step")
    kp, vp = m.pool_tensors(0)
    assert np.array_equal(kp.view(torch.int16).cpu().numpy().view(np.uint16).reshape(o_kp.shape), o_kp)
    graph.close()


def test_graph_after_host_only_growth():
    """Pages grown with append_kv_pages before a captured step (more than one
    pending table entry) reach the device table first."""
    cases, ma, mb = twin_managers([40, 90], 40, seed=5)
    for m in (ma, mb):
        m.append_kv_pages(0, 50)   # 3 pending pages on layer 0
        m.append_kv_pages(1, 2)
    dev = ma.device
    qa, ka, va, oa = bound_tensors(2, dev)
    qb, kb, vb, ob = bound_tensors(2, dev)
    graph = DecodeGraph(ma, [0, 1], qa, ka, va, oa, HQ)
    step = DecodeStep(mb, [0, 1], qb, kb, vb, ob, HQ)
    g = torch.Generator(device=dev).manual_seed(4)
    for _ in range(3):
        for l in range(2):
            for a, b in ((qa[l], qb[l]), (ka[l], kb[l]), (va[l], vb[l])):
                a.copy_(torch.randn(a.shape, generator=g, device=dev).to(torch.bfloat16))
                b.copy_(a)
        graph.run()
        step.run()
    torch.cuda.synchronize()
    for l in range(2):
        assert torch.equal(oa[l], ob[l])
        assert ma.device_table(l) == mb.device_table(l)
    graph.close()


def test_graph_with_qk_norm_matches_per_layer_calls():
    n_prior, max_seq = 500, 600
    cases, ma, mb = twin_managers([n_prior, n_prior + 3], 48, seed=9)
    dev = ma.device
    p = [qk_rope_case(60 + l, HQ, HKV, 1, n_prior) for l in range(2)]
    qks = [QkNorm(torch.from_numpy(c.q_norm_w), torch.from_numpy(c.k_norm_w), c.eps, c.theta, max_seq, 0) for c in p]
    qa = [torch.empty((1, HQ * 128), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    ka = [torch.empty((1, HKV * 128), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    va = [torch.empty((1, HKV * 128), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    oa = [torch.empty((HQ, 128), dtype=torch.float32, device=dev) for _ in range(2)]
    ob = [torch.empty((HQ, 1, 128), dtype=torch.float32, device=dev) for _ in range(2)]
    graph = DecodeGraph(ma, [0, 1], qa, ka, va, oa, HQ, qk=qks)
    g = torch.Generator(device=dev).manual_seed(8)
    for _ in range(5):
        for l in range(2):
            for t in (qa[l], ka[l], va[l]):
                t.copy_(torch.randn(t.shape, generator=g, device=dev).to(torch.bfloat16))
        graph.run()
        for l in range(2):
            paged_attention_qknorm(mb, l, qa[l], ka[l], va[l], HQ, qks[l], out=ob[l])
        torch.cuda.synchronize()
        for l in range(2):
            assert torch.equal(oa[l], ob[l].view(HQ, 128))
    for l in range(2):
        assert torch.equal(ma.pool_tensors(l)[0], mb.pool_tensors(l)[0])
    graph.close()


def test_graph_step_fails_whole_when_a_pool_runs_out():
    """Layer 1's pool has no page for the next token: the step raises
    GKV_ERR_NO_PAGES and no layer advances."""
    cases, ma, _ = twin_managers([20, 32], 3, seed=11)  # 2 of 3 pages used in each layer
    dev = ma.device
    q, k, v, o = bound_tensors(2, dev)
    for t in q + k + v:
        t.normal_()
    graph = DecodeGraph(ma, [0, 1], q, k, v, o, HQ)
    # layer 1 takes its third page at position 32 (step 1); position 48
    # (step 17) would need a fourth, while layer 0 still has room
    for _ in range(16):
        graph.run()
    before = [ma.get_layer(l).num_cached for l in range(2)]
    with pytest.raises(GkvError) as e:
        graph.run()
    assert e.value.status == GKV_ERR_NO_PAGES
    assert [ma.get_layer(l).num_cached for l in range(2)] == before
    torch.cuda.synchronize()
    assert ma.check_device_errors(0) == 0 and ma.check_device_errors(1) == 0
    graph.close()


@pytest.mark.parametrize("runner", ["graph", "one_call"])
def test_multi_layer_steps_back_to_back_match_per_layer_calls(runner):
    """Thirty steps of a four-layer step (early release between layers) with
    no host synchronisation between steps, against per-layer calls (each
    launch ordered after the previous one): every step's outputs and the
    final pages bit-identical. Contexts of very different lengths make the
    layers' grids end unevenly."""
    priors = [2000, 17, 3000, 500]
    cases, ma, mb = twin_managers(priors, 3000 // 16 + 8, seed=21)
    dev = ma.device
    n, steps = len(priors), 30
    qa, ka, va, oa = bound_tensors(n, dev)
    g = torch.Generator(device=dev).manual_seed(12)
    feed_q = torch.randn((steps, n, HQ, 128), generator=g, device=dev).to(torch.bfloat16)
    feed_k = torch.randn((steps, n, HKV, 128), generator=g, device=dev).to(torch.bfloat16)
    feed_v = torch.randn((steps, n, HKV, 128), generator=g, device=dev).to(torch.bfloat16)
    hist_a = torch.empty((steps, n, HQ, 128), dtype=torch.bfloat16, device=dev)
    hist_b = torch.empty_like(hist_a)
    r = (DecodeGraph if runner == "graph" else DecodeStep)(ma, list(range(n)), qa, ka, va, oa, HQ)
    torch.cuda.synchronize()
    for t in range(steps):
        for l in range(n):
            qa[l].copy_(feed_q[t, l])
            ka[l].copy_(feed_k[t, l])
            va[l].copy_(feed_v[t, l])
        r.run()
        for l in range(n):
            hist_a[t, l].copy_(oa[l])
    from genllm_b200.paged_attention import paged_attention
    ob = torch.empty((1, HQ, 1, 128), dtype=torch.bfloat16, device=dev)
    for t in range(steps):
        for l in range(n):
            paged_attention(mb, l, feed_q[t, l].view(1, HQ, 1, 128), feed_k[t, l].view(1, HKV, 1, 128),
                            feed_v[t, l].view(1, HKV, 1, 128), out=ob)
            hist_b[t, l].copy_(ob[0, :, 0])
    torch.cuda.synchronize()
    assert torch.equal(hist_a, hist_b)
    for l in range(n):
        assert torch.equal(ma.pool_tensors(l)[0], mb.pool_tensors(l)[0])
        assert torch.equal(ma.pool_tensors(l)[1], mb.pool_tensors(l)[1])
        assert ma.check_device_errors(l) == 0
    if runner == "graph":
        r.close()
