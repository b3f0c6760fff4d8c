"""GPU parity of the CUDA path against the CPU oracle and the reference's
golden outputs, through the public API (Python -> C ABI -> sm_100a kernels).

Bars: the append (pool bytes) and the page tables are bit-exact; attention
outputs are within max-abs 2e-3 and max-rel 1e-2 (gpu_util.assert_close) of the oracle's fp32
values (bf16 inputs, fp32 accumulation)."""
import os

import numpy as np
import pytest
import torch

from genllm_b200._lib import GkvError
from genllm_b200.paged_attention import PagedAttentionManager, paged_attention
from genllm_b200.synth import bf16_to_f32, fragmented_case
from golden_util import SMALL, load_config1, load_small, sha
from gpu_util import assert_bf16_close, assert_close, bits_of, build_state, run_step, to_dev_bf16
from oracle.oracle import Oracle, run_oracle_case

pytestmark = pytest.mark.gpu
ORC = Oracle()
NPROC = os.cpu_count() or 1


def check_case(case, causal, golden_bf16=None):
    o_out, o_kp, o_vp, o_k, o_v, o_n = run_oracle_case(case, ORC, causal, threads=min(NPROC, 32))
    m, out = run_step(case, torch.float32, causal)
    err = assert_close(out.cpu().numpy(), o_out, "fp32 out")
    kp, vp = m.pool_tensors(0)
    assert np.array_equal(bits_of(kp).reshape(o_kp.shape), o_kp), "K pool bytes differ after append"
    assert np.array_equal(bits_of(vp).reshape(o_vp.shape), o_vp), "V pool bytes differ after append"
    L = m.get_layer(0)
    assert L.num_cached == o_n
    assert [e.k_block_id for e in L.page_table] == o_k.tolist()
    assert [e.v_block_id for e in L.page_table] == o_v.tolist()
    dk, dv = m.device_table(0)
    assert dk == o_k.tolist() and dv == o_v.tolist(), "device table differs from host table"
    assert m.check_device_errors(0) == 0
    if golden_bf16 is not None:
        m2, out2 = run_step(case, torch.bfloat16, causal)
        assert_bf16_close(bits_of(out2), golden_bf16, "bf16 out vs reference")
    return err


@pytest.mark.parametrize("name", [n for n, _, _ in SMALL])
def test_golden_cases(name):
    case, causal, z = load_small(name)
    check_case(case, causal, z["out_bf16"])


def test_config1_qwen3_0p6b_layer():
    case, causal, z = load_config1()
    check_case(case, causal, z["out_bf16"])


@pytest.mark.parametrize("ctx", [4096, 32768])
def test_config3_qwen3_4b_layer(ctx):
    case = fragmented_case(7, 32, 8, 128, ctx, 4096)
    check_case(case, True)


@pytest.mark.parametrize("g,hkv", [(1, 8), (2, 8), (4, 8), (8, 2), (4, 1), (2, 3)])
@pytest.mark.parametrize("n_prior", [15, 16, 17, 255, 1000])
def test_group_sizes_and_boundaries(g, hkv, n_prior):
    case = fragmented_case(1000 + n_prior + g, g * hkv, hkv, 128, n_prior, (n_prior + 16) // 16 + 5)
    check_case(case, True)


def test_poisoned_unused_slots():
    """NaN bit patterns in every slot no table entry covers: a kernel reading
    past the valid tokens would produce NaN."""
    case = fragmented_case(21, 32, 8, 128, 999, 80, poison_unused=True)
    check_case(case, True)


@pytest.mark.parametrize("n_prior,n_new,causal", [(0, 1, True), (5, 40, True), (16, 16, True), (100, 77, False),
                                                  (3, 600, True), (128, 200, True), (256, 77, False),
                                                  (640, 129, True)])
def test_chunk_paths(n_prior, n_new, causal):
    """Chunks that start on a 128-token tile boundary read their own KV tiles
    from the chunk's inputs (the append runs beside the attention); the
    others read every tile from the pages."""
    case = fragmented_case(300 + n_new, 16, 8, 128, n_prior, (n_prior + n_new) // 16 + 4, n_new=n_new)
    check_case(case, causal)


@pytest.mark.parametrize("g,hkv", [(1, 8), (4, 8), (8, 2), (8, 1), (2, 3), (1, 5)])
@pytest.mark.parametrize("causal", [True, False])
def test_chunk_group_sizes(g, hkv, causal):
    """The chunk path (tensor-core prefill) at every group size and at kv
    head counts that are not a power of two, with the context ending mid-page."""
    case = fragmented_case(400 + 10 * g + hkv, g * hkv, hkv, 128, 203, (203 + 150) // 16 + 5, n_new=150,
                           poison_unused=True)
    check_case(case, causal)


@pytest.mark.parametrize("n_prior", [40, 128])
def test_long_chunk_over_1024_tokens(n_prior):
    """Chunks longer than one append launch carries (64 pages) are split
    (from a tile boundary: several appends, the last one beside the
    attention)."""
    case = fragmented_case(77, 4, 2, 128, n_prior, 200, n_new=1500)
    check_case(case, True)


def test_multi_step_decode_sequence():
    """40 decode steps from an empty cache; each step checked against the
    oracle's state evolving in lockstep."""
    hq, hkv, d, pool = 8, 2, 128, 6
    rng = np.random.default_rng(5)
    m = PagedAttentionManager(0)
    m.init_layer(0, hkv, d)
    m.reserve_layer(0, pool)
    from oracle.oracle import OraclePool
    from genllm_b200.synth import randn_bf16
    op = OraclePool(pool, ORC)
    kp = np.zeros((pool, 16, hkv, d), np.uint16)
    vp = np.zeros((pool, 16, hkv, d), np.uint16)
    for step in range(40):
        q = randn_bf16(rng, (hq, 1, d))
        kn = randn_bf16(rng, (hkv, 1, d))
        vn = randn_bf16(rng, (hkv, 1, d))
        out = torch.empty((1, hq, 1, d), dtype=torch.float32, device="cuda")
        paged_attention(m, 0, to_dev_bf16(q, "cuda").view(1, hq, 1, d), to_dev_bf16(kn, "cuda").view(1, hkv, 1, d),
                        to_dev_bf16(vn, "cuda").view(1, hkv, 1, d), out=out)
        op.append_kv(kp, vp, kn, vn, hkv, 1, d)
        k_ids, v_ids = op.table()
        want = ORC.paged_attention_f32(q, kp, vp, k_ids, v_ids, op.num_cached, hq, hkv, 1, d, 1 / np.sqrt(d))
        torch.cuda.synchronize()
        assert_close(out[0].cpu().numpy(), want, f"step {step}")
        L = m.get_layer(0)
        assert [e.k_block_id for e in L.page_table] == k_ids.tolist()
    gk, gv = m.pool_tensors(0)
    gkb, gvb = bits_of(gk), bits_of(gv)
    for pos in range(op.num_cached):  # every written row, bit for bit
        lp, slot = divmod(pos, 16)
        assert np.array_equal(gkb[k_ids[lp], slot], kp[k_ids[lp], slot])
        assert np.array_equal(gvb[v_ids[lp], slot], vp[v_ids[lp], slot])


def test_reset_then_reuse_lifo():
    case = fragmented_case(31, 8, 2, 128, 64, 10)
    m, _ = run_step(case)
    before = m.get_layer(0)
    m.reset()
    L = m.get_layer(0)
    assert L.num_cached == 0 and L.page_table == []
    # After reset every page handed out is free, ascending; the next page is the highest id.
    assert m.pool(0, 0).num_free() == m.pool(0, 0).num_blocks()
    hq, hkv, d = 8, 2, 128
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, hq, 1, d)).astype(np.float32)
    Q = torch.from_numpy(q).to(torch.bfloat16).cuda()
    K = torch.randn(1, hkv, 1, d, device="cuda").to(torch.bfloat16)
    V = torch.randn(1, hkv, 1, d, device="cuda").to(torch.bfloat16)
    out = paged_attention(m, 0, Q, K, V)
    torch.cuda.synchronize()
    L = m.get_layer(0)
    assert L.num_cached == 1 and L.page_table[0].k_block_id == m.pool(0, 0).num_blocks() - 1
    # One token: the output is V itself (softmax over a single score).
    want = V[0].float().repeat_interleave(hq // hkv, dim=0)
    assert_close(out[0].float().cpu().numpy(), want.cpu().numpy(), "single token")
    assert before.num_cached == 65


def test_pool_exhaustion_leaves_state_unchanged():
    case = fragmented_case(41, 8, 2, 128, 32, 2)  # both pages used; the step needs a third
    m = build_state(case)
    Q = to_dev_bf16(case.q, "cuda").view(1, 8, 1, 128)
    K = to_dev_bf16(case.k_new, "cuda").view(1, 2, 1, 128)
    V = to_dev_bf16(case.v_new, "cuda").view(1, 2, 1, 128)
    with pytest.raises(GkvError) as e:
        paged_attention(m, 0, Q, K, V, out=torch.empty(1, 8, 1, 128, device="cuda"))
    assert e.value.status == 2
    L = m.get_layer(0)
    assert L.num_cached == 32 and len(L.page_table) == 2


def test_unsupported_shapes_rejected():
    m = PagedAttentionManager(0)
    m.init_layer(0, 2, 128)
    m.reserve_layer(0, 4)
    Q = torch.zeros(2, 8, 1, 128, dtype=torch.bfloat16, device="cuda")
    K = torch.zeros(2, 2, 1, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(GkvError):
        paged_attention(m, 0, Q, K, K)  # batch 2
    Q = torch.zeros(1, 6, 1, 128, dtype=torch.bfloat16, device="cuda")
    K = torch.zeros(1, 2, 1, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(GkvError):
        paged_attention(m, 0, Q, K, K)  # group size 3
    m.init_layer(1, 2, 64)
    m.reserve_layer(1, 4)
    Q = torch.zeros(1, 4, 1, 64, dtype=torch.bfloat16, device="cuda")
    K = torch.zeros(1, 2, 1, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(GkvError):
        paged_attention(m, 1, Q, K, K)  # head_dim 64
    with pytest.raises(GkvError):
        paged_attention(m, 7, Q, K, K)  # unknown layer
    assert m.get_layer(0).num_cached == 0


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_output_dtypes(dt):
    case = fragmented_case(51, 16, 8, 128, 500, 40)
    want = run_oracle_case(case, ORC)[0]
    _, out = run_step(case, dt)
    assert_close(out.float().cpu().numpy(), want, str(dt))


def test_unpublished_table_flags_device_error():
    """Raw tier: attending over table entries that were never published (the
    table starts as -1) skips those pages and sets the bad-page bit; nothing
    faults and the context stays usable."""
    import ctypes as C
    from genllm_b200 import _lib
    L = _lib.lib()
    t = C.c_void_p()
    _lib.check(L.gkv_table_create(0, 8, C.byref(t)))
    kp = torch.zeros(8, 16, 2, 128, dtype=torch.bfloat16, device="cuda")
    vp = torch.zeros_like(kp)
    pool = _lib.PoolDesc(kp.data_ptr(), vp.data_ptr(), 8, 2, 128, 30)
    Q = torch.zeros(1, 4, 1, 128, dtype=torch.bfloat16, device="cuda")
    K = torch.zeros(1, 2, 1, 128, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(1, 4, 1, 128, device="cuda")
    _lib.check(L.gkv_paged_attention_raw(C.byref(pool), t, 40, None, Q.data_ptr(), K.data_ptr(), K.data_ptr(),
                                         out.data_ptr(), 4, 1, 0.1, 1, 0, None))
    f = C.c_uint32()
    _lib.check(L.gkv_table_check_errors(t, C.byref(f)))
    assert f.value & 1
    _lib.check(L.gkv_table_destroy(t))
    torch.cuda.synchronize()
    assert torch.isfinite(torch.ones(1, device="cuda")).all()


def test_raw_tier_caller_managed_pages():
    """The raw tier with allocation done by the caller (as the reference's
    BlockPool would) gives the managed tier's results."""
    import ctypes as C
    from genllm_b200 import _lib
    L = _lib.lib()
    case = fragmented_case(61, 16, 8, 128, 200, 20)
    o_out, o_kp, o_vp, o_k, o_v, o_n = run_oracle_case(case, ORC)
    t = C.c_void_p()
    _lib.check(L.gkv_table_create(0, 20, C.byref(t)))
    kp = to_dev_bf16(case.k_pool, "cuda")
    vp = to_dev_bf16(case.v_pool, "cuda")
    pool = _lib.PoolDesc(kp.data_ptr(), vp.data_ptr(), 20, 8, 128, 30)
    # Publish the prior table (13 pages) plus the appended token's page 13 in one delta.
    ks = (C.c_int32 * 13)(*o_k.tolist())
    vs = (C.c_int32 * 13)(*o_v.tolist())
    np_ = _lib.NewPages(0, 13, ks, vs)
    Q = to_dev_bf16(case.q, "cuda")
    K = to_dev_bf16(case.k_new, "cuda")
    V = to_dev_bf16(case.v_new, "cuda")
    out = torch.empty(16, 1, 128, device="cuda")
    _lib.check(L.gkv_paged_attention_raw(C.byref(pool), t, 200, C.byref(np_), Q.data_ptr(), K.data_ptr(),
                                         V.data_ptr(), out.data_ptr(), 16, 1, case.scale, 1, 0, None))
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), o_out, "raw tier")
    assert np.array_equal(bits_of(kp).reshape(o_kp.shape), o_kp)
    f = C.c_uint32()
    _lib.check(L.gkv_table_check_errors(t, C.byref(f)))
    assert f.value == 0
    _lib.check(L.gkv_table_destroy(t))


def test_append_only_bit_exact():
    """append_kv_from_tensor alone (prefill-style append, 70 tokens across pages)."""
    case = fragmented_case(71, 8, 4, 128, 9, 12, n_new=70)
    m = build_state(case)
    K = to_dev_bf16(case.k_new, "cuda").view(1, 4, 70, 128)
    V = to_dev_bf16(case.v_new, "cuda").view(1, 4, 70, 128)
    m.append_kv_from_tensor(0, K, V)
    torch.cuda.synchronize()
    _, o_kp, o_vp, o_k, o_v, o_n = run_oracle_case(case, ORC)
    kp, vp = m.pool_tensors(0)
    assert np.array_equal(bits_of(kp).reshape(o_kp.shape), o_kp)
    assert np.array_equal(bits_of(vp).reshape(o_vp.shape), o_vp)
    assert m.get_layer(0).num_cached == o_n
    assert m.device_table(0)[0] == o_k.tolist()


def test_config4_chunked_prefill_qwen3_1p7b():
    """Config 4: an 8192-token prompt in 16 chunks of 512 (Hq 16, Hkv 8),
    each chunk appended into 16-token pages and attended causally over all
    prior pages on the tensor cores. Every chunk's pool bytes are bit-exact
    against the restated appender; 48 output rows per chunk (first, last and
    random rows of random heads) are checked against the oracle."""
    from genllm_b200.synth import randn_bf16
    from oracle.oracle import OraclePool
    hq, hkv, d, chunk, n_chunks = 16, 8, 128, 512, 16
    pool_pages = chunk * n_chunks // 16 + 8
    rng = np.random.default_rng(4)
    m = PagedAttentionManager(0)
    m.init_layer(0, hkv, d)
    m.reserve_layer(0, pool_pages)
    for t in m.pool_tensors(0):  # fresh device memory is not zeroed; the restated pools are
        t.zero_()
    op = OraclePool(pool_pages, ORC)
    kp = np.zeros((pool_pages, 16, hkv, d), np.uint16)
    vp = np.zeros((pool_pages, 16, hkv, d), np.uint16)
    scale = 1 / np.sqrt(d)
    for c in range(n_chunks):
        q = randn_bf16(rng, (hq, chunk, d))
        kn = randn_bf16(rng, (hkv, chunk, d))
        vn = randn_bf16(rng, (hkv, chunk, d))
        out = torch.empty((1, hq, chunk, d), dtype=torch.float32, device="cuda")
        paged_attention(m, 0, to_dev_bf16(q, "cuda").view(1, hq, chunk, d),
                        to_dev_bf16(kn, "cuda").view(1, hkv, chunk, d),
                        to_dev_bf16(vn, "cuda").view(1, hkv, chunk, d), out=out, scale=scale)
        op.append_kv(kp, vp, kn, vn, hkv, chunk, d)
        k_ids, v_ids = op.table()
        rows = np.concatenate([[0, chunk - 1, hq * chunk - 1], rng.integers(0, hq * chunk, 45)]).astype(np.int32)
        want = ORC.paged_attention_rows(q, kp, vp, k_ids, v_ids, op.num_cached, hq, hkv, chunk, d, scale, rows,
                                        threads=min(NPROC, 32))
        torch.cuda.synchronize()
        got = out[0].reshape(hq * chunk, d).cpu().numpy()[rows]
        assert_close(got, want, f"chunk {c}")
    gk, gv = m.pool_tensors(0)
    assert np.array_equal(bits_of(gk), kp) and np.array_equal(bits_of(gv), vp)
    assert m.check_device_errors(0) == 0


def test_prefill_kernels_agree_simt_subprocess():
    """The CUDA-core prefill kernel (GKV_PREFILL_KERNEL=simt) is an
    independent second implementation; both must match the oracle."""
    import subprocess
    import sys
    code = (
        "import sys; sys.path.insert(0, %r); sys.path.insert(0, %r)\n"
        "from test_gpu_parity import check_case\n"
        "from genllm_b200.synth import fragmented_case\n"
        "check_case(fragmented_case(401, 16, 8, 128, 70, 30, n_new=130), True)\n"
        "check_case(fragmented_case(402, 8, 2, 128, 5, 20, n_new=77), False)\n"
        "print('simt ok')\n" % (os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                os.path.dirname(os.path.abspath(__file__))))
    env = dict(os.environ, GKV_PREFILL_KERNEL="simt")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "simt ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.parametrize("n_prior,n_new,causal", [(0, 128, True), (1, 255, True), (127, 129, False),
                                                  (300, 384, True), (2000, 130, True)])
def test_prefill_tile_edges(n_prior, n_new, causal):
    """Query tiles of exactly / one past 128 rows, KV tiles ending mid-page."""
    case = fragmented_case(500 + n_new, 16, 8, 128, n_prior, (n_prior + n_new) // 16 + 3, n_new=n_new,
                           poison_unused=True)
    check_case(case, causal)


@pytest.mark.parametrize("order", ["asc", "desc", "broken", "kv_mismatch"])
@pytest.mark.parametrize("n_prior,n_new,causal", [(1000, 300, True), (2040, 130, True), (517, 256, False)])
def test_prefill_page_runs(order, n_prior, n_new, causal):
    """Tiles whose 8 pages have consecutive ids are copied as one run
    (ascending, or descending and reversed in shared memory); interrupted
    runs and K/V tables that disagree fall back to page-by-page copies.
    Contexts ending mid-page and causal diagonals cross reversed tiles."""
    case = fragmented_case(600 + n_new, 16, 8, 128, n_prior, (n_prior + n_new) // 16 + 24, n_new=n_new,
                           poison_unused=True, page_order=order)
    check_case(case, causal)



def test_decode_layers_one_call_matches_per_layer_calls():
    """gkv_decode_layers (one host call for a token through several layers)
    launches exactly what per-layer gkv_paged_attention calls launch."""
    from genllm_b200.paged_attention import DecodeStep
    cases = [fragmented_case(900 + l, 16, 8, 128, 300 + 37 * l, 40) for l in range(3)]
    ma = PagedAttentionManager(0)
    mb = PagedAttentionManager(0)
    outs_a, outs_b, ins = [], [], []
    for l, c in enumerate(cases):
        build_state(c, mgr=ma, layer=l)
        build_state(c, mgr=mb, layer=l)
        q = to_dev_bf16(c.q, ma.device).view(16, 128)
        k = to_dev_bf16(c.k_new, ma.device).view(8, 128)
        v = to_dev_bf16(c.v_new, ma.device).view(8, 128)
        ins.append((q, k, v))
        outs_a.append(torch.empty((16, 128), dtype=torch.bfloat16, device=ma.device))
        outs_b.append(torch.empty((1, 16, 1, 128), dtype=torch.bfloat16, device=mb.device))
    step = DecodeStep(ma, [0, 1, 2], [i[0] for i in ins], [i[1] for i in ins], [i[2] for i in ins], outs_a, 16,
                      cases[0].scale)
    step.run()
    for l, (q, k, v) in enumerate(ins):
        paged_attention(mb, l, q.view(1, 16, 1, 128), k.view(1, 8, 1, 128), v.view(1, 8, 1, 128), out=outs_b[l],
                        scale=cases[0].scale)
    torch.cuda.synchronize()
    for l in range(3):
        assert torch.equal(outs_a[l].view(-1), outs_b[l].view(-1))
        ka, va = ma.pool_tensors(l)
        kb, vb = mb.pool_tensors(l)
        assert torch.equal(ka, kb) and torch.equal(va, vb)
        assert ma.get_layer(l).num_cached == mb.get_layer(l).num_cached == cases[l].n_prior + 1
