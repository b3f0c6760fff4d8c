"""The no-allocation decode entry point, gkv_paged_decode_static_scratch.

It exists for callers that may not allocate device memory (a host framework
that owns every allocation through its own arena, or a latency-critical loop
that cannot pay for cudaMalloc), and keeps its split-K scratch in a fixed
array inside the library. Here it is called through the C ABI on two decode
steps in a row — the second one opening a new page — and each output must
match the regular managed entry point (gkv_paged_attention) on the same cache
within the tolerance of the other parity tests, with identical appended pool
bytes. This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest
import torch

from genllm_b200 import _lib
from genllm_b200.paged_attention import paged_attention
from genllm_b200.synth import fragmented_case, randn_bf16
from gpu_util import assert_close, bits_of, build_state, to_dev_bf16

pytestmark = pytest.mark.gpu


def _static_decode(L, pool, table, n_prior, q, k, v, got, hq, scale):
    return L.gkv_paged_decode_static_scratch(C.byref(pool), C.c_void_p(table.data_ptr()), n_prior,
                                             C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()),
                                             C.c_void_p(v.data_ptr()), C.c_void_p(got.data_ptr()), hq,
                                             C.c_float(scale), _lib.GKV_F32, None)


def _errors(L):
    flags = C.c_uint32(0xFFFFFFFF)
    assert L.gkv_paged_decode_static_scratch_errors(C.byref(flags), None) == 0, L.gkv_last_error()
    return flags.value


@pytest.mark.parametrize("hq,n_prior,pool_pages", [(32, 4095, 300), (64, 2000 * 16 - 1, 2100)],
                         ids=["hq32-256pages", "hq64-2000pages"])
def test_static_scratch_decode_matches_managed_entry_point(hq, n_prior, pool_pages):
    """Two calls in a row against gkv_paged_attention on the same cache.
    hq64: group 8, where the 4096 static partial rows cap the splits at 64,
    so each split covers ~31 pages of the 2000-page context."""
    hkv, d = 8, 128
    case = fragmented_case(808, hq, hkv, d, n_prior, pool_pages)
    m = build_state(case)
    kp, vp = m.pool_tensors(0)
    kp2, vp2 = kp.clone(), vp.clone()  # the static-scratch path's own copy of the cache
    pool = _lib.PoolDesc(kp2.data_ptr(), vp2.data_ptr(), case.pool_pages, hkv, d, _lib.GKV_BF16)
    rng = np.random.default_rng(9)
    L = _lib.lib()
    for step in range(2):
        n_prior = case.n_prior + step
        q = to_dev_bf16(randn_bf16(rng, (hq, 1, d)), "cuda")
        k = to_dev_bf16(randn_bf16(rng, (hkv, 1, d)), "cuda")
        v = to_dev_bf16(randn_bf16(rng, (hkv, 1, d)), "cuda")
        want = torch.empty(1, hq, 1, d, device="cuda")
        paged_attention(m, 0, q.view(1, hq, 1, d), k.view(1, hkv, 1, d), v.view(1, hkv, 1, d), out=want,
                        scale=case.scale)
        lay = m.get_layer(0)
        table = torch.tensor([[e.k_block_id, e.v_block_id] for e in lay.page_table], dtype=torch.int32,
                             device="cuda")
        got = torch.full((hq, d), float("nan"), device="cuda")
        torch.cuda.synchronize()
        free0, alloc0 = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
        st = _static_decode(L, pool, table, n_prior, q, k, v, got, hq, case.scale)
        assert st == 0, L.gkv_last_error()
        torch.cuda.synchronize()
        if step == 1:  # after the first call's one-time set-up, a call takes no device memory
            assert torch.cuda.mem_get_info()[0] == free0 and torch.cuda.memory_allocated() == alloc0
        assert _errors(L) == 0
        assert_close(got.cpu().numpy(), want[0, :, 0].cpu().numpy(), f"static scratch, call {step + 1}")
        assert np.array_equal(bits_of(kp2), bits_of(kp)) and np.array_equal(bits_of(vp2), bits_of(vp))
    assert len(m.get_layer(0).page_table) == (n_prior + 1) // 16 + 1  # the second call opened a new page


def test_static_scratch_reports_bad_page_id():
    """A page id outside the pool in device_table: the call returns normally,
    the page is skipped, and the error reader shows the bad-page bit; the
    next call clears it."""
    hq, hkv, d = 16, 8, 128
    case = fragmented_case(31, hq, hkv, d, 100, 16)
    m = build_state(case)
    kp, vp = m.pool_tensors(0)
    pool = _lib.PoolDesc(kp.data_ptr(), vp.data_ptr(), case.pool_pages, hkv, d, _lib.GKV_BF16)
    lay = m.get_layer(0)
    ids = [[e.k_block_id, e.v_block_id] for e in lay.page_table]
    L = _lib.lib()
    rng = np.random.default_rng(3)
    q = to_dev_bf16(randn_bf16(rng, (hq, 1, d)), "cuda")
    k = to_dev_bf16(randn_bf16(rng, (hkv, 1, d)), "cuda")
    got = torch.empty((hq, d), device="cuda")
    bad = [list(r) for r in ids[:7]]
    bad[2][1] = case.pool_pages + 5  # V id of logical page 2 out of range
    table = torch.tensor(bad, dtype=torch.int32, device="cuda")
    assert _static_decode(L, pool, table, 100, q, k, k, got, hq, case.scale) == 0, L.gkv_last_error()
    assert _errors(L) & 1
    good = torch.tensor([list(r) for r in ids[:7]], dtype=torch.int32, device="cuda")
    assert _static_decode(L, pool, good, 100, q, k, k, got, hq, case.scale) == 0, L.gkv_last_error()
    assert _errors(L) == 0


def test_static_scratch_rejects_oversized_requests():
    L = _lib.lib()
    kp = torch.zeros(4, 16, 8, 128, dtype=torch.bfloat16, device="cuda")
    pool = _lib.PoolDesc(kp.data_ptr(), kp.data_ptr(), 4, 8, 128, _lib.GKV_BF16)
    dummy = torch.zeros(64, 128, dtype=torch.bfloat16, device="cuda")
    table = torch.zeros(8, 2, dtype=torch.int32, device="cuda")
    p = C.c_void_p(dummy.data_ptr())
    # 10M cached tokens: more pages than the fixed scratch's splits can cover.
    st = L.gkv_paged_decode_static_scratch(C.byref(pool), C.c_void_p(table.data_ptr()), 10_000_000, p, p, p, p, 64,
                                           C.c_float(0.1), _lib.GKV_F32, None)
    assert st == _lib.GKV_ERR_INVALID and b"static scratch" in L.gkv_last_error()
    st = L.gkv_paged_decode_static_scratch(C.byref(pool), C.c_void_p(table.data_ptr()), 10, p, p, p, p, 24,
                                           C.c_float(0.1), _lib.GKV_F32, None)
    assert st == _lib.GKV_ERR_UNSUPPORTED  # group size 3
