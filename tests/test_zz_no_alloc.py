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


def test_static_scratch_decode_matches_managed_entry_point():
    hq, hkv, d = 32, 8, 128
    case = fragmented_case(808, hq, hkv, d, 4095, 300)
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
        st = L.gkv_paged_decode_static_scratch(C.byref(pool), C.c_void_p(table.data_ptr()), n_prior,
                                               C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()),
                                               C.c_void_p(v.data_ptr()), C.c_void_p(got.data_ptr()), hq,
                                               C.c_float(case.scale), _lib.GKV_F32, None)
        assert st == 0, L.gkv_last_error()
        torch.cuda.synchronize()
        assert_close(got.cpu().numpy(), want[0, :, 0].cpu().numpy(), f"static scratch, call {step + 1}")
        assert np.array_equal(bits_of(kp2), bits_of(kp)) and np.array_equal(bits_of(vp2), bits_of(vp))
    assert len(m.get_layer(0).page_table) == 257  # the second call opened a new page


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
