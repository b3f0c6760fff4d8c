"""Helpers for the GPU parity tests: put a FragmentedCase into the product
(through the public Python API over the C ABI) exactly as the checkers build
it, run one step, and compare."""
import numpy as np
import torch

from genllm_b200.paged_attention import PagedAttentionManager, paged_attention

# Tolerance of the path (bf16 inputs, fp32 accumulation), two separate
# bounds: max |got - want| <= ATOL over every element, and
# max |got - want| / |want| <= RTOL over the elements with |want| >= REL_FLOOR
# (below it the relative error of a value near zero says nothing about the
# kernel; the absolute bound still covers those elements).
ATOL = 2e-3
RTOL = 1e-2
REL_FLOOR = 1e-3


def to_dev_bf16(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def build_state(case, device=0, layer=0, mgr=None):
    """Manager whose layer holds the case's fragmented cache (before the step)."""
    m = mgr or PagedAttentionManager(device)
    m.init_layer(layer, case.n_kv_heads, case.head_dim)
    m.reserve_layer(layer, case.pool_pages)
    kp, vp = m.pool_tensors(layer)
    kp.copy_(to_dev_bf16(case.k_pool, m.device).view(kp.shape))
    vp.copy_(to_dev_bf16(case.v_pool, m.device).view(vp.shape))
    for w, order in ((0, case.k_free_order), (1, case.v_free_order)):
        p = m.pool(layer, w)
        for _ in range(case.pool_pages):
            p.alloc()
        for i in order:
            p.free(int(i))
    m.set_page_table(layer, case.k_ids, case.v_ids, case.n_prior)
    return m


def run_step(case, out_dtype=torch.float32, causal=True, device=0, mgr=None, layer=0):
    m = build_state(case, device, layer, mgr)
    dev = m.device
    Q = to_dev_bf16(case.q, dev).view(1, case.n_q_heads, case.n_new, case.head_dim)
    K = to_dev_bf16(case.k_new, dev).view(1, case.n_kv_heads, case.n_new, case.head_dim)
    V = to_dev_bf16(case.v_new, dev).view(1, case.n_kv_heads, case.n_new, case.head_dim)
    out = torch.empty((1, case.n_q_heads, case.n_new, case.head_dim), dtype=out_dtype, device=dev)
    paged_attention(m, layer, Q, K, V, out=out, scale=case.scale, causal=causal)
    torch.cuda.synchronize(dev)
    return m, out[0]


def assert_close(got: np.ndarray, want: np.ndarray, what=""):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    max_abs, max_rel = error_bounds(got, want)
    assert max_abs <= ATOL, f"{what}: max abs err {max_abs:.3g} > {ATOL}"
    assert max_rel <= RTOL, f"{what}: max rel err {max_rel:.3g} > {RTOL} (|want| >= {REL_FLOOR})"
    return max_abs


def assert_bf16_close(got_bits: np.ndarray, want_bits: np.ndarray, what=""):
    """bf16 outputs against the reference's bf16 outputs: two roundings of
    values that agree to within the path's tolerance may land one bf16 step
    apart, so each element must be within one unit in the last place or
    within the absolute bound ATOL."""
    g = np.asarray(got_bits, dtype=np.uint16).astype(np.int32)
    w = np.asarray(want_bits, dtype=np.uint16).astype(np.int32)
    assert g.shape == w.shape, (g.shape, w.shape)
    # bf16 bit patterns -> monotonic integer line (sign-magnitude to two's complement)
    key = lambda b: np.where(b & 0x8000, -(b & 0x7FFF), b & 0x7FFF)
    ulps = np.abs(key(g) - key(w))
    f = lambda b: (b.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    diff = np.abs(f(g) - f(w))
    # Near zero an ulp is tiny: there the absolute bound applies instead.
    bad = (ulps > 1) & (diff > ATOL)
    assert not bad.any(), (f"{what}: {int(bad.sum())} elements more than 1 bf16 ulp and {ATOL} apart "
                           f"(max {diff[bad].max():.3g})")
    return int(ulps.max())


def error_bounds(got, want):
    """(max abs error, max rel error over |want| >= REL_FLOOR)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    err = np.abs(got - want)
    big = np.abs(want) >= REL_FLOOR
    max_rel = float((err[big] / np.abs(want[big])).max()) if big.any() else 0.0
    return (float(err.max()) if err.size else 0.0), max_rel
