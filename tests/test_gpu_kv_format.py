"""KV format export / import on the GPU (gkv_export_kv / gkv_import_kv),
bit-exact against the committed fixtures (pages from the reference's own
append) and the oracle (oracle/kv_format_oracle.c): bf16 head-major export,
e4m3 export (bytes and block scales), e4m3 import; ragged lengths, fragmented
and descending tables, edge values (zero, subnormal, infinite, NaN blocks);
full size (Qwen3-4B layer at 32k tokens) through size-independent properties."""
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

from cases import KV_FORMAT  # noqa: E402
from genllm_b200._lib import GKV_ERR_INVALID, GkvError  # noqa: E402
from genllm_b200.paged_attention import PagedAttentionManager  # noqa: E402
from genllm_b200.synth import fragmented_case, kv_format_values  # noqa: E402
from golden_util import GOLDEN  # noqa: E402
from gpu_util import bits_of, to_dev_bf16  # noqa: E402
from oracle.oracle import Oracle  # noqa: E402

pytestmark = pytest.mark.gpu
ORC = Oracle()


def u8_of(t):
    return t.contiguous().view(torch.uint8).cpu().numpy()


def f32_bits(t):
    return t.contiguous().cpu().numpy().view(np.uint32)


def manager_with_pages(k_pool, v_pool, k_ids, v_ids, n_tokens, hkv, pool_pages, device=0):
    """A manager whose layer 0 holds these pages and this table."""
    m = PagedAttentionManager(device)
    m.init_layer(0, hkv, 128)
    m.reserve_layer(0, pool_pages)
    kp, vp = m.pool_tensors(0)
    kp.copy_(to_dev_bf16(np.asarray(k_pool).reshape(-1), m.device).view(kp.shape))
    vp.copy_(to_dev_bf16(np.asarray(v_pool).reshape(-1), m.device).view(vp.shape))
    for w, ids in ((0, k_ids), (1, v_ids)):
        p = m.pool(0, w)
        for _ in range(pool_pages):
            p.alloc()
        used = set(int(i) for i in ids)
        for i in range(pool_pages):
            if i not in used:
                p.free(i)
    m.set_page_table(0, list(k_ids), list(v_ids), n_tokens)
    return m


@pytest.mark.parametrize("name,seed,hkv,chunks,pages", KV_FORMAT)
def test_export_golden(name, seed, hkv, chunks, pages):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    K, V = kv_format_values(seed, hkv, sum(chunks))
    n = int(z["num_cached"])
    m = manager_with_pages(z["k_pool"], z["v_pool"], z["k_ids"], z["v_ids"], n, hkv, pages)
    ko, vo = m.export_kv(0)
    kq, vq, ks, vs = m.export_kv(0, fp8=True)
    torch.cuda.synchronize()
    assert np.array_equal(bits_of(ko), K) and np.array_equal(bits_of(vo), V), "bf16 export differs"
    assert np.array_equal(u8_of(kq), z["k_fp8"]) and np.array_equal(u8_of(vq), z["v_fp8"]), "e4m3 bytes differ"
    assert np.array_equal(f32_bits(ks), z["k_scales"].view(np.uint32)), "K block scales differ"
    assert np.array_equal(f32_bits(vs), z["v_scales"].view(np.uint32)), "V block scales differ"
    assert m.check_device_errors(0) == 0


@pytest.mark.parametrize("n,hkv,order", [(1, 8, "random"), (15, 2, "random"), (16, 8, "desc"), (17, 1, "asc"),
                                         (257, 8, "broken"), (4099, 8, "random"), (1000, 4, "kv_mismatch")])
def test_export_matches_oracle(n, hkv, order):
    c = fragmented_case(900 + n, hkv, hkv, 128, n, n // 16 + 5, page_order=order, poison_unused=True)
    # magnitudes per block and edge values, written into the case's pages
    K, V = kv_format_values(950 + n, hkv, n)
    kp = c.k_pool.reshape(c.pool_pages, 16, hkv, 128)
    vp = c.v_pool.reshape(c.pool_pages, 16, hkv, 128)
    for t in range(n):
        kp[c.k_ids[t // 16], t % 16] = K[:, t]
        vp[c.v_ids[t // 16], t % 16] = V[:, t]
    m = manager_with_pages(kp, vp, c.k_ids, c.v_ids, n, hkv, c.pool_pages)
    ko, vo = m.export_kv(0)
    kq, vq, ks, vs = m.export_kv(0, fp8=True)
    torch.cuda.synchronize()
    assert np.array_equal(bits_of(ko), K) and np.array_equal(bits_of(vo), V)
    okq, ovq, oks, ovs = ORC.export_kv(kp, vp, c.k_ids, c.v_ids, n, hkv, fp8=True)
    assert np.array_equal(u8_of(kq), okq) and np.array_equal(u8_of(vq), ovq)
    assert np.array_equal(f32_bits(ks), oks.view(np.uint32)) and np.array_equal(f32_bits(vs), ovs.view(np.uint32))
    assert m.check_device_errors(0) == 0


@pytest.mark.parametrize("n_prior,s,hkv", [(0, 37, 2), (23, 29, 8), (16, 16, 8), (5, 1, 4), (0, 1030, 8)])
def test_import_fp8_matches_oracle(n_prior, s, hkv):
    rng = np.random.default_rng(n_prior * 7 + s)
    pages = (n_prior + s) // 16 + 4
    c = fragmented_case(990 + s, hkv, hkv, 128, n_prior, pages)
    q = rng.integers(0, 256, size=(2, hkv, s, 128)).astype(np.uint8)
    q[q & 0x7F == 0x7F] = 0x3C  # no NaN codes: NaN payloads are not part of the contract
    scales = (2.0 ** rng.integers(-12, 12, size=(2, hkv, (s + 15) // 16))).astype(np.float32)
    scales[0, 0, 0] = 1e-38  # products below the bf16 normal range flush to signed zero
    m = manager_with_pages(c.k_pool, c.v_pool, c.k_ids, c.v_ids, n_prior, hkv, pages)
    dev = m.device
    kq = torch.from_numpy(q[0]).to(dev).view(torch.float8_e4m3fn)
    vq = torch.from_numpy(q[1]).to(dev).view(torch.float8_e4m3fn)
    m.import_kv(0, kq, vq, torch.from_numpy(scales[0]).to(dev), torch.from_numpy(scales[1]).to(dev))
    torch.cuda.synchronize()
    k_ids, v_ids = m.page_table(0)
    assert m.get_layer(0).num_cached == n_prior + s
    okp = c.k_pool.reshape(pages, 16, hkv, 128).copy()
    ovp = c.v_pool.reshape(pages, 16, hkv, 128).copy()
    ORC.import_fp8(okp, ovp, k_ids, v_ids, n_prior, q[0], q[1], scales[0], scales[1])
    kp, vp = m.pool_tensors(0)
    assert np.array_equal(bits_of(kp).reshape(okp.shape), okp), "K pages differ"
    assert np.array_equal(bits_of(vp).reshape(ovp.shape), ovp), "V pages differ"
    assert m.check_device_errors(0) == 0


def test_round_trips_through_a_second_manager():
    """export -> import into a fresh layer reproduces the tokens: bf16 exactly,
    e4m3 as the oracle's dequantisation of the exported bytes."""
    hkv, n = 8, 333
    K, V = kv_format_values(77, hkv, n)
    a = PagedAttentionManager(0)
    a.init_layer(0, hkv, 128)
    a.reserve_layer(0, 32)
    a.append_kv_from_tensor(0, to_dev_bf16(K, a.device), to_dev_bf16(V, a.device))
    ko, vo = a.export_kv(0)
    kq, vq, ks, vs = a.export_kv(0, fp8=True)
    b = PagedAttentionManager(0)
    for layer, args in ((0, (ko, vo)), (1, (kq, vq, ks, vs))):
        b.init_layer(layer, hkv, 128)
        b.reserve_layer(layer, 32)
        b.import_kv(layer, *args)
    k2, v2 = b.export_kv(0)
    k3, v3 = b.export_kv(1)
    torch.cuda.synchronize()
    assert np.array_equal(bits_of(k2), K) and np.array_equal(bits_of(v2), V)
    kp, vp = np.zeros((32, 16, hkv, 128), np.uint16), np.zeros((32, 16, hkv, 128), np.uint16)
    ids = np.arange(32, dtype=np.int32)
    ORC.import_fp8(kp, vp, ids, ids, 0, u8_of(kq), u8_of(vq), ks.cpu().numpy(), vs.cpu().numpy())
    want_k, want_v, _, _ = ORC.export_kv(kp, vp, ids, ids, n, hkv)
    assert np.array_equal(bits_of(k3), want_k) and np.array_equal(bits_of(v3), want_v)


def test_export_after_host_only_growth_and_empty():
    """Pages grown with append_kv_pages reach the device table before the
    export; an empty layer exports nothing."""
    hkv = 2
    m = PagedAttentionManager(0)
    m.init_layer(0, hkv, 128)
    m.reserve_layer(0, 8)
    ko, vo = m.export_kv(0)
    assert ko.shape == (hkv, 0, 128)
    K, V = kv_format_values(78, hkv, 20, special=False)
    m.append_kv_from_tensor(0, to_dev_bf16(K, m.device), to_dev_bf16(V, m.device))
    m.append_kv_pages(0, 30)  # host-only: tokens 20..49, pages 2..3 not yet on the device
    ko, vo = m.export_kv(0)
    torch.cuda.synchronize()
    assert ko.shape == (hkv, 50, 128)
    assert np.array_equal(bits_of(ko)[:, :20], K) and np.array_equal(bits_of(vo)[:, :20], V)
    assert m.device_table(0) == m.page_table(0)
    assert m.check_device_errors(0) == 0


def test_bad_arguments_rejected():
    m = PagedAttentionManager(0)
    m.init_layer(0, 2, 128)
    m.reserve_layer(0, 4)
    K = torch.zeros((2, 4, 128), dtype=torch.float8_e4m3fn, device="cuda:0")
    with pytest.raises(GkvError) as e:
        m.import_kv(0, K, K)  # e4m3 without scales
    assert e.value.status == GKV_ERR_INVALID
    with pytest.raises(GkvError):
        m.import_kv(0, K, K, torch.ones(2, 1, device="cuda:0", dtype=torch.float64),
                    torch.ones(2, 1, device="cuda:0", dtype=torch.float64))
    assert m.get_layer(0).num_cached == 0


def test_full_size_layer_export():
    """Qwen3-4B layer at 32k tokens over a 4096-page fragmented pool: the bf16
    export equals a torch gather of the pages, and the e4m3 export's
    dequantised values stay within the format's error bound."""
    hkv, n, pages = 8, 32768, 4096
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(5)
    m = PagedAttentionManager(0)
    m.init_layer(0, hkv, 128)
    m.reserve_layer(0, pages)
    kp, vp = m.pool_tensors(0)
    kp.copy_(torch.randn(kp.shape, generator=g, device=dev).to(torch.bfloat16))
    vp.copy_(torch.randn(vp.shape, generator=g, device=dev).to(torch.bfloat16))
    perm_k = torch.randperm(pages, generator=torch.Generator().manual_seed(1))[: n // 16]
    perm_v = torch.randperm(pages, generator=torch.Generator().manual_seed(2))[: n // 16]
    for w in (0, 1):
        p = m.pool(0, w)
        for _ in range(pages):
            p.alloc()
    m.set_page_table(0, perm_k.tolist(), perm_v.tolist(), n)
    ko, vo = m.export_kv(0)
    kq, vq, ks, vs = m.export_kv(0, fp8=True)
    torch.cuda.synchronize()
    for pool, perm, out, q, s in ((kp, perm_k, ko, kq, ks), (vp, perm_v, vo, vq, vs)):
        want = pool[perm.to(dev)].permute(2, 0, 1, 3).reshape(hkv, n, 128)
        assert torch.equal(out.view(torch.int16), want.contiguous().view(torch.int16))
        x = want.float()
        deq = q.float() * s.repeat_interleave(16, dim=1)[:, :, None]
        bound = 2.0 ** -4 * x.abs() + 2.0 ** -10 * s.repeat_interleave(16, dim=1)[:, :, None]
        assert bool(((deq - x).abs() <= bound * (1 + 1e-6)).all())
    assert m.check_device_errors(0) == 0
