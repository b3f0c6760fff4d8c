"""The KV format export / import oracle (oracle/kv_format_oracle.c), pinned:

* its e4m3 decoder against torch's float8_e4m3fn for all 256 codes, and its
  encoder against torch's conversion for every finite bf16 value inside
  +-448 plus random fp32 values (torch rounds to nearest even there; the
  saturation and NaN rules of the format are checked case by case);
* its bf16 export as the inverse of the reference's own append
  (append_kv_from_tensor, run from oracle/_ref) on ragged multi-call appends;
* its fp8 export against the committed fixtures (numpy fp32 block scales +
  torch's conversion), and its import against the format's error bound."""
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

from cases import KV_FORMAT  # noqa: E402
from genllm_b200.synth import bf16_bits, kv_format_values  # noqa: E402
from golden_util import GOLDEN  # noqa: E402
from oracle.oracle import Oracle, OraclePool, RefSession, ref_available  # noqa: E402

ORC = Oracle()


def f32_of_bf16(b):
    return (np.asarray(b, dtype=np.uint32) << 16).view(np.float32)


def test_e4m3_decoder_all_codes():
    codes = np.arange(256, dtype=np.uint8)
    ours = ORC.e4m3_to_f32(codes)
    want = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(ours), np.isnan(want))
    ok = ~np.isnan(want)
    assert np.array_equal(ours[ok].view(np.uint32), want[ok].view(np.uint32))


def test_e4m3_encoder_matches_torch_in_range():
    x = f32_of_bf16(np.arange(65536, dtype=np.uint32))
    x = x[np.isfinite(x) & (np.abs(x) < 448)]
    rng = np.random.default_rng(3)
    x = np.concatenate([x, rng.standard_normal(20000).astype(np.float32) * 60,
                        rng.standard_normal(20000).astype(np.float32) * 2e-3,
                        # exact ties between neighbouring codes
                        np.array([2.0 ** -10, 3 * 2.0 ** -10, 1.0625, 1.1875, 17.0, 19.0, 416.0], np.float32)])
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ORC.e4m3_from_f32(x), want)


@pytest.mark.parametrize("x,code", [(448.0, 0x7E), (-448.0, 0xFE), (464.0, 0x7E), (1e30, 0x7E), (np.inf, 0x7E),
                                    (-np.inf, 0xFE), (np.nan, 0x7F), (-0.0, 0x80), (0.0, 0x00),
                                    (2.0 ** -10, 0x00), (-(2.0 ** -11), 0x80), (2.0 ** -9, 0x01),
                                    (0.0146484375, 0x08)])
def test_e4m3_encoder_edges(x, code):
    assert int(ORC.e4m3_from_f32(np.array([x], np.float32))[0]) == code


def _ref_pages(seed, hkv, chunks, pages):
    n = sum(chunks)
    K, V = kv_format_values(seed, hkv, n)
    R = RefSession(1, hkv, 128, pages)
    p0 = 0
    for c in chunks:
        R.append_kv(0, np.ascontiguousarray(K[:, p0:p0 + c]), np.ascontiguousarray(V[:, p0:p0 + c]), c)
        p0 += c
    k_ids, v_ids, nc = R.table(0)
    kp, vp = R.pool_view(0, 0).copy(), R.pool_view(0, 1).copy()
    R.close()
    return K, V, kp, vp, k_ids, v_ids, nc


@pytest.mark.skipif(not ref_available(), reason="reference build (oracle/_ref) absent")
@pytest.mark.parametrize("seed,hkv,chunks,pages", [(61, 1, [1], 1), (62, 2, [15, 1, 1], 2), (63, 8, [16], 1),
                                                   (64, 4, [7, 40, 33, 2], 6), (65, 8, [300], 19)])
def test_bf16_export_inverts_reference_append(seed, hkv, chunks, pages):
    K, V, kp, vp, k_ids, v_ids, nc = _ref_pages(seed, hkv, chunks, pages)
    assert nc == sum(chunks)
    ko, vo, _, _ = ORC.export_kv(kp, vp, k_ids, v_ids, nc, hkv)
    assert np.array_equal(ko, K) and np.array_equal(vo, V)


@pytest.mark.parametrize("name,seed,hkv,chunks,pages", KV_FORMAT)
def test_export_golden(name, seed, hkv, chunks, pages):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    K, V = kv_format_values(seed, hkv, sum(chunks))
    n = int(z["num_cached"])
    ko, vo, _, _ = ORC.export_kv(z["k_pool"], z["v_pool"], z["k_ids"], z["v_ids"], n, hkv)
    assert np.array_equal(ko, K) and np.array_equal(vo, V)
    kq, vq, ks, vs = ORC.export_kv(z["k_pool"], z["v_pool"], z["k_ids"], z["v_ids"], n, hkv, fp8=True)
    assert np.array_equal(kq, z["k_fp8"]) and np.array_equal(vq, z["v_fp8"])
    assert np.array_equal(ks.view(np.uint32), z["k_scales"].view(np.uint32))
    assert np.array_equal(vs.view(np.uint32), z["v_scales"].view(np.uint32))


def test_golden_has_the_edge_blocks():
    z = np.load(os.path.join(GOLDEN, "kvfmt_heads8.npz"))
    assert (z["k_fp8"] == 0x7F).any(), "a NaN element"
    assert (z["k_scales"] == 1.0).any(), "a block with scale 1 (all zero / subnormal)"
    assert (z["k_fp8"] == 0x7E).sum() > 16, "saturated +inf and block maxima"


def test_fp8_round_trip_error_bound():
    """import(export(x)) stays within the format's rounding: half a unit in the
    last place of a 3-bit mantissa (2^-4 relative) for normal codes, half the
    subnormal step (2^-10 * scale) below, plus the bf16 rounding of the result."""
    hkv, n = 4, 203
    K, V = kv_format_values(71, hkv, n, special=False)
    pool = OraclePool(16, ORC)
    kp = np.zeros((16, 16, hkv, 128), np.uint16)
    vp = np.zeros_like(kp)
    pool.append_kv(kp, vp, K, V, hkv, n, 128)
    k_ids, v_ids = pool.table()
    kq, vq, ks, vs = ORC.export_kv(kp, vp, k_ids, v_ids, n, hkv, fp8=True)
    kp2, vp2 = np.zeros_like(kp), np.zeros_like(vp)
    ORC.import_fp8(kp2, vp2, k_ids, v_ids, 0, kq, vq, ks, vs)
    k2, v2, _, _ = ORC.export_kv(kp2, vp2, k_ids, v_ids, n, hkv)
    for x, y, s in ((K, k2, ks), (V, v2, vs)):
        xf, yf = f32_of_bf16(x).astype(np.float64), f32_of_bf16(y).astype(np.float64)
        sc = np.repeat(s, 16, axis=1)[:, :n, None].astype(np.float64)
        bound = 2.0 ** -4 * np.abs(xf) + 2.0 ** -10 * sc
        bound = bound * (1 + 2.0 ** -8) + 2.0 ** -8 * np.abs(xf)
        assert (np.abs(yf - xf) <= bound).all()


def test_import_at_an_offset_matches_append_of_dequantised_values():
    """Importing e4m3 tokens after n_prior cached ones lands each row where
    the reference's append would put the dequantised row."""
    hkv, n_prior, s = 2, 23, 29
    rng = np.random.default_rng(5)
    q = rng.integers(0, 0x7F, size=(2, hkv, s, 128)).astype(np.uint8)
    q |= (rng.integers(0, 2, size=q.shape) << 7).astype(np.uint8)
    scales = (2.0 ** rng.integers(-8, 8, size=(2, hkv, (s + 15) // 16))).astype(np.float32)
    pool = OraclePool(8, ORC)
    kp = np.zeros((8, 16, hkv, 128), np.uint16)
    vp = np.zeros_like(kp)
    pool.append_kv(kp, vp, np.zeros((hkv, n_prior, 128), np.uint16), np.zeros((hkv, n_prior, 128), np.uint16),
                   hkv, n_prior, 128)
    deq = [bf16_bits(ORC.e4m3_to_f32(q[w]).reshape(q[w].shape) *
                     np.repeat(scales[w], 16, axis=1)[:, :s, None]) for w in range(2)]
    kp_a, vp_a = kp.copy(), vp.copy()
    pool_a = OraclePool(8, ORC)
    pool_a.append_kv(kp_a, vp_a, np.zeros((hkv, n_prior, 128), np.uint16),
                     np.zeros((hkv, n_prior, 128), np.uint16), hkv, n_prior, 128)
    pool_a.append_kv(kp_a, vp_a, deq[0], deq[1], hkv, s, 128)
    pool.append_pages(s)  # allocate the same pages the append took
    k_ids, v_ids = pool.table()
    ORC.import_fp8(kp, vp, k_ids, v_ids, n_prior, q[0], q[1], scales[0], scales[1])
    assert np.array_equal(kp, kp_a) and np.array_equal(vp, vp_a)


def test_e4m3_encoder_is_nearest_even_by_brute_force():
    """Independent of torch: for random fp32 inputs inside +-448 the code is
    the nearest of all 255 finite e4m3 values, ties to the even code."""
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], dtype=np.uint8)
    vals = ORC.e4m3_to_f32(codes).astype(np.float64)
    rng = np.random.default_rng(9)
    x = np.concatenate([rng.uniform(-448, 448, 3000), rng.standard_normal(3000) * 2.0 ** rng.integers(-12, 8, 3000),
                        (vals[:, None] + vals[None, :]).ravel()[::7] / 2]).astype(np.float32)  # midpoints: ties
    x = x[np.abs(x) <= 448]
    got = ORC.e4m3_from_f32(x)
    d = np.abs(vals[None, :] - x.astype(np.float64)[:, None])
    best = d.min(axis=1)
    for i in range(len(x)):
        cand = codes[d[i] == best[i]]
        if len(cand) == 1:
            want = cand[0]
        else:  # a tie: the even mantissa (for +-0, the code with x's sign)
            even = [c for c in cand if (c & 1) == 0]
            want = even[0] if len(even) == 1 else (0x80 if np.signbit(x[i]) else 0x00)
        assert got[i] == want, (float(x[i]), int(got[i]), int(want))


def test_e4m3_encoder_monotone_and_symmetric():
    x = np.sort(np.random.default_rng(4).uniform(0, 500, 5000).astype(np.float32))
    v = ORC.e4m3_to_f32(ORC.e4m3_from_f32(x))
    assert (np.diff(v) >= 0).all()
    assert np.array_equal(ORC.e4m3_from_f32(-x), ORC.e4m3_from_f32(x) | 0x80)
