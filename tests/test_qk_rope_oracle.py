"""The QK-norm + RoPE restatement (oracle/qk_rope_oracle.c) against the
reference's own ops: the golden fixtures (made by the reference, see
tests/golden/make_golden.py) and, where oracle/_ref was built here, the live
reference on more seeds and shapes. All comparisons are bit-exact."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

from cases import QK_ROPE  # noqa: E402
from genllm_b200.synth import heads_major, qk_rope_case, randn_bf16  # noqa: E402
from golden_util import GOLDEN, sha  # noqa: E402
from oracle.oracle import Oracle, RefOps, bf16_from_f32, bf16_to_f32, ref_ops_available  # noqa: E402

ORC = Oracle()
needs_ref = pytest.mark.skipif(not ref_ops_available(), reason="oracle/_ref/libgenllm_ref_ops.so not built")


def oracle_pipeline(c, max_seq):
    cos, sin = ORC.rope_cache(c.theta, c.head_dim, max_seq)
    qn = ORC.rms_norm_bf16(heads_major(c.q_flat, c.n_q_heads), c.q_norm_w, c.eps)
    kn = ORC.rms_norm_bf16(heads_major(c.k_flat, c.n_kv_heads), c.k_norm_w, c.eps)
    return cos, sin, qn, kn, ORC.apply_rope_bf16(qn, cos, sin, c.start_pos), ORC.apply_rope_bf16(kn, cos, sin, c.start_pos)


@pytest.mark.parametrize("name,kw,max_seq", QK_ROPE)
def test_golden_qk_rope(name, kw, max_seq):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    c = qk_rope_case(**kw)
    assert [sha(c.q_flat), sha(c.k_flat), sha(c.q_norm_w), sha(c.k_norm_w)] == [str(s) for s in z["inputs_sha"]]
    cos, sin, qn, kn, qr, kr = oracle_pipeline(c, max_seq)
    assert [sha(cos), sha(sin)] == [str(s) for s in z["cache_sha"]], "RoPE table differs from the reference's"
    assert np.array_equal(qn, z["q_normed"]) and np.array_equal(kn, z["k_normed"]), "QK-norm differs"
    assert np.array_equal(qr, z["q_rope"]) and np.array_equal(kr, z["k_rope"]), "RoPE differs"


@needs_ref
@pytest.mark.parametrize("dim", [128, 64, 136, 100, 8, 5])
def test_rms_norm_live(dim):
    rng = np.random.default_rng(dim)
    R = RefOps()
    x = randn_bf16(rng, (97, dim))
    x[3] = 0  # an all-zero row: rms = 1/sqrt(eps)
    x[5] = bf16_from_f32(bf16_to_f32(x[5]) * np.float32(1e25))  # finite, but the sum of squares overflows
    w = (1 + 0.3 * rng.standard_normal(dim)).astype(np.float32)
    for eps in (1e-6, 1e-5):
        assert np.array_equal(ORC.rms_norm_bf16(x, w, eps), R.rms_norm_bf16(x, w, eps))


@needs_ref
@pytest.mark.parametrize("theta,head_dim,max_seq", [(1e6, 128, 2048), (1e4, 64, 300), (5e5, 128, 40960)])
def test_rope_cache_live(theta, head_dim, max_seq):
    R = RefOps()
    c1, s1 = ORC.rope_cache(theta, head_dim, max_seq)
    c2, s2 = R.rope_cache(theta, head_dim, max_seq)
    assert np.array_equal(c1, c2) and np.array_equal(s1, s2)


@needs_ref
@pytest.mark.parametrize("seed,start", [(1, 0), (2, 7), (3, 4000), (4, 39000)])
def test_apply_rope_live(seed, start):
    rng = np.random.default_rng(seed)
    R = RefOps()
    cos, sin = R.rope_cache(1e6, 128, 40960)
    x = randn_bf16(rng, (8, 33, 128))
    if start + 33 > 40960:
        start = 40960 - 33
    assert np.array_equal(ORC.apply_rope_bf16(x, cos, sin, start), R.apply_rope_bf16(x, cos, sin, start))


@pytest.mark.parametrize("name,kw,max_seq", QK_ROPE)
def test_library_rope_cache_matches_reference(name, kw, max_seq):
    """gkv_rope_cache (the product's host-side table builder) against the
    reference's table checksums in the fixtures."""
    from genllm_b200.paged_attention import rope_cache
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    c = qk_rope_case(**kw)
    cos, sin = rope_cache(c.theta, c.head_dim, max_seq)
    assert [sha(cos), sha(sin)] == [str(s) for s in z["cache_sha"]]

