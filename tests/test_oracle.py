"""The CPU oracle (C restatement) against the reference's own outputs.

Pins the oracle before it is trusted as the GPU checker:
* against the golden fixtures made by running the reference op
  (tests/golden/make_golden.py): bf16 outputs, post-append pool bytes and
  page tables must be bit-identical;
* against the reference build itself (oracle/_ref) on further seeds, when it
  is present (it is built wherever the reference tree exists).
"""
import numpy as np
import pytest

from genllm_b200.synth import fragmented_case
from golden_util import SMALL, load_config1, load_small, sha
from oracle.oracle import Oracle, bf16_from_f32, ref_available, run_oracle_case, run_ref_case

ORC = Oracle()


@pytest.mark.parametrize("name", [n for n, _, _ in SMALL])
def test_oracle_matches_reference_golden(name):
    case, causal, z = load_small(name)
    out, kp, vp, k_ids, v_ids, nc = run_oracle_case(case, ORC, causal)
    assert nc == int(z["num_cached"])
    assert k_ids.tolist() == z["k_ids"].tolist() and v_ids.tolist() == z["v_ids"].tolist()
    assert np.array_equal(kp, z["k_pool_after"]) and np.array_equal(vp, z["v_pool_after"])
    assert np.array_equal(ORC.round_bf16(out), z["out_bf16"])


def test_oracle_matches_reference_golden_config1():
    case, causal, z = load_config1()
    out, kp, vp, k_ids, v_ids, nc = run_oracle_case(case, ORC, causal)
    assert nc == int(z["num_cached"]) == 1025
    assert k_ids.tolist() == z["k_ids"].tolist() and v_ids.tolist() == z["v_ids"].tolist()
    assert [sha(kp), sha(vp)] == [str(x) for x in z["pools_after_sha"]]
    assert np.array_equal(ORC.round_bf16(out), z["out_bf16"])


def test_bf16_rounding_matches_reference_rules():
    cases = np.array([0.0, -0.0, 1.0, 1.00390625, 1.01171875, 3.4e38, -3.4e38, 1e-39, -1e-39,
                      np.inf, -np.inf, np.nan, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -9], dtype=np.float32)
    a = bf16_from_f32(cases)
    b = ORC.round_bf16(cases)
    assert np.array_equal(a, b)
    assert a[7] == 0 and a[8] == 0x8000  # subnormals flush to signed zero
    assert a[5] == 0x7F80  # rounds past the largest finite value -> inf
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(100000) * np.exp(rng.uniform(-90, 90, 100000))).astype(np.float32)
    assert np.array_equal(bf16_from_f32(x), ORC.round_bf16(x))


def test_threaded_oracle_is_identical():
    case = fragmented_case(5, 8, 2, 128, 300, 32)
    a = run_oracle_case(case, ORC)[0]
    b = run_oracle_case(case, ORC, threads=4)[0]
    assert np.array_equal(a, b)


@pytest.mark.skipif(not ref_available(), reason="reference build (oracle/_ref) absent")
@pytest.mark.parametrize("seed,hq,hkv,n_prior,pool,n_new,causal", [
    (101, 32, 8, 300, 40, 1, True),
    (102, 16, 8, 15, 4, 1, True),
    (103, 8, 8, 64, 8, 1, True),
    (104, 16, 2, 100, 16, 1, True),
    (105, 16, 8, 40, 12, 33, True),
    (106, 4, 2, 17, 6, 16, False),
])
def test_oracle_matches_reference_live(seed, hq, hkv, n_prior, pool, n_new, causal):
    case = fragmented_case(seed, hq, hkv, 128, n_prior, pool, n_new=n_new)
    o = run_oracle_case(case, ORC, causal)
    r = run_ref_case(case, causal)
    assert np.array_equal(ORC.round_bf16(o[0]), r[0])
    for a, b in zip(o[1:], r[1:]):
        assert np.array_equal(np.asarray(a), np.asarray(b))
