"""The non-paged attention restatement (oracle/flash_oracle.c) against the
reference's FlashAttentionImpl<CPU> built from its own sources (oracle/_ref):
bit-exact after the reference's bf16 output rounding."""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))

from genllm_b200.synth import randn_bf16
from oracle.oracle import Oracle, ref_available, ref_flash_attention

ORC = Oracle()


@pytest.mark.skipif(not ref_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("B,Hq,Hkv,S,causal", [(1, 4, 2, 1, True), (1, 8, 2, 37, True), (2, 4, 4, 20, False),
                                               (2, 8, 1, 64, True), (1, 16, 8, 130, True)])
def test_flash_oracle_matches_reference(B, Hq, Hkv, S, causal):
    rng = np.random.default_rng(B * 1000 + S)
    q = randn_bf16(rng, (B, Hq, S, 128))
    k = randn_bf16(rng, (B, Hkv, S, 128))
    v = randn_bf16(rng, (B, Hkv, S, 128))
    scale = float(1 / np.sqrt(128))
    got = ORC.round_bf16(ORC.flash_attention_f32(q, k, v, scale, causal))
    want = ref_flash_attention(q, k, v, scale, causal)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("name,seed,B,Hq,Hkv,S,causal", __import__("cases").FLASH)
def test_flash_oracle_golden(name, seed, B, Hq, Hkv, S, causal):
    """Against the reference's outputs stored in tests/golden (made by
    tests/golden/make_golden.py from the reference op)."""
    from golden_util import GOLDEN, sha
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    rng = np.random.default_rng(seed)
    q = randn_bf16(rng, (B, Hq, S, 128))
    k = randn_bf16(rng, (B, Hkv, S, 128))
    v = randn_bf16(rng, (B, Hkv, S, 128))
    assert [sha(q), sha(k), sha(v)] == [str(x) for x in z["inputs_sha"]]
    got = ORC.round_bf16(ORC.flash_attention_f32(q, k, v, float(1 / np.sqrt(128)), causal))
    assert np.array_equal(got, z["out_bf16"])
