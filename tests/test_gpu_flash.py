"""Non-paged attention (gkv_flash_attention, the reference's
FlashAttentionImpl) on the tcgen05 kernel against the oracle
(oracle/flash_oracle.c, pinned to the reference op): within
max-abs 2e-3 and max-rel 1e-2 (gpu_util.assert_close); bf16 output against the reference's own
bf16 output where oracle/_ref is present."""
import numpy as np
import pytest
import torch

from genllm_b200.paged_attention import flash_attention, flash_check_errors
from genllm_b200.synth import bf16_to_f32, randn_bf16
from gpu_util import assert_bf16_close, assert_close, bits_of, to_dev_bf16
from oracle.oracle import Oracle, ref_available, ref_flash_attention

pytestmark = pytest.mark.gpu
ORC = Oracle()


def inputs(seed, B, Hq, Hkv, S):
    rng = np.random.default_rng(seed)
    return (randn_bf16(rng, (B, Hq, S, 128)), randn_bf16(rng, (B, Hkv, S, 128)), randn_bf16(rng, (B, Hkv, S, 128)))


@pytest.mark.parametrize("B,Hq,Hkv,S,causal", [(1, 16, 8, 512, True), (2, 8, 2, 300, True), (1, 4, 4, 1, True),
                                               (3, 8, 1, 129, False), (1, 32, 8, 1000, True), (2, 16, 8, 127, False),
                                               (1, 2, 2, 2048, True)])
def test_flash_attention(B, Hq, Hkv, S, causal):
    q, k, v = inputs(B * 7919 + S, B, Hq, Hkv, S)
    scale = float(1 / np.sqrt(128))
    out = torch.empty((B, Hq, S, 128), dtype=torch.float32, device="cuda")
    flash_attention(to_dev_bf16(q, "cuda"), to_dev_bf16(k, "cuda"), to_dev_bf16(v, "cuda"), out=out, scale=scale,
                    causal=causal)
    torch.cuda.synchronize()
    assert flash_check_errors() == 0
    want = ORC.flash_attention_f32(q, k, v, scale, causal)
    assert_close(out.cpu().numpy(), want, "flash attention")


@pytest.mark.skipif(not ref_available(), reason="oracle/_ref not built")
def test_flash_attention_bf16_against_reference():
    q, k, v = inputs(5, 2, 8, 2, 200)
    scale = float(1 / np.sqrt(128))
    got = flash_attention(to_dev_bf16(q, "cuda"), to_dev_bf16(k, "cuda"), to_dev_bf16(v, "cuda"), scale=scale)
    torch.cuda.synchronize()
    want = ref_flash_attention(q, k, v, scale, True)
    assert_bf16_close(bits_of(got), want, "bf16 out vs reference")
