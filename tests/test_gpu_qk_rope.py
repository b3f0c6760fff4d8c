"""QK-norm + RoPE on the GPU against the reference (golden fixtures) and the
oracle, through the public API: the standalone fused kernel bit-exact, and
the attention op on the projections (decode: fused into the decode kernel;
chunks: fused kernel + prefill) with the appended pages bit-exact and the
output within max-abs 2e-3 and max-rel 1e-2 (gpu_util.assert_close)."""
import dataclasses
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

from cases import QK_ROPE  # noqa: E402
from genllm_b200.paged_attention import QkNorm, paged_attention_qknorm, qk_norm_rope  # noqa: E402
from genllm_b200.synth import fragmented_case, heads_major, qk_rope_case  # noqa: E402
from golden_util import GOLDEN  # noqa: E402
from gpu_util import assert_close, bits_of, build_state, to_dev_bf16  # noqa: E402
from oracle.oracle import Oracle, run_oracle_case  # noqa: E402

pytestmark = pytest.mark.gpu
ORC = Oracle()


def qknorm_of(c, max_seq):
    return QkNorm(torch.from_numpy(c.q_norm_w), torch.from_numpy(c.k_norm_w), c.eps, c.theta, max_seq, 0)


@pytest.mark.parametrize("name,kw,max_seq", QK_ROPE)
def test_qk_norm_rope_golden(name, kw, max_seq):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    c = qk_rope_case(**kw)
    qk = qknorm_of(c, max_seq)
    q, k, v = qk_norm_rope(to_dev_bf16(c.q_flat, "cuda:0"), to_dev_bf16(c.k_flat, "cuda:0"),
                           to_dev_bf16(c.v_flat, "cuda:0"), c.n_q_heads, c.n_kv_heads, qk, c.start_pos)
    torch.cuda.synchronize()
    assert np.array_equal(bits_of(q), z["q_rope"]), "Q differs from the reference"
    assert np.array_equal(bits_of(k), z["k_rope"]), "K differs from the reference"
    assert np.array_equal(bits_of(v), heads_major(c.v_flat, c.n_kv_heads)), "V permute differs"


def step_case(seed, hq, hkv, n_prior, n_new, pool_pages, order="random"):
    """A fragmented cache plus this step's projections; the oracle's view of
    the step (Q / K / V after QK-norm + RoPE + permute) as a FragmentedCase."""
    base = fragmented_case(seed, hq, hkv, 128, n_prior, pool_pages, n_new=n_new, page_order=order)
    p = qk_rope_case(seed + 1, hq, hkv, n_new, n_prior)
    max_seq = n_prior + n_new + 16
    cos, sin = ORC.rope_cache(p.theta, 128, max_seq)
    qr = ORC.apply_rope_bf16(ORC.rms_norm_bf16(heads_major(p.q_flat, hq), p.q_norm_w, p.eps), cos, sin, n_prior)
    kr = ORC.apply_rope_bf16(ORC.rms_norm_bf16(heads_major(p.k_flat, hkv), p.k_norm_w, p.eps), cos, sin, n_prior)
    case = dataclasses.replace(base, q=qr, k_new=kr, v_new=heads_major(p.v_flat, hkv))
    return case, p, max_seq


@pytest.mark.parametrize("hq,hkv,n_prior,n_new", [(32, 8, 4000, 1), (16, 8, 37, 1), (8, 2, 0, 1), (16, 8, 100, 45),
                                                  (16, 8, 0, 300), (4, 1, 2000, 130)])
def test_attention_on_projections(hq, hkv, n_prior, n_new):
    case, p, max_seq = step_case(700 + n_new + hq, hq, hkv, n_prior, n_new, (n_prior + n_new) // 16 + 6)
    o_out, o_kp, o_vp, o_k, o_v, o_n = run_oracle_case(case, ORC, True, threads=min(os.cpu_count() or 1, 32))
    m = build_state(case)
    qk = qknorm_of(p, max_seq)
    out = torch.empty((hq, n_new, 128), dtype=torch.float32, device=m.device)
    paged_attention_qknorm(m, 0, to_dev_bf16(p.q_flat, m.device), to_dev_bf16(p.k_flat, m.device),
                           to_dev_bf16(p.v_flat, m.device), hq, qk, out=out)
    torch.cuda.synchronize()
    kp, vp = m.pool_tensors(0)
    assert np.array_equal(bits_of(kp).reshape(o_kp.shape), o_kp), "K pool bytes differ (post-norm, post-RoPE rows)"
    assert np.array_equal(bits_of(vp).reshape(o_vp.shape), o_vp), "V pool bytes differ"
    L = m.get_layer(0)
    assert L.num_cached == o_n
    assert m.check_device_errors(0) == 0
    assert_close(out.cpu().numpy(), o_out, "attention on projections")


def test_positions_past_the_table_rejected():
    case, p, max_seq = step_case(801, 16, 8, 50, 1, 10)
    m = build_state(case)
    qk = qknorm_of(p, 50)  # table rows 0..49: position 50 is outside
    from genllm_b200._lib import GkvError
    with pytest.raises(GkvError):
        paged_attention_qknorm(m, 0, to_dev_bf16(p.q_flat, m.device), to_dev_bf16(p.k_flat, m.device),
                               to_dev_bf16(p.v_flat, m.device), 16, qk)
    assert m.get_layer(0).num_cached == 50, "a rejected step must leave the layer unchanged"
