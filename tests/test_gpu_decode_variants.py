"""The decode kernel's build-time-equal, run-time-selected variants against
the oracle: split merge inside the decode grid (GKV_DECODE_FUSED_MERGE=1),
per-(page, head) TMA boxes (GKV_DECODE_BOX=head), L2 prefetch of the
stages past the ring (GKV_DECODE_L2_PREFETCH) and a combine that waits for
the decode CTAs' arrival count (GKV_DECODE_COMBINE_WAIT=count). The library reads these once
per process, so each variant runs in a child process: config 1 (Qwen3-0.6B
layer), a 3-page context with a group of 8, 4 kv heads (2 pages per stage),
and two consecutive steps across a page boundary, each checked against the
oracle within the path's tolerance with bit-exact pool bytes."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

CHILD = r"""
import sys
sys.path[:0] = [ROOT, HERE]
import numpy as np, torch
from genllm_b200.synth import fragmented_case
from gpu_util import assert_close, bits_of, build_state, to_dev_bf16
from genllm_b200.paged_attention import paged_attention
from oracle.oracle import Oracle, run_oracle_case
orc = Oracle()
cases = [fragmented_case(0, 16, 8, 128, 1024, 256), fragmented_case(3, 64, 8, 128, 40, 8),
         fragmented_case(4, 16, 4, 128, 700, 60), fragmented_case(5, 32, 8, 128, 2000, 200)]
for case in cases:
    want, o_kp, o_vp, _, _, _ = run_oracle_case(case, orc)
    m = build_state(case)
    hq, hkv = case.n_q_heads, case.n_kv_heads
    out = torch.empty(1, hq, 1, 128, device="cuda")
    paged_attention(m, 0, to_dev_bf16(case.q, "cuda").view(1, hq, 1, 128),
                    to_dev_bf16(case.k_new, "cuda").view(1, hkv, 1, 128),
                    to_dev_bf16(case.v_new, "cuda").view(1, hkv, 1, 128), out=out, scale=case.scale)
    torch.cuda.synchronize()
    assert_close(out[0].cpu().numpy(), want, "variant")
    kp, vp = m.pool_tensors(0)
    assert np.array_equal(bits_of(kp).reshape(o_kp.shape), o_kp)
    assert np.array_equal(bits_of(vp).reshape(o_vp.shape), o_vp)
    assert m.check_device_errors(0) == 0
# two steps in a row on one cache (the second opens a page)
case = fragmented_case(6, 32, 8, 128, 1007, 80)
m = build_state(case)
rng = np.random.default_rng(1)
outs = []
for step in range(2):
    q = torch.randn(1, 32, 1, 128, device="cuda").to(torch.bfloat16)
    k = torch.randn(1, 8, 1, 128, device="cuda").to(torch.bfloat16)
    o = paged_attention(m, 0, q, k, k, scale=case.scale)
    outs.append(o)
torch.cuda.synchronize()
assert all(torch.isfinite(o.float()).all() for o in outs) and m.check_device_errors(0) == 0
print("VARIANT OK")
"""


@pytest.mark.parametrize("env", [{"GKV_DECODE_FUSED_MERGE": "1"}, {"GKV_DECODE_BOX": "head"},
                                 {"GKV_DECODE_L2_PREFETCH": "4"},
                                 {"GKV_DECODE_FUSED_MERGE": "1", "GKV_DECODE_L2_PREFETCH": "2"},
                                 {"GKV_DECODE_COMBINE_WAIT": "count"}],
                         ids=["fused-merge", "head-boxes", "l2-prefetch", "fused+prefetch", "counted-combine"])
def test_decode_variant_matches_oracle(env):
    code = CHILD.replace("ROOT", repr(ROOT)).replace("HERE", repr(HERE))
    r = subprocess.run([sys.executable, "-c", code], env={**os.environ, **env}, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and "VARIANT OK" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]


def test_multi_layer_steps_with_fused_merge():
    """Captured and one-call multi-layer steps (tests/test_gpu_decode_graph.py:
    oracle checks, bit-identity with per-layer calls, exhaustion rollback)
    with the split merge inside the decode grid, whose first layer of an
    uncaptured step releases the next layer only after its own wait."""
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider",
                        os.path.join(HERE, "test_gpu_decode_graph.py")],
                       env={**os.environ, "GKV_DECODE_FUSED_MERGE": "1"}, capture_output=True, text=True,
                       timeout=900, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
