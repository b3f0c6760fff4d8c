"""Generate the golden fixtures in this directory from the REFERENCE itself.

Runs the unmodified reference CPU op (oracle/_ref/libgenllm_ref.so, compiled
from the Genllm sources by oracle/Makefile) on the seeded cases of cases.py
and stores its outputs. Needs the reference tree (only present where the
fixtures are made); the tests only read the .npz files.

    make -C oracle && python tests/golden/make_golden.py
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from cases import CONFIG1, SMALL  # noqa: E402
from genllm_b200.synth import fragmented_case  # noqa: E402
from oracle.oracle import run_ref_case  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    for name, kw, causal in SMALL:
        c = fragmented_case(**kw)
        out, kp, vp, k_ids, v_ids, nc = run_ref_case(c, causal)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), q=c.q, k_new=c.k_new, v_new=c.v_new,
                            k_pool=c.k_pool, v_pool=c.v_pool, k_ids_in=c.k_ids, v_ids_in=c.v_ids,
                            k_free_order=c.k_free_order, v_free_order=c.v_free_order,
                            out_bf16=out, k_pool_after=kp, v_pool_after=vp, k_ids=k_ids, v_ids=v_ids,
                            num_cached=nc)
        print(name, out.shape, nc)
    name, kw, causal = CONFIG1
    c = fragmented_case(**kw)
    out, kp, vp, k_ids, v_ids, nc = run_ref_case(c, causal)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), out_bf16=out, k_ids=k_ids, v_ids=v_ids,
                        num_cached=nc, inputs_sha=np.array([sha(c.k_pool), sha(c.v_pool), sha(c.q),
                                                            sha(c.k_new), sha(c.v_new)]),
                        pools_after_sha=np.array([sha(kp), sha(vp)]))
    print(name, out.shape, nc)


if __name__ == "__main__":
    main()
