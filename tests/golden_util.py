"""Load the golden fixtures (tests/golden/*.npz, made by the reference itself)
back into FragmentedCase objects."""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
sys.path.insert(0, GOLDEN)

from cases import CONFIG1, SMALL  # noqa: E402,F401
from genllm_b200.synth import FragmentedCase, fragmented_case  # noqa: E402


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def load_small(name):
    kw = dict(next(k for n, k, _ in SMALL if n == name))
    causal = next(c for n, _, c in SMALL if n == name)
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    case = FragmentedCase(kw["n_q_heads"], kw["n_kv_heads"], kw["head_dim"], kw["n_prior"], kw.get("n_new", 1),
                          kw["pool_pages"], z["k_ids_in"], z["v_ids_in"], z["k_free_order"], z["v_free_order"],
                          z["k_pool"], z["v_pool"], z["q"], z["k_new"], z["v_new"],
                          float(1.0 / np.sqrt(kw["head_dim"])))
    return case, causal, z


def load_config1():
    name, kw, causal = CONFIG1
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    case = fragmented_case(**kw)
    got = [sha(case.k_pool), sha(case.v_pool), sha(case.q), sha(case.k_new), sha(case.v_new)]
    if got != [str(x) for x in z["inputs_sha"]]:
        raise AssertionError("seeded input generator drifted from the one the fixture was made with")
    return case, causal, z
