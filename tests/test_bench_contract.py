"""bench.py's reference arm (the reference's CPU op on the host cores) keeps
the driver's JSON contract; it needs no GPU, so it is checked here on a
small sample of config 3."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

KEYS = ["metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config"]


def run_bench(args, env_extra=None):
    env = dict(os.environ, **(env_extra or {}))
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + args, capture_output=True, text=True,
                       timeout=600, env=env, cwd=ROOT)
    assert p.returncode == 0, p.stderr[-2000:]
    return [l for l in p.stdout.splitlines() if l.strip()]


def test_reference_arm_prints_one_contract_line():
    lines = run_bench(["--impl", "reference", "--steps", "1", "--warmup", "1", "--ctx", "1024", "--layers", "2"])
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in KEYS:
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["kind"] in ("reference", "port")
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]


@pytest.mark.parametrize("rank", ["1"])
def test_reference_arm_other_ranks_do_no_work(rank):
    lines = run_bench(["--impl", "reference", "--steps", "1", "--warmup", "1", "--ctx", "1024", "--layers", "2"],
                      {"RANK": rank, "WORLD_SIZE": "2", "LOCAL_RANK": rank})
    assert lines == []
