"""Config 2, the drop-in check: the Genllm engine itself (GGUF loader, graph
builder, GraphScheduler, MemoryManager, Executor; built from its sources by
oracle/engine/Makefile) runs a synthetic Qwen3-0.6B (seed 1, 28 layers,
vocab 151936) with this repository's ops::PagedAttentionImpl<Device::CUDA>
(genllm_b200/adapter/paged_attention_cuda.cpp) linked in place of Genllm's
own (src/backend/cuda/attention.cu:491-580); nothing else of the engine
changes. A 128-token seeded prompt is prefilled in 4 chunks of 32 with
Executor::append_tokens (the tensor-core chunk path), then 256 decode_step
calls (the fused decode path) take seeded random ids, so that every engine
sees the same inputs. Each position's prediction is compared with the CPU
engine's (Genllm's CPU backend, its reference path) and with the CUDA engine
running Genllm's own paged attention: the argmax must agree wherever the
reference's top-2 margin is wider than the logits' rounding, and full
logits rows are compared at four positions.

The binaries exist only where the Genllm tree was present at build time
(oracle/_ref is git-ignored); the test is skipped without them."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENG = os.path.join(ROOT, "oracle", "_ref", "engine")
VOCAB, PROMPT, STEPS, CHUNK, SEED = 151936, 128, 256, 32, 1
DUMPS = sorted({0, 1, STEPS // 2, STEPS})


def _read(path):
    raw = open(path, "rb").read()
    off, rec, rows = 0, [], {}
    for i in range(STEPS + 1):
        a = int(np.frombuffer(raw, np.int32, 1, off)[0])
        t1, t2 = np.frombuffer(raw, np.float32, 2, off + 4)
        off += 12
        rec.append((a, float(t1), float(t2)))
        if i in DUMPS:
            r = np.frombuffer(raw, np.uint16, VOCAB, off)
            off += 2 * VOCAB
            rows[i] = (r.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    assert off == len(raw)
    return rec, rows


@pytest.fixture(scope="module")
def runs(tmp_path_factory):
    names = ["engine_cpu", "engine_cuda_ref", "engine_cuda_b200"]
    if not all(os.path.exists(os.path.join(ENG, n)) for n in names):
        pytest.skip("engine binaries not built (oracle/engine/Makefile needs the Genllm tree)")
    d = tmp_path_factory.mktemp("engine")
    gguf = str(d / "qwen3_0p6b_synth.gguf")
    subprocess.run([sys.executable, os.path.join(ROOT, "oracle", "engine", "make_gguf.py"), gguf, "--seed", str(SEED)],
                   check=True, timeout=900)
    out = {}
    for n in names:
        res = str(d / f"{n}.bin")
        r = subprocess.run([os.path.join(ENG, n), gguf, str(PROMPT), str(STEPS), str(CHUNK), str(SEED), res, "random"],
                           capture_output=True, text=True, timeout=1800, cwd=str(d))
        assert r.returncode == 0, f"{n} failed:\n{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
        summary = json.loads([l for l in r.stdout.splitlines() if l.startswith("{\"prompt_len\"")][-1])
        out[n] = (summary, *_read(res))
    os.makedirs(os.path.join(ROOT, "gpurun_out"), exist_ok=True)
    summary = {n: {k: v for k, v in s.items() if k != "tokens"} for n, (s, _, _) in out.items()}
    for a, b in (("engine_cuda_b200", "engine_cuda_ref"), ("engine_cuda_b200", "engine_cpu"),
                 ("engine_cuda_ref", "engine_cpu")):
        summary[f"{a} vs {b}"] = {f"pos{i}_max_abs_logit_diff": float(np.abs(out[a][2][i] - out[b][2][i]).max())
                                  for i in DUMPS}
        summary[f"{a} vs {b}"]["argmax_agree"] = int(sum(x[0] == y[0] for x, y in zip(out[a][1], out[b][1])))
    with open(os.path.join(ROOT, "gpurun_out", "engine_config2.json"), "w") as f:
        json.dump(summary, f, indent=1)
    return out


def _compare(ref, got, margin_floor):
    """Positions where the reference's top-2 margin exceeds margin_floor must
    have the same argmax; returns (agreeing positions, positions checked)."""
    agree = checked = 0
    for (ra, r1, r2), (ga, _, _) in zip(ref, got):
        if r1 - r2 > margin_floor:
            checked += 1
            agree += ra == ga
    return agree, checked


def test_engine_with_b200_attention_matches_genllm_cuda_attention(runs):
    """Same engine, same CUDA ops; only the paged-attention op differs. Its
    outputs are rounded to bf16 and pass through 28 layers of bf16
    activations, so the logits move by a few bf16 steps; the swap must move
    them less than Genllm's own two backends differ from each other."""
    _, rec_ref, rows_ref = runs["engine_cuda_ref"]
    _, rec_b2, rows_b2 = runs["engine_cuda_b200"]
    _, _, rows_cpu = runs["engine_cpu"]
    agree, checked = _compare(rec_ref, rec_b2, 1.0)
    assert checked > 0.8 * len(rec_ref) and agree == checked, (agree, checked)
    for i in DUMPS:
        swap = np.abs(rows_ref[i] - rows_b2[i]).max()
        backends = np.abs(rows_ref[i] - rows_cpu[i]).max()
        assert swap <= backends, (i, swap, backends)
        assert np.corrcoef(rows_ref[i], rows_b2[i])[0, 1] > 0.9995, i


def test_engine_with_b200_attention_matches_cpu_engine(runs):
    """Against Genllm's CPU engine (its reference path end to end)."""
    _, rec_cpu, rows_cpu = runs["engine_cpu"]
    _, rec_b2, rows_b2 = runs["engine_cuda_b200"]
    agree, checked = _compare(rec_cpu, rec_b2, 2.0)
    assert checked > 0.7 * len(rec_cpu) and agree >= checked - 2, (agree, checked)
    for i in DUMPS:
        c = np.corrcoef(rows_cpu[i], rows_b2[i])[0, 1]
        assert c > 0.999, (i, c)
