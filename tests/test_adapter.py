"""The drop-in adapter (genllm_b200/adapter/paged_attention_cuda.cpp) compiles
against the reference's own headers, unchanged. Needs the reference tree, so
it runs only where that tree exists (the build container)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("GENLLM_REF") or os.path.join(os.path.dirname(ROOT), "reference")


@pytest.mark.skipif(not os.path.isdir(REF) or not shutil.which("g++"), reason="reference tree absent")
@pytest.mark.parametrize("name", ["paged_attention_cuda.cpp", "flash_attention_cuda.cpp"])
def test_adapter_compiles_against_reference_headers(name):
    src = os.path.join(ROOT, "genllm_b200", "adapter", name)
    cmd = ["g++", "-std=c++23", "-fsyntax-only", "-DBACKEND_CUDA", "-I", os.path.join(ROOT, "oracle", "polyfill"),
           "-I", os.path.join(ROOT, "include"), "-I", f"{REF}/include", "-I", f"{REF}/include/utils",
           "-I", f"{REF}/include/core", "-I", f"{REF}/include/3rd", "-I", "/usr/local/cuda/include", src]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
