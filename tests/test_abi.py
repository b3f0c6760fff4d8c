"""The C-ABI library loads and exports every entry point include/genllm_kv.h declares."""
import os
import re

from genllm_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "genllm_kv.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gkv_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "gkv_paged_attention" in names and "gkv_paged_attention_raw" in names
    assert len(names) >= 25


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing


def test_python_signatures_cover_header():
    missing = [n for n in declared_functions() if n not in _lib.SIGNATURES]
    assert not missing, missing


def test_status_strings():
    L = _lib.lib()
    assert L.gkv_status_string(0) == b"ok"
    assert L.gkv_status_string(2) == b"page pool exhausted"
