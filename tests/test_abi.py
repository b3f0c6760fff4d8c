"""The C-ABI library loads and exports every entry point include/genllm_kv.h declares."""
import os
import re

import pytest

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


def test_new_entry_points_reject_bad_arguments_without_a_gpu():
    """Argument checks come before any CUDA call: they answer on a host
    without a GPU too."""
    import ctypes as C
    from genllm_b200 import _lib
    L = _lib.lib()
    assert L.gkv_flash_attention(None, None, None, None, 1, 8, 8, 16, 128, 0.1, 1, 30, 30, None) == _lib.GKV_ERR_INVALID
    assert L.gkv_qk_norm_rope(None, None, None, 1, 8, 8, None, 0, None, None, None, None) == _lib.GKV_ERR_INVALID
    assert L.gkv_decode_layers(None, 0, None, None, None, None, None, 8, 0.1, 30, None) == _lib.GKV_ERR_INVALID
    assert L.gkv_rope_cache(1e6, 127, 4, None, None) == _lib.GKV_ERR_INVALID
    import numpy as np
    c = np.zeros((4, 128), np.float32)
    s = np.zeros((4, 128), np.float32)
    assert L.gkv_rope_cache(1e6, 128, 4, C.c_void_p(c.ctypes.data), C.c_void_p(s.ctypes.data)) == 0
    assert c[0, 0] == 1.0 and s[0, 0] == 0.0


def test_kv_format_entry_points_reject_bad_arguments_without_a_gpu():
    import ctypes as C
    L = _lib.lib()
    assert L.gkv_export_kv_raw(None, None, 16, 0, None, None, None, None, None) == _lib.GKV_ERR_INVALID
    assert L.gkv_import_kv_raw(None, None, 0, None, 1, None, None, None, None, 16, None) == _lib.GKV_ERR_INVALID
    pool = _lib.PoolDesc(C.c_void_p(16), C.c_void_p(16), 4, 2, 128, _lib.GKV_BF16)
    # unknown format; a missing table
    assert L.gkv_export_kv_raw(C.byref(pool), None, 16, 7, None, None, None, None, None) == _lib.GKV_ERR_INVALID
    assert L.gkv_import_kv_raw(C.byref(pool), None, 0, None, 7, None, None, None, None, 16, None) == \
        _lib.GKV_ERR_INVALID
    # a host-only manager has no device pools
    m = C.c_void_p()
    assert L.gkv_manager_create(-1, C.byref(m)) == 0
    assert L.gkv_init_layer(m, 0, 2, 128, _lib.GKV_BF16) == 0
    n = C.c_int32(-1)
    assert L.gkv_export_kv(m, 0, 0, None, None, None, None, C.byref(n), None) == _lib.GKV_ERR_STATE
    assert L.gkv_import_kv(m, 0, 1, None, None, None, None, 4, None) == _lib.GKV_ERR_STATE
    assert L.gkv_manager_destroy(m) == 0


def test_decode_graph_entry_points_reject_bad_arguments_without_a_gpu():
    import ctypes as C
    L = _lib.lib()
    g = C.c_void_p()
    assert L.gkv_decode_graph_create(None, 1, None, None, None, None, None, 8, 0.1, 30, None, C.byref(g)) == \
        _lib.GKV_ERR_INVALID
    assert L.gkv_decode_graph_step(None, None) == _lib.GKV_ERR_INVALID
    assert L.gkv_decode_graph_destroy(None) == 0
    m = C.c_void_p()
    assert L.gkv_manager_create(-1, C.byref(m)) == 0
    assert L.gkv_init_layer(m, 0, 8, 128, _lib.GKV_BF16) == 0
    ids = (C.c_int32 * 1)(0)
    ptrs = (C.c_void_p * 1)(16)
    # a host-only manager has no device pools to capture
    assert L.gkv_decode_graph_create(m, 1, ids, ptrs, ptrs, ptrs, ptrs, 8, 0.1, 30, None, C.byref(g)) == \
        _lib.GKV_ERR_STATE
    assert L.gkv_manager_destroy(m) == 0


def test_nccl_unique_id_through_the_c_abi():
    """The NCCL tier opens libnccl at run time; making a unique id needs no
    GPU, so this checks the loading and the call path on the CPU."""
    import ctypes as C
    from genllm_b200 import _lib
    L = _lib.lib()
    uid = (C.c_char * 128)()
    st = L.gkv_nccl_unique_id(uid)
    if st == _lib.GKV_ERR_UNSUPPORTED:
        pytest.skip("no libnccl.so.2 on this machine")
    assert st == 0, L.gkv_last_error()
    assert any(bytes(uid)), "unique id left empty"
    assert L.gkv_nccl_unique_id(None) == _lib.GKV_ERR_INVALID
