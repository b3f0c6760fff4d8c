"""ctypes binding of libgenllm_kv.so (the C ABI declared in include/genllm_kv.h).

The library is built in-tree by ``make -C genllm_b200/csrc`` (``__graft_entry__.build()``).
There is no fallback: if the shared object is missing, importing this module
raises, so a GPU run can never silently take another path.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# GKV_LIB points at another build of the same library (e.g. an instrumented
# one); by default the in-tree build is used.
LIB_PATH = os.environ.get("GKV_LIB") or os.path.join(_HERE, "libgenllm_kv.so")

GKV_OK = 0
GKV_ERR_INVALID = 1
GKV_ERR_NO_PAGES = 2
GKV_ERR_CUDA = 3
GKV_ERR_UNSUPPORTED = 4
GKV_ERR_STATE = 5
GKV_ERR_DEVICE = 6

GKV_F32, GKV_F16, GKV_BF16 = 0, 1, 30
GKV_KV_BF16, GKV_KV_FP8_E4M3 = 0, 1  # gkv_kv_format

i32 = C.c_int32
vp = C.c_void_p
i32p = C.POINTER(C.c_int32)
u32p = C.POINTER(C.c_uint32)


class LayerInfo(C.Structure):
    _fields_ = [("active", i32), ("num_cached", i32), ("n_pages", i32), ("max_blocks", i32),
                ("n_kv_heads", i32), ("head_dim", i32), ("dtype", i32), ("reserved", i32),
                ("k_base", vp), ("v_base", vp), ("device_table", vp)]


class PoolDesc(C.Structure):
    _fields_ = [("k_base", vp), ("v_base", vp), ("pool_pages", i32), ("n_kv_heads", i32),
                ("head_dim", i32), ("dtype", i32)]


class NewPages(C.Structure):
    _fields_ = [("first_new_page", i32), ("n_new_pages", i32), ("k_ids", i32p), ("v_ids", i32p)]


class QkNormDesc(C.Structure):
    _fields_ = [("q_norm_w", vp), ("k_norm_w", vp), ("cos_tab", vp), ("sin_tab", vp), ("max_seq", i32),
                ("eps", C.c_float)]


# name -> (argtypes, restype); every entry point returns an int status unless noted.
SIGNATURES = {
    "gkv_status_string": ([C.c_int], C.c_char_p),
    "gkv_last_error": ([], C.c_char_p),
    "gkv_manager_create": ([C.c_int, C.POINTER(vp)], C.c_int),
    "gkv_manager_destroy": ([vp], C.c_int),
    "gkv_init_layer": ([vp, i32, i32, i32, i32], C.c_int),
    "gkv_reserve_layer": ([vp, i32, i32, vp, vp], C.c_int),
    "gkv_is_active": ([vp, i32], C.c_int),
    "gkv_append_kv_pages": ([vp, i32, i32], C.c_int),
    "gkv_append_kv": ([vp, i32, vp, vp, i32, i32, i32, i32, vp], C.c_int),
    "gkv_paged_attention": ([vp, i32, vp, vp, vp, vp, i32, i32, i32, i32, i32, C.c_float, i32, i32, i32,
                             i32, vp], C.c_int),
    "gkv_reset": ([vp], C.c_int),
    "gkv_reset_layer": ([vp, i32], C.c_int),
    "gkv_get_layer_info": ([vp, i32, C.POINTER(LayerInfo)], C.c_int),
    "gkv_get_page_table": ([vp, i32, i32p, i32p, i32, i32p], C.c_int),
    "gkv_read_device_table": ([vp, i32, i32p, i32p, i32, i32p], C.c_int),
    "gkv_set_page_table": ([vp, i32, i32p, i32p, i32, i32, vp], C.c_int),
    "gkv_page_alloc": ([vp, i32, i32, i32p], C.c_int),
    "gkv_page_free": ([vp, i32, i32, i32], C.c_int),
    "gkv_pool_reset": ([vp, i32, i32], C.c_int),
    "gkv_pool_stats": ([vp, i32, i32, i32p, i32p, i32p], C.c_int),
    "gkv_check_device_errors": ([vp, i32, u32p], C.c_int),
    "gkv_table_create": ([C.c_int, i32, C.POINTER(vp)], C.c_int),
    "gkv_table_destroy": ([vp], C.c_int),
    "gkv_table_device_ptr": ([vp], vp),
    "gkv_table_check_errors": ([vp, u32p], C.c_int),
    "gkv_append_kv_raw": ([C.POINTER(PoolDesc), vp, i32, C.POINTER(NewPages), vp, vp, i32, vp], C.c_int),
    "gkv_paged_attention_raw": ([C.POINTER(PoolDesc), vp, i32, C.POINTER(NewPages), vp, vp, vp, vp, i32, i32,
                                 C.c_float, i32, i32, vp], C.c_int),
    "gkv_device_alloc": ([C.c_int, C.c_size_t, C.POINTER(vp)], C.c_int),
    "gkv_device_free": ([C.c_int, vp], C.c_int),
    "gkv_ipc_export": ([C.c_int, vp, vp], C.c_int),
    "gkv_ipc_open": ([C.c_int, vp, C.POINTER(vp)], C.c_int),
    "gkv_ipc_close": ([C.c_int, vp], C.c_int),
    "gkv_gather_create": ([C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(vp), C.POINTER(vp), C.POINTER(vp)], C.c_int),
    "gkv_gather_destroy": ([vp], C.c_int),
    "gkv_gather_set_wait_limit": ([vp, C.c_uint64], C.c_int),
    "gkv_nccl_unique_id": ([vp], C.c_int),
    "gkv_nccl_comm_create": ([C.c_int, C.c_int, C.c_int, vp, C.POINTER(vp)], C.c_int),
    "gkv_nccl_comm_destroy": ([vp], C.c_int),
    "gkv_allgather_heads": ([vp, vp, vp, C.c_size_t, vp], C.c_int),
    "gkv_paged_attention_gather": ([vp, i32, vp, vp, vp, vp, C.c_size_t, i32, C.c_float, i32, vp], C.c_int),
    "gkv_paged_decode_static_scratch": ([C.POINTER(PoolDesc), vp, i32, vp, vp, vp, vp, i32, C.c_float, i32, vp],
                                        C.c_int),
    "gkv_paged_decode_static_scratch_errors": ([u32p, vp], C.c_int),
    "gkv_rope_cache": ([C.c_float, i32, i32, vp, vp], C.c_int),
    "gkv_flash_attention": ([vp, vp, vp, vp, i32, i32, i32, i32, i32, C.c_float, i32, i32, i32, vp], C.c_int),
    "gkv_flash_check_errors": ([u32p], C.c_int),
    "gkv_decode_graph_create": ([vp, i32, i32p, C.POINTER(vp), C.POINTER(vp), C.POINTER(vp), C.POINTER(vp), i32,
                                 C.c_float, i32, C.POINTER(C.POINTER(QkNormDesc)), C.POINTER(vp)], C.c_int),
    "gkv_decode_graph_step": ([vp, vp], C.c_int),
    "gkv_decode_graph_destroy": ([vp], C.c_int),
    "gkv_export_kv_raw": ([C.POINTER(PoolDesc), vp, i32, i32, vp, vp, vp, vp, vp], C.c_int),
    "gkv_import_kv_raw": ([C.POINTER(PoolDesc), vp, i32, C.POINTER(NewPages), i32, vp, vp, vp, vp, i32, vp],
                          C.c_int),
    "gkv_export_kv": ([vp, i32, i32, vp, vp, vp, vp, i32p, vp], C.c_int),
    "gkv_import_kv": ([vp, i32, i32, vp, vp, vp, vp, i32, vp], C.c_int),
    "gkv_decode_layers": ([vp, i32, i32p, C.POINTER(vp), C.POINTER(vp), C.POINTER(vp), C.POINTER(vp), i32, C.c_float,
                           i32, vp], C.c_int),
    "gkv_qk_norm_rope": ([vp, vp, vp, i32, i32, i32, C.POINTER(QkNormDesc), i32, vp, vp, vp, vp], C.c_int),
    "gkv_paged_attention_raw_qknorm": ([C.POINTER(PoolDesc), vp, i32, C.POINTER(NewPages), vp, vp, vp, vp, i32, i32,
                                        C.c_float, i32, i32, C.POINTER(QkNormDesc), vp], C.c_int),
    "gkv_paged_attention_qknorm": ([vp, i32, vp, vp, vp, vp, i32, i32, C.c_float, i32, i32, C.POINTER(QkNormDesc),
                                    vp], C.c_int),
}


class GkvError(RuntimeError):
    """A non-zero gkv_status, with the library's message."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C genllm_b200/csrc` "
                              "(no CPU fallback exists)")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != GKV_OK:
        msg = lib().gkv_last_error().decode(errors="replace")
        raise GkvError(status, msg or lib().gkv_status_string(status).decode())
