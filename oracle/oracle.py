"""ctypes bindings to the test-only checkers built by oracle/Makefile.

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
bench.py's CPU-baseline / reference arm. The product package (genllm_b200)
never imports this module.

* :class:`Oracle` wraps ``liboracle.so``, the C restatement (paged_oracle.c) of
  the reference path: BlockPool (src/core/page_attention.cpp:25-64), the page
  appender (:104-162) and the CPU paged-attention op
  (src/backend/cpu/attention.cpp:156-215), returning fp32 before the final
  bf16 store.
* :class:`RefSession` wraps ``_ref/libgenllm_ref.so``, the reference's own CPU
  translation units plus ref_harness.cpp. It exists only where the reference
  tree was present when ``make ref`` ran.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libgenllm_ref.so")

F32, F16, BF16 = 0, 1, 30
PAGE_SLOTS = 16

_i32p = C.POINTER(C.c_int32)
_vp = C.c_void_p


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_vp)


def bf16_from_f32(x: np.ndarray) -> np.ndarray:
    """Vectorised restatement of include/utils/bfloat16.hpp:18-41 (RNE,
    exponent-0 inputs flushed to signed zero, NaN keeps one mantissa bit)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    sign = (u >> 31).astype(np.uint32)
    e = (u >> 23) & 0xFF
    m = u & 0x7FFFFF
    low = u & 0xFFFF
    up = (low > 0x8000) | ((low == 0x8000) & ((m & 0x10000) != 0))
    hm = (m >> 16) + up.astype(np.uint32)
    carry = hm >= 0x80
    e2 = e + carry.astype(np.uint32)
    hm = np.where(carry, 0, hm)
    out = (sign << 15) | (e2 << 7) | hm
    out = np.where(e2 >= 0xFF, (sign << 15) | 0x7F80, out)
    out = np.where(e == 0, sign << 15, out)
    out = np.where(e == 0xFF, (sign << 15) | 0x7F80 | (m != 0).astype(np.uint32), out)
    return out.astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


class Oracle:
    """The C restatement (liboracle.so)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle oracle`")
        L = self.lib = C.CDLL(path)
        L.orc_paged_attention_f32.argtypes = [_vp, C.c_int32, _vp, _vp, _vp, _vp] + [C.c_int32] * 7 + [C.c_float, C.c_int, _vp]
        L.orc_paged_attention_f32.restype = None
        L.orc_paged_attention_f32_mt.argtypes = L.orc_paged_attention_f32.argtypes + [C.c_int32]
        L.orc_paged_attention_f32_mt.restype = None
        L.orc_paged_attention_rows.argtypes = ([_vp, C.c_int32, _vp, _vp, _vp, _vp] + [C.c_int32] * 7 +
                                               [C.c_float, C.c_int, _vp, C.c_int32, _vp, C.c_int32])
        L.orc_paged_attention_rows.restype = None
        L.orc_bf16_from_f32.argtypes = [C.c_float]
        L.orc_bf16_from_f32.restype = C.c_uint16
        L.orc_round_bf16.argtypes = [_vp, _vp, C.c_size_t]
        L.orc_rms_norm_bf16.argtypes = [_vp, _vp, _vp, C.c_int64, C.c_int64, C.c_float]
        L.orc_rms_norm_bf16.restype = None
        L.orc_apply_rope_bf16.argtypes = [_vp, _vp, _vp, _vp] + [C.c_int64] * 4
        L.orc_apply_rope_bf16.restype = None
        L.orc_rope_cache.argtypes = [C.c_float, C.c_int32, C.c_int32, _vp, _vp]
        L.orc_rope_cache.restype = None
        L.orc_flash_attention_f32.argtypes = [_vp, _vp, _vp] + [C.c_int32] * 6 + [C.c_float, C.c_int, _vp]
        L.orc_flash_attention_f32.restype = None
        L.orc_e4m3_from_f32.argtypes = [C.c_float]
        L.orc_e4m3_from_f32.restype = C.c_uint8
        L.orc_e4m3_to_f32.argtypes = [C.c_uint8]
        L.orc_e4m3_to_f32.restype = C.c_float
        L.orc_export_kv.argtypes = [_vp, _vp, _vp, _vp] + [C.c_int32] * 3 + [C.c_int, _vp, _vp, _vp, _vp]
        L.orc_export_kv.restype = None
        L.orc_import_fp8.argtypes = [_vp, _vp, _vp, _vp, C.c_int32, _vp, _vp, _vp, _vp] + [C.c_int32] * 3
        L.orc_import_fp8.restype = None

    def paged_attention_f32(self, q, k_pool, v_pool, k_ids, v_ids, total, n_q_heads, n_kv_heads,
                            seq_len, head_dim, scale, causal=True, dtype=BF16, threads=0):
        """q: uint16 [Hq][S][D]; pools: flat uint16 arrays of the page layout
        [page][16][Hkv][D]; returns fp32 [Hq][S][D]."""
        q = np.ascontiguousarray(q)
        k_ids = np.ascontiguousarray(k_ids, dtype=np.int32)
        v_ids = np.ascontiguousarray(v_ids, dtype=np.int32)
        out = np.empty((n_q_heads, seq_len, head_dim), dtype=np.float32)
        args = [_ptr(q), dtype, _ptr(k_pool), _ptr(v_pool), _ptr(k_ids), _ptr(v_ids),
                len(k_ids), total, n_q_heads, n_kv_heads, seq_len, head_dim,
                n_q_heads // n_kv_heads, scale, int(bool(causal)), _ptr(out)]
        if threads:
            self.lib.orc_paged_attention_f32_mt(*args, int(threads))
        else:
            self.lib.orc_paged_attention_f32(*args)
        return out

    def paged_attention_rows(self, q, k_pool, v_pool, k_ids, v_ids, total, n_q_heads, n_kv_heads,
                             seq_len, head_dim, scale, rows, causal=True, dtype=BF16, threads=1):
        """Only the listed output rows (r = head * seq_len + query): fp32 [len(rows)][D]."""
        q = np.ascontiguousarray(q)
        k_ids = np.ascontiguousarray(k_ids, dtype=np.int32)
        v_ids = np.ascontiguousarray(v_ids, dtype=np.int32)
        rows = np.ascontiguousarray(rows, dtype=np.int32)
        out = np.empty((len(rows), head_dim), dtype=np.float32)
        self.lib.orc_paged_attention_rows(_ptr(q), dtype, _ptr(k_pool), _ptr(v_pool), _ptr(k_ids), _ptr(v_ids),
                                          len(k_ids), total, n_q_heads, n_kv_heads, seq_len, head_dim,
                                          n_q_heads // n_kv_heads, scale, int(bool(causal)), _ptr(rows),
                                          len(rows), _ptr(out), int(threads))
        return out

    def round_bf16(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(x.shape, dtype=np.uint16)
        self.lib.orc_round_bf16(_ptr(x), _ptr(out), x.size)
        return out

    def rms_norm_bf16(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        """Rows of x (uint16 bf16, last axis = len(w)) normalised: qk_rope_oracle.c."""
        x = np.ascontiguousarray(x, dtype=np.uint16)
        w = np.ascontiguousarray(w, dtype=np.float32)
        out = np.empty_like(x)
        self.lib.orc_rms_norm_bf16(_ptr(x), _ptr(w), _ptr(out), x.size // w.size, w.size, eps)
        return out

    def apply_rope_bf16(self, x: np.ndarray, cos: np.ndarray, sin: np.ndarray, start_pos: int) -> np.ndarray:
        """x: uint16 [H][S][D]; cos/sin f32 [max_seq][D]."""
        x = np.ascontiguousarray(x, dtype=np.uint16)
        cos = np.ascontiguousarray(cos, dtype=np.float32)
        sin = np.ascontiguousarray(sin, dtype=np.float32)
        out = np.empty_like(x)
        H, S, D = x.shape
        self.lib.orc_apply_rope_bf16(_ptr(x), _ptr(out), _ptr(cos), _ptr(sin), H, S, D, start_pos)
        return out

    def rope_cache(self, theta: float, head_dim: int, max_seq: int):
        cos = np.empty((max_seq, head_dim), dtype=np.float32)
        sin = np.empty((max_seq, head_dim), dtype=np.float32)
        self.lib.orc_rope_cache(theta, head_dim, max_seq, _ptr(cos), _ptr(sin))
        return cos, sin

    def e4m3_from_f32(self, x: np.ndarray) -> np.ndarray:
        """Elementwise OCP e4m3 encoding (kv_format_oracle.c), uint8."""
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        return np.array([self.lib.orc_e4m3_from_f32(float(v)) for v in x], dtype=np.uint8)

    def e4m3_to_f32(self, b: np.ndarray) -> np.ndarray:
        b = np.ascontiguousarray(b, dtype=np.uint8).ravel()
        return np.array([self.lib.orc_e4m3_to_f32(int(v)) for v in b], dtype=np.float32)

    def export_kv(self, k_pool, v_pool, k_ids, v_ids, n_tokens, n_kv_heads, head_dim=128, fp8=False):
        """Pages -> dense [Hkv][n_tokens][D]: uint16 (bf16) or uint8 (e4m3) arrays,
        plus fp32 scales [Hkv][blocks] for fp8 (None for bf16)."""
        k_ids = np.ascontiguousarray(k_ids, dtype=np.int32)
        v_ids = np.ascontiguousarray(v_ids, dtype=np.int32)
        dt = np.uint8 if fp8 else np.uint16
        ko = np.zeros((n_kv_heads, n_tokens, head_dim), dtype=dt)
        vo = np.zeros_like(ko)
        nb = (n_tokens + 15) // 16
        ks = np.zeros((n_kv_heads, nb), dtype=np.float32)
        vs = np.zeros_like(ks)
        self.lib.orc_export_kv(_ptr(k_pool), _ptr(v_pool), _ptr(k_ids), _ptr(v_ids), n_tokens, n_kv_heads, head_dim,
                               int(bool(fp8)), _ptr(ko), _ptr(vo), _ptr(ks), _ptr(vs))
        return ko, vo, (ks if fp8 else None), (vs if fp8 else None)

    def import_fp8(self, k_pool, v_pool, k_ids, v_ids, n_prior, k_in, v_in, k_scales, v_scales):
        """Dequantise e4m3 [Hkv][S][D] into the pools in place (kv_format_oracle.c)."""
        k_ids = np.ascontiguousarray(k_ids, dtype=np.int32)
        v_ids = np.ascontiguousarray(v_ids, dtype=np.int32)
        k_in, v_in = (np.ascontiguousarray(a, dtype=np.uint8) for a in (k_in, v_in))
        k_scales, v_scales = (np.ascontiguousarray(a, dtype=np.float32) for a in (k_scales, v_scales))
        Hkv, S, D = k_in.shape
        self.lib.orc_import_fp8(_ptr(k_pool), _ptr(v_pool), _ptr(k_ids), _ptr(v_ids), n_prior, _ptr(k_in),
                                _ptr(v_in), _ptr(k_scales), _ptr(v_scales), S, Hkv, D)

    def flash_attention_f32(self, q, k, v, scale, causal=True):
        """q uint16 [B][Hq][S][D], k/v [B][Hkv][S][D] -> fp32 [B][Hq][S][D]
        (flash_oracle.c)."""
        q, k, v = (np.ascontiguousarray(a, dtype=np.uint16) for a in (q, k, v))
        B, Hq, S, D = q.shape
        Hkv = k.shape[1]
        out = np.empty((B, Hq, S, D), dtype=np.float32)
        self.lib.orc_flash_attention_f32(_ptr(q), _ptr(k), _ptr(v), B, Hq, Hkv, S, D, Hq // Hkv, scale,
                                         int(bool(causal)), _ptr(out))
        return out


class OraclePool:
    """The restated BlockPool + page table of one layer (paged_oracle.c)."""

    class _Pool(C.Structure):
        _fields_ = [("capacity", C.c_int32), ("num_blocks", C.c_int32), ("n_free", C.c_int32),
                    ("free_list", _i32p)]

    class _Layer(C.Structure):
        pass

    _Layer._fields_ = [("num_cached", C.c_int32), ("n_pages", C.c_int32), ("table_cap", C.c_int32),
                       ("k_ids", _i32p), ("v_ids", _i32p), ("k_pool", _Pool), ("v_pool", _Pool)]

    def __init__(self, max_pages: int, oracle: Oracle | None = None):
        self.o = oracle or Oracle()
        L = self.o.lib
        for name, args, res in [
            ("orc_layer_init", [C.c_void_p, C.c_int32], C.c_int),
            ("orc_layer_release", [C.c_void_p], None),
            ("orc_layer_append_pages", [C.c_void_p, C.c_int32], C.c_int32),
            ("orc_layer_reset", [C.c_void_p], None),
            ("orc_pool_alloc", [C.c_void_p], C.c_int32),
            ("orc_pool_free", [C.c_void_p, C.c_int32], None),
            ("orc_pool_reset", [C.c_void_p], None),
            ("orc_layer_append_kv", [C.c_void_p, _vp, _vp, _vp, _vp] + [C.c_int32] * 4, None),
        ]:
            getattr(L, name).argtypes = args
            getattr(L, name).restype = res
        self.layer = self._Layer()
        if L.orc_layer_init(C.byref(self.layer), max_pages) != 0:
            raise MemoryError("orc_layer_init")

    def __del__(self):
        try:
            self.o.lib.orc_layer_release(C.byref(self.layer))
        except Exception:
            pass

    def _pool(self, which):
        return C.byref(self.layer, self._Layer.k_pool.offset if which == 0 else self._Layer.v_pool.offset)

    def alloc(self, which=0):
        return self.o.lib.orc_pool_alloc(self._pool(which))

    def free(self, which, page_id):
        self.o.lib.orc_pool_free(self._pool(which), page_id)

    def pool_reset(self, which):
        self.o.lib.orc_pool_reset(self._pool(which))

    def stats(self, which=0):
        p = self.layer.k_pool if which == 0 else self.layer.v_pool
        return p.num_blocks, p.n_free

    def append_pages(self, count):
        return self.o.lib.orc_layer_append_pages(C.byref(self.layer), count)

    def reset(self):
        self.o.lib.orc_layer_reset(C.byref(self.layer))

    def set_table(self, k_ids, v_ids, num_cached):
        n = len(k_ids)
        assert n <= self.layer.table_cap
        for i in range(n):
            self.layer.k_ids[i] = int(k_ids[i])
            self.layer.v_ids[i] = int(v_ids[i])
        self.layer.n_pages = n
        self.layer.num_cached = num_cached

    def table(self):
        n = self.layer.n_pages
        return (np.array([self.layer.k_ids[i] for i in range(n)], dtype=np.int32),
                np.array([self.layer.v_ids[i] for i in range(n)], dtype=np.int32))

    @property
    def num_cached(self):
        return self.layer.num_cached

    def append_kv(self, k_pool, v_pool, K, V, n_kv_heads, seq_len, head_dim, elem_bytes=2):
        K = np.ascontiguousarray(K)
        V = np.ascontiguousarray(V)
        self.o.lib.orc_layer_append_kv(C.byref(self.layer), _ptr(k_pool), _ptr(v_pool), _ptr(K), _ptr(V),
                                       n_kv_heads, seq_len, head_dim, elem_bytes)


def ref_available() -> bool:
    return os.path.exists(REF_SO)


REF_OPS_SO = os.path.join(HERE, "_ref", "libgenllm_ref_ops.so")


def ref_ops_available() -> bool:
    return os.path.exists(REF_OPS_SO)


class RefOps:
    """The reference's own CPU RMSNorm / RoPE / RoPE-cache ops
    (oracle/_ref/libgenllm_ref_ops.so, built with the reference's CPU flags)."""

    def __init__(self, path: str = REF_OPS_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref` where the reference tree exists")
        L = self.lib = C.CDLL(path)
        L.ref_rms_norm.argtypes = [_vp, _vp, _vp, C.c_int64, C.c_int64, C.c_float]
        L.ref_rms_norm.restype = None
        L.ref_apply_rope.argtypes = [_vp, _vp, _vp, _vp] + [C.c_int64] * 5
        L.ref_apply_rope.restype = None
        L.ref_rope_cache.argtypes = [C.c_float, C.c_int32, C.c_int32, _vp, _vp]
        L.ref_rope_cache.restype = None

    def rms_norm_bf16(self, x, w, eps):
        x = np.ascontiguousarray(x, dtype=np.uint16)
        w = np.ascontiguousarray(w, dtype=np.float32)
        out = np.empty_like(x)
        self.lib.ref_rms_norm(_ptr(x), _ptr(w), _ptr(out), x.size // w.size, w.size, eps)
        return out

    def apply_rope_bf16(self, x, cos, sin, start_pos):
        x = np.ascontiguousarray(x, dtype=np.uint16)
        cos = np.ascontiguousarray(cos, dtype=np.float32)
        sin = np.ascontiguousarray(sin, dtype=np.float32)
        out = np.empty_like(x)
        H, S, D = x.shape
        self.lib.ref_apply_rope(_ptr(x), _ptr(out), _ptr(cos), _ptr(sin), H, S, D, start_pos, cos.shape[0])
        return out

    def rope_cache(self, theta, head_dim, max_seq):
        cos = np.empty((max_seq, head_dim), dtype=np.float32)
        sin = np.empty((max_seq, head_dim), dtype=np.float32)
        self.lib.ref_rope_cache(theta, head_dim, max_seq, _ptr(cos), _ptr(sin))
        return cos, sin


class RefSession:
    """The reference's own CPU op and allocator (oracle/_ref/libgenllm_ref.so)."""

    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            if not os.path.exists(REF_SO):
                raise FileNotFoundError(f"{REF_SO} missing: run `make -C oracle ref` where the reference tree exists")
            L = C.CDLL(REF_SO)
            sig = {
                "ref_session_create": ([C.c_int32] * 5, _vp),
                "ref_session_destroy": ([_vp], None),
                "ref_layer_k_base": ([_vp, C.c_int32], _vp),
                "ref_layer_v_base": ([_vp, C.c_int32], _vp),
                "ref_page_alloc": ([_vp, C.c_int32, C.c_int32], C.c_int32),
                "ref_page_free": ([_vp, C.c_int32, C.c_int32, C.c_int32], None),
                "ref_pool_stats": ([_vp, C.c_int32, C.c_int32, _i32p, _i32p], None),
                "ref_set_table": ([_vp, C.c_int32, _vp, _vp, C.c_int32, C.c_int32], None),
                "ref_get_table": ([_vp, C.c_int32, _vp, _vp, C.c_int32, _i32p], C.c_int32),
                "ref_append_pages": ([_vp, C.c_int32, C.c_int32], None),
                "ref_append_kv": ([_vp, C.c_int32, _vp, _vp, C.c_int32], None),
                "ref_reset": ([_vp], None),
                "ref_paged_attention": ([_vp, C.c_int32, _vp, _vp, _vp, _vp, C.c_int32, C.c_int32,
                                         C.c_float, C.c_int32], None),
                "ref_paged_attention_layers": ([_vp, C.c_int32, _vp, _vp, _vp, _vp, C.c_int32,
                                                C.c_int32, C.c_float, C.c_int32], None),
                "ref_flash_attention": ([_vp, _vp, _vp, _vp] + [C.c_int32] * 5 + [C.c_float, C.c_int32], None),
            }
            for k, (a, r) in sig.items():
                getattr(L, k).argtypes = a
                getattr(L, k).restype = r
            cls._lib = L
        return cls._lib

    def __init__(self, n_layers, n_kv_heads, head_dim, max_blocks, dtype=BF16):
        self.L = self.lib()
        self.n_layers, self.n_kv_heads, self.head_dim, self.max_blocks = n_layers, n_kv_heads, head_dim, max_blocks
        self.h = self.L.ref_session_create(n_layers, n_kv_heads, head_dim, max_blocks, dtype)
        self.page_elems = PAGE_SLOTS * n_kv_heads * head_dim

    def close(self):
        if self.h:
            self.L.ref_session_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def pool_view(self, layer, which):
        """uint16 view [max_blocks][16][Hkv][D] of a layer's K (0) or V (1) region."""
        base = self.L.ref_layer_k_base(self.h, layer) if which == 0 else self.L.ref_layer_v_base(self.h, layer)
        n = self.max_blocks * self.page_elems
        buf = (C.c_uint16 * n).from_address(base)
        return np.ctypeslib.as_array(buf).reshape(self.max_blocks, PAGE_SLOTS, self.n_kv_heads, self.head_dim)

    def alloc(self, layer, which):
        return self.L.ref_page_alloc(self.h, layer, which)

    def free(self, layer, which, page_id):
        self.L.ref_page_free(self.h, layer, which, page_id)

    def stats(self, layer, which):
        a, b = C.c_int32(), C.c_int32()
        self.L.ref_pool_stats(self.h, layer, which, C.byref(a), C.byref(b))
        return a.value, b.value

    def set_table(self, layer, k_ids, v_ids, num_cached):
        k = np.ascontiguousarray(k_ids, dtype=np.int32)
        v = np.ascontiguousarray(v_ids, dtype=np.int32)
        self.L.ref_set_table(self.h, layer, _ptr(k), _ptr(v), len(k), num_cached)

    def table(self, layer):
        cap = self.max_blocks + 1
        k = np.zeros(cap, np.int32)
        v = np.zeros(cap, np.int32)
        nc = C.c_int32()
        n = self.L.ref_get_table(self.h, layer, _ptr(k), _ptr(v), cap, C.byref(nc))
        return k[:n].copy(), v[:n].copy(), nc.value

    def append_pages(self, layer, count):
        self.L.ref_append_pages(self.h, layer, count)

    def append_kv(self, layer, K, V, seq_len):
        K = np.ascontiguousarray(K)
        V = np.ascontiguousarray(V)
        self.L.ref_append_kv(self.h, layer, _ptr(K), _ptr(V), seq_len)

    def reset(self):
        self.L.ref_reset(self.h)

    def paged_attention(self, layer, Q, K, V, n_q_heads, seq_len, scale, causal=True):
        """Returns the reference op's bf16 output [Hq][S][D] (uint16)."""
        Q = np.ascontiguousarray(Q)
        K = np.ascontiguousarray(K)
        V = np.ascontiguousarray(V)
        out = np.zeros((n_q_heads, seq_len, self.head_dim), np.uint16)
        self.L.ref_paged_attention(self.h, layer, _ptr(Q), _ptr(K), _ptr(V), _ptr(out), n_q_heads,
                                   seq_len, scale, int(bool(causal)))
        return out

    def paged_attention_layers(self, Qs, Ks, Vs, outs, n_q_heads, seq_len, scale, causal=True):
        n = len(Qs)
        arr = lambda xs: (C.c_void_p * n)(*[x.ctypes.data for x in xs])
        self.L.ref_paged_attention_layers(self.h, n, arr(Qs), arr(Ks), arr(Vs), arr(outs), n_q_heads,
                                          seq_len, scale, int(bool(causal)))


# ---- one paged-attention step on a fragmented cache -----------------------
#
# Both checkers build the same state the product tests build: every pool page
# handed out (ids 0..P-1 in order), the pages outside the table returned to
# the free list in the case's free order, the table set to the case's
# permutation with n_prior tokens cached. The step then appends n_new tokens
# (taking pages from the free list, LIFO) and attends.

def run_oracle_case(case, oracle: Oracle | None = None, causal=True, threads=0):
    """Returns (out_f32 [Hq][S][D], k_pool, v_pool, k_ids, v_ids, num_cached)
    from the C restatement."""
    o = oracle or Oracle()
    pool = OraclePool(case.pool_pages, o)
    for w, order in ((0, case.k_free_order), (1, case.v_free_order)):
        for _ in range(case.pool_pages):
            pool.alloc(w)
        for i in order:
            pool.free(w, int(i))
    pool.set_table(case.k_ids, case.v_ids, case.n_prior)
    kp = case.k_pool.copy()
    vp = case.v_pool.copy()
    pool.append_kv(kp, vp, case.k_new, case.v_new, case.n_kv_heads, case.n_new, case.head_dim)
    k_ids, v_ids = pool.table()
    out = o.paged_attention_f32(case.q, kp, vp, k_ids, v_ids, pool.num_cached, case.n_q_heads,
                                case.n_kv_heads, case.n_new, case.head_dim, case.scale, causal,
                                threads=threads)
    return out, kp, vp, k_ids, v_ids, pool.num_cached


def run_ref_case(case, causal=True):
    """The reference op itself on the same state. Returns (out_bf16 [Hq][S][D],
    k_pool, v_pool, k_ids, v_ids, num_cached)."""
    ref = RefSession(1, case.n_kv_heads, case.head_dim, case.pool_pages)
    try:
        for w, order in ((0, case.k_free_order), (1, case.v_free_order)):
            for _ in range(case.pool_pages):
                ref.alloc(0, w)
            for i in order:
                ref.free(0, w, int(i))
        ref.pool_view(0, 0)[:] = case.k_pool
        ref.pool_view(0, 1)[:] = case.v_pool
        ref.set_table(0, case.k_ids, case.v_ids, case.n_prior)
        out = ref.paged_attention(0, case.q, case.k_new, case.v_new, case.n_q_heads, case.n_new,
                                  case.scale, causal)
        k_ids, v_ids, nc = ref.table(0)
        return out, ref.pool_view(0, 0).copy(), ref.pool_view(0, 1).copy(), k_ids, v_ids, nc
    finally:
        ref.close()


def ref_flash_attention(q, k, v, scale, causal=True):
    """The reference's FlashAttentionImpl<CPU> (oracle/_ref): bf16 out bits."""
    L = RefSession.lib()
    q, k, v = (np.ascontiguousarray(a, dtype=np.uint16) for a in (q, k, v))
    B, Hq, S, D = q.shape
    out = np.empty_like(q)
    L.ref_flash_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(out), B, Hq, k.shape[1], S, D, scale, int(bool(causal)))
    return out

