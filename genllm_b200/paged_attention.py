"""Python mirror of Genllm's paged-attention operator interface, on the C ABI.

Names, argument meaning and error behaviour follow the reference (paths
relative to the Genllm source tree):

* :class:`PagedAttentionManager` — ``PagedAttentionManager``
  (include/core/page_attention.h:52-89): ``init_layer``, ``reserve_layer``,
  ``append_kv_from_tensor``, ``append_kv_pages``, ``reset``, ``is_active``,
  ``get_layer``; the layer's K/V ``BlockPool`` s (page_attention.h:11-45) are
  reached through :meth:`PagedAttentionManager.pool`.
* :func:`paged_attention` — ``kernel::paged_attention`` /
  ``PagedAttentionImpl<Device::CUDA>::execute`` (include/core/kernels.h:32,
  src/backend/cuda/attention.cu:491-580): append this step's K/V into the
  layer's pages, then attend Q over the whole cache.

torch supplies device memory and the current stream only; all the work runs
in libgenllm_kv.so. Where the reference fails silently (inactive layer,
exhausted pool) this raises :class:`GkvError`.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import List, Optional

import torch

from . import _lib
from ._lib import GKV_BF16, GKV_F16, GKV_F32, GkvError, check, lib

PAGE_BLOCK_SIZE = 16

_TORCH_TO_GKV = {torch.float32: GKV_F32, torch.float16: GKV_F16, torch.bfloat16: GKV_BF16}
_GKV_TO_TORCH = {v: k for k, v in _TORCH_TO_GKV.items()}


def _stream_handle(device: Optional[torch.device], stream=None):
    if device is None:
        return C.c_void_p(0)
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return C.c_void_p(s.cuda_stream)


@dataclass
class PageEntry:
    """include/core/page_attention.h:47-50"""
    k_block_id: int
    v_block_id: int


@dataclass
class LayerState:
    """Snapshot of include/core/page_attention.h:57-66 (LayerState)."""
    active: bool
    num_cached: int
    n_kv_heads: int
    head_dim: int
    dtype: int
    max_blocks: int
    page_table: List[PageEntry] = field(default_factory=list)


class BlockPoolView:
    """The K (which=0) or V (which=1) BlockPool of one layer
    (src/core/page_attention.cpp:25-64)."""

    def __init__(self, mgr: "PagedAttentionManager", layer_id: int, which: int):
        self._m, self._layer, self._which = mgr, layer_id, which

    def alloc(self) -> int:
        """LIFO id, or -1 when exhausted (the reference's contract)."""
        out = C.c_int32(-1)
        st = lib().gkv_page_alloc(self._m.handle, self._layer, self._which, C.byref(out))
        if st == _lib.GKV_ERR_NO_PAGES:
            return -1
        check(st)
        return out.value

    def free(self, block_id: int) -> None:
        check(lib().gkv_page_free(self._m.handle, self._layer, self._which, int(block_id)))

    def reset(self) -> None:
        check(lib().gkv_pool_reset(self._m.handle, self._layer, self._which))

    def _stats(self):
        a, b, c = C.c_int32(), C.c_int32(), C.c_int32()
        check(lib().gkv_pool_stats(self._m.handle, self._layer, self._which, C.byref(a), C.byref(b), C.byref(c)))
        return a.value, b.value, c.value

    def num_blocks(self) -> int:
        return self._stats()[0]

    def num_free(self) -> int:
        return self._stats()[1]

    def capacity(self) -> int:
        return self._stats()[2]

    def empty(self) -> bool:
        return self.num_blocks() == 0


class PagedAttentionManager:
    """Per-device paged KV-cache manager (include/core/page_attention.h:52-89)."""

    def __init__(self, device: int | torch.device = 0):
        """``device=-1`` gives a host-only manager (page bookkeeping, no device
        memory), the counterpart of the reference's pool-less manager."""
        if isinstance(device, int) and device == -1:
            self.device = None
        else:
            dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
            if dev.type != "cuda":
                raise ValueError("the paged KV cache lives on a CUDA device")
            self.device = torch.device("cuda", dev.index if dev.index is not None else torch.cuda.current_device())
        h = C.c_void_p()
        check(lib().gkv_manager_create(-1 if self.device is None else self.device.index, C.byref(h)))
        self.handle = h
        self._regions = {}  # layer -> (k_pool tensor, v_pool tensor)

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().gkv_manager_destroy(self.handle)
            self.handle = None
            self._regions.clear()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- page_attention.cpp:72-101 -------------------------------------
    def init_layer(self, layer_id: int, n_kv_heads: int, head_dim: int, dtype: int = GKV_BF16) -> None:
        check(lib().gkv_init_layer(self.handle, layer_id, n_kv_heads, head_dim, dtype))

    def reserve_layer(self, layer_id: int, max_blocks: int,
                      k_region: Optional[torch.Tensor] = None, v_region: Optional[torch.Tensor] = None) -> None:
        """Give the layer K and V pools of max_blocks pages. Without regions the
        pools are torch allocations owned by this manager (exposed by
        :meth:`pool_tensors`); with regions they are caller memory."""
        info = self._info(layer_id)
        if self.device is None:
            check(lib().gkv_reserve_layer(self.handle, layer_id, max_blocks, None, None))
            return
        if k_region is None:
            shape = (max_blocks, PAGE_BLOCK_SIZE, info.n_kv_heads, info.head_dim)
            td = {GKV_BF16: torch.bfloat16, GKV_F16: torch.float16, GKV_F32: torch.float32}[info.dtype]
            k_region = torch.empty(shape, dtype=td, device=self.device)
            v_region = torch.empty(shape, dtype=td, device=self.device)
        check(lib().gkv_reserve_layer(self.handle, layer_id, max_blocks, C.c_void_p(k_region.data_ptr()),
                                      C.c_void_p(v_region.data_ptr())))
        self._regions[layer_id] = (k_region, v_region)

    def is_active(self, layer_id: int) -> bool:
        return bool(lib().gkv_is_active(self.handle, layer_id))

    # -- page_attention.cpp:104-162 -------------------------------------
    def append_kv_pages(self, layer_id: int, count: int) -> None:
        check(lib().gkv_append_kv_pages(self.handle, layer_id, count))

    def append_kv_from_tensor(self, layer_id: int, K: torch.Tensor, V: torch.Tensor, stream=None) -> None:
        """K, V: [1, Hkv, S, D] (or [Hkv, S, D]) contiguous on this device."""
        Kc, Vc = _kv_view(K), _kv_view(V)
        hkv, s, d = Kc.shape
        check(lib().gkv_append_kv(self.handle, layer_id, C.c_void_p(Kc.data_ptr()), C.c_void_p(Vc.data_ptr()),
                                  hkv, s, d, _TORCH_TO_GKV[Kc.dtype], _stream_handle(self.device, stream)))

    # -- format export / import (no reference counterpart) --------------
    def export_kv(self, layer_id: int, fp8: bool = False, stream=None):
        """The layer's cached tokens as dense head-major tensors [Hkv, n, D]:
        ``(K, V)`` in the pool dtype, or with ``fp8`` ``(K, V, k_scales,
        v_scales)``, K/V ``float8_e4m3fn`` and scales fp32 [Hkv, ceil(n/16)]
        (one per head and 16-token block). gkv_export_kv."""
        info = self._info(layer_id)
        n, hkv, d = info.num_cached, info.n_kv_heads, info.head_dim
        dt = torch.float8_e4m3fn if fp8 else _GKV_TO_TORCH[info.dtype]
        K = torch.empty((hkv, n, d), dtype=dt, device=self.device)
        V = torch.empty_like(K)
        nb = (n + PAGE_BLOCK_SIZE - 1) // PAGE_BLOCK_SIZE
        ks = torch.empty((hkv, nb), dtype=torch.float32, device=self.device) if fp8 else None
        vs = torch.empty_like(ks) if fp8 else None
        got = C.c_int32()
        check(lib().gkv_export_kv(self.handle, layer_id, _lib.GKV_KV_FP8_E4M3 if fp8 else _lib.GKV_KV_BF16,
                                  C.c_void_p(K.data_ptr()), C.c_void_p(V.data_ptr()),
                                  C.c_void_p(ks.data_ptr() if fp8 else 0), C.c_void_p(vs.data_ptr() if fp8 else 0),
                                  C.byref(got), _stream_handle(self.device, stream)))
        return (K, V, ks, vs) if fp8 else (K, V)

    def import_kv(self, layer_id: int, K: torch.Tensor, V: torch.Tensor, k_scales: Optional[torch.Tensor] = None,
                  v_scales: Optional[torch.Tensor] = None, stream=None) -> None:
        """Append dense head-major tokens [Hkv, S, D] to the layer: in the pool
        dtype (== append_kv_from_tensor), or e4m3 (``float8_e4m3fn`` / uint8)
        with their fp32 block scales [Hkv, ceil(S/16)]. gkv_import_kv."""
        Kc, Vc = _kv_view(K), _kv_view(V)
        fp8 = Kc.dtype in (torch.float8_e4m3fn, torch.uint8)
        if fp8 and (k_scales is None or v_scales is None):
            raise GkvError(_lib.GKV_ERR_INVALID, "e4m3 K/V need their block scales")
        if fp8:
            for t in (k_scales, v_scales):
                if t.dtype != torch.float32 or not t.is_contiguous() or t.device != Kc.device:
                    raise GkvError(_lib.GKV_ERR_INVALID, "scales must be contiguous fp32 on K's device")
        check(lib().gkv_import_kv(self.handle, layer_id, _lib.GKV_KV_FP8_E4M3 if fp8 else _lib.GKV_KV_BF16,
                                  C.c_void_p(Kc.data_ptr()), C.c_void_p(Vc.data_ptr()),
                                  C.c_void_p(k_scales.data_ptr() if fp8 else 0),
                                  C.c_void_p(v_scales.data_ptr() if fp8 else 0), Kc.shape[1],
                                  _stream_handle(self.device, stream)))

    # -- page_attention.cpp:205-216 -------------------------------------
    def reset(self) -> None:
        check(lib().gkv_reset(self.handle))

    def reset_layer(self, layer_id: int) -> None:
        check(lib().gkv_reset_layer(self.handle, layer_id))

    def get_layer(self, layer_id: int) -> LayerState:
        info = self._info(layer_id)
        k, v = self.page_table(layer_id)
        return LayerState(bool(info.active), info.num_cached, info.n_kv_heads, info.head_dim, info.dtype,
                          info.max_blocks, [PageEntry(int(a), int(b)) for a, b in zip(k, v)])

    def pool(self, layer_id: int, which: int) -> BlockPoolView:
        return BlockPoolView(self, layer_id, which)

    def pool_tensors(self, layer_id: int):
        """(K pool, V pool) tensors [max_blocks][16][Hkv][D] of the layer."""
        return self._regions[layer_id]

    def page_table(self, layer_id: int):
        n = C.c_int32()
        check(lib().gkv_get_page_table(self.handle, layer_id, None, None, 0, C.byref(n)))
        k = (C.c_int32 * max(n.value, 1))()
        v = (C.c_int32 * max(n.value, 1))()
        check(lib().gkv_get_page_table(self.handle, layer_id, k, v, n.value, C.byref(n)))
        return list(k)[: n.value], list(v)[: n.value]

    def set_page_table(self, layer_id: int, k_ids, v_ids, num_cached: int, stream=None) -> None:
        n = len(k_ids)
        ka = (C.c_int32 * max(n, 1))(*[int(x) for x in k_ids])
        va = (C.c_int32 * max(n, 1))(*[int(x) for x in v_ids])
        check(lib().gkv_set_page_table(self.handle, layer_id, ka, va, n, num_cached,
                                       _stream_handle(self.device, stream)))

    def device_table(self, layer_id: int):
        """The device copy of the block table (synchronises): (k_ids, v_ids)."""
        n = C.c_int32()
        check(lib().gkv_read_device_table(self.handle, layer_id, None, None, 0, C.byref(n)))
        k = (C.c_int32 * max(n.value, 1))()
        v = (C.c_int32 * max(n.value, 1))()
        check(lib().gkv_read_device_table(self.handle, layer_id, k, v, n.value, C.byref(n)))
        return list(k)[: n.value], list(v)[: n.value]

    def check_device_errors(self, layer_id: int) -> int:
        f = C.c_uint32()
        check(lib().gkv_check_device_errors(self.handle, layer_id, C.byref(f)))
        return f.value

    def _info(self, layer_id: int) -> _lib.LayerInfo:
        info = _lib.LayerInfo()
        check(lib().gkv_get_layer_info(self.handle, layer_id, C.byref(info)))
        return info


def _kv_view(t: torch.Tensor) -> torch.Tensor:
    if t.dim() == 4:
        if t.shape[0] != 1:
            raise GkvError(_lib.GKV_ERR_UNSUPPORTED, "batch must be 1")
        t = t[0]
    if t.dim() != 3 or not t.is_contiguous():
        raise GkvError(_lib.GKV_ERR_INVALID, "expected a contiguous [1, H, S, D] tensor")
    return t


def paged_attention(manager: PagedAttentionManager, layer_id: int, Q: torch.Tensor, K: torch.Tensor,
                    V: torch.Tensor, out: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                    causal: bool = True, num_kv_groups: Optional[int] = None, stream=None) -> torch.Tensor:
    """``PagedAttentionImpl<CUDA>::execute`` on torch tensors.

    Q: [1, Hq, S, D]; K, V: [1, Hkv, S, D] (post-RoPE, post-QK-norm); out
    (optional, preallocated like the reference's activation-pool output):
    [1, Hq, S, D] in any of f32/f16/bf16 — Q's dtype by default, as the
    reference. ``scale`` defaults to 1/sqrt(D) (op_params[1]), ``causal`` is
    op_params[2], ``num_kv_groups`` = Hq / Hkv (op_params[3]).
    """
    if Q.dim() != 4 or K.dim() != 4 or V.dim() != 4:
        raise GkvError(_lib.GKV_ERR_INVALID, "Q, K, V must be [B, H, S, D]")
    B, Hq, S, D = Q.shape
    Hkv = K.shape[1]
    if out is None:
        out = torch.empty_like(Q)
    groups = num_kv_groups if num_kv_groups is not None else Hq // Hkv
    sc = float(scale) if scale is not None else 1.0 / float(D) ** 0.5
    for t in (Q, K, V, out):
        if not t.is_contiguous() or t.device != manager.device:
            raise GkvError(_lib.GKV_ERR_INVALID, "tensors must be contiguous and on the manager's device")
    check(lib().gkv_paged_attention(manager.handle, layer_id, C.c_void_p(Q.data_ptr()), C.c_void_p(K.data_ptr()),
                                    C.c_void_p(V.data_ptr()), C.c_void_p(out.data_ptr()), B, Hq, S, D, Hkv, sc,
                                    1 if causal else 0, groups, _TORCH_TO_GKV[Q.dtype], _TORCH_TO_GKV[out.dtype],
                                    _stream_handle(manager.device, stream)))
    return out


def rope_cache(theta: float, head_dim: int, max_seq: int):
    """``RopeCacheImpl<CPU>`` tables [max_seq, head_dim] fp32 (host numpy),
    computed by the library (gkv_rope_cache)."""
    import numpy as np
    cos = np.empty((max_seq, head_dim), dtype=np.float32)
    sin = np.empty((max_seq, head_dim), dtype=np.float32)
    check(lib().gkv_rope_cache(float(theta), head_dim, max_seq, C.c_void_p(cos.ctypes.data),
                               C.c_void_p(sin.ctypes.data)))
    return cos, sin


class QkNorm:
    """Qwen3's per-head QK-norm + RoPE parameters on a device: the two
    RMSNorm weights [128] fp32, eps and the RoPE tables for max_seq positions.
    """

    def __init__(self, q_norm_w: torch.Tensor, k_norm_w: torch.Tensor, eps: float, theta: float, max_seq: int,
                 device: int | torch.device = 0):
        dev = torch.device("cuda", device) if isinstance(device, int) else device
        cos, sin = rope_cache(theta, 128, max_seq)
        self.q_w = q_norm_w.to(device=dev, dtype=torch.float32).contiguous()
        self.k_w = k_norm_w.to(device=dev, dtype=torch.float32).contiguous()
        self.cos = torch.from_numpy(cos).to(dev)
        self.sin = torch.from_numpy(sin).to(dev)
        self.eps = float(eps)
        self.max_seq = max_seq
        self.desc = _lib.QkNormDesc(self.q_w.data_ptr(), self.k_w.data_ptr(), self.cos.data_ptr(),
                                    self.sin.data_ptr(), max_seq, self.eps)


def qk_norm_rope(q_flat: torch.Tensor, k_flat: torch.Tensor, v_flat: torch.Tensor, n_q_heads: int,
                 n_kv_heads: int, qk: QkNorm, start_pos: int, stream=None):
    """[S, H*128] projections -> ([Hq, S, 128], [Hkv, S, 128], [Hkv, S, 128])
    bf16: QK-norm + RoPE of Q and K, head-major permute of all three, in one
    launch (gkv_qk_norm_rope)."""
    S = q_flat.shape[0]
    dev = q_flat.device
    q = torch.empty((n_q_heads, S, 128), dtype=torch.bfloat16, device=dev)
    k = torch.empty((n_kv_heads, S, 128), dtype=torch.bfloat16, device=dev)
    v = torch.empty((n_kv_heads, S, 128), dtype=torch.bfloat16, device=dev)
    for t in (q_flat, k_flat, v_flat):
        if t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise GkvError(_lib.GKV_ERR_INVALID, "projections must be contiguous bf16")
    check(lib().gkv_qk_norm_rope(C.c_void_p(q_flat.data_ptr()), C.c_void_p(k_flat.data_ptr()),
                                 C.c_void_p(v_flat.data_ptr()), S, n_q_heads, n_kv_heads, C.byref(qk.desc),
                                 start_pos, C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()),
                                 C.c_void_p(v.data_ptr()), _stream_handle(dev, stream)))
    return q, k, v


def paged_attention_qknorm(manager: PagedAttentionManager, layer_id: int, q_flat: torch.Tensor,
                           k_flat: torch.Tensor, v_flat: torch.Tensor, n_q_heads: int, qk: QkNorm,
                           out: Optional[torch.Tensor] = None, scale: Optional[float] = None, causal: bool = True,
                           stream=None) -> torch.Tensor:
    """The attention op on the Q/K/V projections ([S, H*128] bf16): QK-norm +
    RoPE at the layer's next positions, append, attend — one launch for a
    decode step (gkv_paged_attention_qknorm). out: [Hq, S, 128]."""
    S = q_flat.shape[0]
    if out is None:
        out = torch.empty((n_q_heads, S, 128), dtype=torch.bfloat16, device=q_flat.device)
    sc = float(scale) if scale is not None else 1.0 / 128.0 ** 0.5
    for t in (q_flat, k_flat, v_flat, out):
        if not t.is_contiguous() or t.device != manager.device:
            raise GkvError(_lib.GKV_ERR_INVALID, "tensors must be contiguous and on the manager's device")
    check(lib().gkv_paged_attention_qknorm(manager.handle, layer_id, C.c_void_p(q_flat.data_ptr()),
                                           C.c_void_p(k_flat.data_ptr()), C.c_void_p(v_flat.data_ptr()),
                                           C.c_void_p(out.data_ptr()), n_q_heads, S, sc, 1 if causal else 0,
                                           _TORCH_TO_GKV[out.dtype], C.byref(qk.desc),
                                           _stream_handle(manager.device, stream)))
    return out


class DecodeStep:
    """One decode token through a fixed list of layers with one library call
    (gkv_decode_layers). The tensors are bound once: Q [Hq, 128] and K, V
    [Hkv, 128] per layer (any views of device memory), out [Hq, 128]; each
    ``run()`` appends one token to every layer and attends. The layers are
    independent: their inputs are complete before ``run()`` and no layer's
    out is another's Q/K/V (layer i + 1's kernels start while layer i
    finishes)."""

    def __init__(self, manager: PagedAttentionManager, layer_ids, Qs, Ks, Vs, outs, n_q_heads: int,
                 scale: Optional[float] = None):
        n = len(layer_ids)
        self.manager = manager
        self._keep = (list(Qs), list(Ks), list(Vs), list(outs))
        for group in self._keep:
            if len(group) != n or any((not t.is_contiguous()) or t.device != manager.device for t in group):
                raise GkvError(_lib.GKV_ERR_INVALID, "one contiguous tensor per layer, on the manager's device")
        self._ids = (C.c_int32 * n)(*layer_ids)
        arr = lambda ts: (C.c_void_p * n)(*[t.data_ptr() for t in ts])  # noqa: E731
        self._q, self._k, self._v, self._o = (arr(t) for t in self._keep)
        self._n = n
        self._hq = n_q_heads
        self._scale = float(scale) if scale is not None else 1.0 / 128.0 ** 0.5
        self._odt = _TORCH_TO_GKV[self._keep[3][0].dtype] if n else GKV_BF16

    def run(self, stream=None) -> None:
        check(lib().gkv_decode_layers(self.manager.handle, self._n, self._ids, self._q, self._k, self._v, self._o,
                                      self._hq, self._scale, self._odt, _stream_handle(self.manager.device, stream)))


class DecodeGraph(DecodeStep):
    """:class:`DecodeStep` captured once as a CUDA graph (gkv_decode_graph_*):
    each ``run()`` is one graph launch for all layers, with the step state
    (cached lengths, page counts, split geometry, new page ids) copied to the
    device by the graph's first node. Same results as DecodeStep. With
    ``qk`` (one :class:`QkNorm` per layer) Q and K are the projections and
    QK-norm + RoPE run inside the decode kernel."""

    def __init__(self, manager: PagedAttentionManager, layer_ids, Qs, Ks, Vs, outs, n_q_heads: int,
                 scale: Optional[float] = None, qk=None):
        super().__init__(manager, layer_ids, Qs, Ks, Vs, outs, n_q_heads, scale)
        qk_arr = None
        if qk is not None:
            self._qk = list(qk)
            if len(self._qk) != self._n:
                raise GkvError(_lib.GKV_ERR_INVALID, "one QkNorm per layer")
            qk_arr = (C.POINTER(_lib.QkNormDesc) * self._n)(*[C.pointer(q.desc) for q in self._qk])
        self._qk_arr = qk_arr
        h = C.c_void_p()
        check(lib().gkv_decode_graph_create(self.manager.handle, self._n, self._ids, self._q, self._k, self._v,
                                            self._o, self._hq, self._scale, self._odt, qk_arr, C.byref(h)))
        self.handle = h

    def run(self, stream=None) -> None:
        check(lib().gkv_decode_graph_step(self.handle, _stream_handle(self.manager.device, stream)))

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().gkv_decode_graph_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def flash_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, out: Optional[torch.Tensor] = None,
                    scale: Optional[float] = None, causal: bool = True, stream=None) -> torch.Tensor:
    """``FlashAttentionImpl<CUDA>::execute`` on torch tensors: Q [B, Hq, S, D],
    K/V [B, Hkv, S, D] bf16 contiguous (self-attention over each sequence);
    out [B, Hq, S, D] (Q's dtype by default). gkv_flash_attention."""
    if Q.dim() != 4 or K.dim() != 4 or V.dim() != 4:
        raise GkvError(_lib.GKV_ERR_INVALID, "Q, K, V must be [B, H, S, D]")
    B, Hq, S, D = Q.shape
    if out is None:
        out = torch.empty_like(Q)
    sc = float(scale) if scale is not None else 1.0 / float(D) ** 0.5
    for t in (Q, K, V, out):
        if not t.is_contiguous() or t.device != Q.device:
            raise GkvError(_lib.GKV_ERR_INVALID, "tensors must be contiguous and on one device")
    check(lib().gkv_flash_attention(C.c_void_p(Q.data_ptr()), C.c_void_p(K.data_ptr()), C.c_void_p(V.data_ptr()),
                                    C.c_void_p(out.data_ptr()), B, Hq, K.shape[1], S, D, sc, 1 if causal else 0,
                                    _TORCH_TO_GKV[Q.dtype], _TORCH_TO_GKV[out.dtype],
                                    _stream_handle(Q.device, stream)))
    return out


def flash_check_errors() -> int:
    """The current device's flash-attention error word (read and cleared)."""
    v = C.c_uint32(0)
    st = lib().gkv_flash_check_errors(C.byref(v))
    if st not in (0, _lib.GKV_ERR_DEVICE):
        check(st)
    return v.value

