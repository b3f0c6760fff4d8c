"""Multi-GPU KV-head sharding with the all-gather fused into the decode step.

Each rank (one process per GPU) owns Hkv/N kv heads; ``HeadGather`` sets up a
full-output region per rank that every rank can write over NVLink (CUDA IPC,
handles exchanged through torch.distributed), and ``decode`` runs one layer's
decode step whose split-combine kernel stores the rank's head block into all
ranks' regions and waits (bounded) for the peers' blocks — no separate
collective launch. The region is returned as a torch view for the caller.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _lib
from ._lib import check, lib

_HANDLE = 64


class _CudaArray:
    """Minimal __cuda_array_interface__ so torch can view library memory."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": shape, "typestr": typestr, "version": 3,
                                         "strides": None}


class HeadGather:
    def __init__(self, device: int, n_layers: int, n_q_heads: int, head_dim: int = 128, group=None,
                 dtype=torch.bfloat16):
        self.device, self.group = device, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n_layers, self.n_q_heads, self.head_dim = n_layers, n_q_heads, head_dim
        self.dtype = dtype
        self.esize = torch.tensor([], dtype=dtype).element_size()
        self.layer_bytes = n_q_heads * head_dim * self.esize
        L = lib()
        out, flags = C.c_void_p(), C.c_void_p()
        check(L.gkv_device_alloc(device, self.layer_bytes * n_layers, C.byref(out)))
        check(L.gkv_device_alloc(device, 4 * n_layers * self.world, C.byref(flags)))
        self._own = (out, flags)
        h = (C.c_char * (2 * _HANDLE))()
        check(L.gkv_ipc_export(device, out, h))
        check(L.gkv_ipc_export(device, flags, C.byref(h, _HANDLE)))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(h), group=group)
        bases = (C.c_void_p * self.world)()
        fl = (C.c_void_p * self.world)()
        self._opened = []
        for r in range(self.world):
            if r == self.rank:
                bases[r], fl[r] = out, flags
                continue
            b, f = C.c_void_p(), C.c_void_p()
            check(L.gkv_ipc_open(device, handles[r][:_HANDLE], C.byref(b)))
            check(L.gkv_ipc_open(device, handles[r][_HANDLE:], C.byref(f)))
            self._opened += [b, f]
            bases[r], fl[r] = b, f
        g = C.c_void_p()
        check(L.gkv_gather_create(device, self.world, self.rank, n_layers, bases, fl, C.byref(g)))
        self.handle = g
        raw = torch.as_tensor(_CudaArray(out.value, (n_layers * n_q_heads * head_dim * self.esize // 2,), "<i2"),
                              device=f"cuda:{device}")
        # This rank's gathered outputs (memory valid until close()). full[l]
        # holds layer l's latest step only until layer l's next gather call on
        # any rank: a peer's next call stores over it as soon as that peer
        # gets there, so read it (stream-ordered) before this rank's next call
        # for the same layer (gkv_paged_attention_gather in genllm_kv.h).
        self.full = raw.view(dtype).view(n_layers, n_q_heads, head_dim)
        dist.barrier(group=group)

    def decode(self, manager, layer_id: int, Q, K, V, scale: float, stream=None) -> torch.Tensor:
        """Decode step of this rank's heads; returns the full [Hq, D] output of the layer (a view that
        the layer's next call on any rank overwrites)."""
        hq_local = Q.shape[1]
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        code = {torch.bfloat16: _lib.GKV_BF16, torch.float16: _lib.GKV_F16, torch.float32: _lib.GKV_F32}[self.dtype]
        check(lib().gkv_paged_attention_gather(manager.handle, layer_id, C.c_void_p(Q.data_ptr()),
                                               C.c_void_p(K.data_ptr()), C.c_void_p(V.data_ptr()), self.handle,
                                               layer_id * self.layer_bytes, hq_local, C.c_float(scale), code,
                                               C.c_void_p(s.cuda_stream)))
        return self.full[layer_id]

    def close(self):
        if getattr(self, "handle", None):
            torch.cuda.synchronize(self.device)
            L = lib()
            L.gkv_gather_destroy(self.handle)
            for p in self._opened:
                L.gkv_ipc_close(self.device, p)
            L.gkv_device_free(self.device, self._own[0])
            L.gkv_device_free(self.device, self._own[1])
            self.handle = None
