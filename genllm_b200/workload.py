"""Device-resident decode workload of the paged KV-cache path (bench config 3/5).

Builds ``n_layers`` layers of Qwen3-4B attention shape (Hq=32, Hkv=8, D=128,
bf16) on one GPU, each holding ``ctx`` cached tokens in a fragmented block
table: all pages of a ``pool_pages`` pool handed out, the unused ones freed
(seeded order), the table a seeded permutation. Values are N(0,1) bf16 drawn
on the device (seeded). With ``world``/``rank`` the KV heads are sharded: the
rank owns kv heads [rank*Hkv/world, (rank+1)*Hkv/world) and the matching
query heads, while the page ids (and so the block table) are identical on
every rank.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .paged_attention import PagedAttentionManager

PAGE = 16


def shard_heads(n_q_heads: int, n_kv_heads: int, world: int, rank: int):
    """(q_head_begin, q_head_end, kv_head_begin, kv_head_end) of one rank."""
    if n_kv_heads % world:
        raise ValueError(f"{n_kv_heads} kv heads do not split over {world} ranks")
    g = n_q_heads // n_kv_heads
    hk = n_kv_heads // world
    return rank * hk * g, (rank + 1) * hk * g, rank * hk, (rank + 1) * hk


@dataclass
class LayerBufs:
    q: torch.Tensor      # [1, Hq_local, 1, D] bf16
    k: torch.Tensor      # [1, Hkv_local, 1, D]
    v: torch.Tensor
    out: torch.Tensor    # [1, Hq_local, 1, D] bf16


class DecodeWorkload:
    def __init__(self, device: int, n_layers=36, ctx=32768, pool_pages=4096, n_q_heads=32, n_kv_heads=8,
                 head_dim=128, seed=0, world=1, rank=0):
        self.device = torch.device("cuda", device)
        self.seed = seed
        self.n_layers, self.ctx, self.pool_pages = n_layers, ctx, pool_pages
        self.Hq, self.Hkv, self.D = n_q_heads, n_kv_heads, head_dim
        qb, qe, kb, ke = shard_heads(n_q_heads, n_kv_heads, world, rank)
        self.hq_local, self.hkv_local = qe - qb, ke - kb
        self.scale = 1.0 / float(head_dim) ** 0.5
        self.mgr = PagedAttentionManager(device)
        self.layers = []
        # All layers' step inputs (Q | K | V) in one buffer and all outputs in
        # another, so a host round trip is one copy each way.
        hq_l, hkv_l = qe - qb, ke - kb
        self.in_width = (hq_l + 2 * hkv_l) * head_dim
        self.inbuf = torch.empty((n_layers, self.in_width), dtype=torch.bfloat16, device=self.device)
        self.outbuf = torch.empty((n_layers, hq_l * head_dim), dtype=torch.bfloat16, device=self.device)
        n_pages = (ctx + PAGE - 1) // PAGE
        for l in range(n_layers):
            rng = np.random.default_rng(seed * 1000 + l)
            kperm = rng.permutation(pool_pages).astype(np.int32)
            vperm = rng.permutation(pool_pages).astype(np.int32)
            self.mgr.init_layer(l, self.hkv_local, head_dim)
            self.mgr.reserve_layer(l, pool_pages)
            kp, vp = self.mgr.pool_tensors(l)
            g = torch.Generator(device=self.device)
            # Full-head values drawn per layer, then this rank's heads kept, so
            # that every sharding sees the same cache contents.
            for t, off in ((kp, 1), (vp, 2)):
                g.manual_seed(seed * 1000003 + l * 7 + off)
                for p0 in range(0, pool_pages, 512):
                    p1 = min(pool_pages, p0 + 512)
                    full = torch.randn((p1 - p0, PAGE, n_kv_heads, head_dim), generator=g, device=self.device)
                    t[p0:p1].copy_(full[:, :, kb:ke].to(torch.bfloat16))
            for w, perm in ((0, kperm), (1, vperm)):
                lib = _lib.lib()
                out = C.c_int32()
                for _ in range(pool_pages):
                    _lib.check(lib.gkv_page_alloc(self.mgr.handle, l, w, C.byref(out)))
                for pid in perm[n_pages:]:
                    _lib.check(lib.gkv_page_free(self.mgr.handle, l, w, int(pid)))
            self.mgr.set_page_table(l, kperm[:n_pages], vperm[:n_pages], ctx)
            g.manual_seed(seed * 1000003 + l * 7 + 3)
            q = torch.randn((1, n_q_heads, 1, head_dim), generator=g, device=self.device)[:, qb:qe].to(torch.bfloat16)
            k = torch.randn((1, n_kv_heads, 1, head_dim), generator=g, device=self.device)[:, kb:ke].to(torch.bfloat16)
            v = torch.randn((1, n_kv_heads, 1, head_dim), generator=g, device=self.device)[:, kb:ke].to(torch.bfloat16)
            row = self.inbuf[l]
            qv = row[: hq_l * head_dim].view(1, hq_l, 1, head_dim)
            kv = row[hq_l * head_dim: (hq_l + hkv_l) * head_dim].view(1, hkv_l, 1, head_dim)
            vv = row[(hq_l + hkv_l) * head_dim:].view(1, hkv_l, 1, head_dim)
            qv.copy_(q)
            kv.copy_(k)
            vv.copy_(v)
            out_t = self.outbuf[l].view(1, hq_l, 1, head_dim)
            self.layers.append(LayerBufs(qv, kv, vv, out_t))
        torch.cuda.synchronize(self.device)
        self._fn = _lib.lib().gkv_paged_attention
        self._args = [
            (self.mgr.handle, l, C.c_void_p(b.q.data_ptr()), C.c_void_p(b.k.data_ptr()), C.c_void_p(b.v.data_ptr()),
             C.c_void_p(b.out.data_ptr()), 1, self.hq_local, 1, head_dim, self.hkv_local, C.c_float(self.scale), 1,
             self.hq_local // self.hkv_local, _lib.GKV_BF16, _lib.GKV_BF16)
            for l, b in enumerate(self.layers)]

    def cached(self, layer: int = 0) -> int:
        return self.mgr.get_layer(layer).num_cached

    def layer_step(self, l: int, stream_handle) -> None:
        """One decode step of layer l through the C ABI (append + attention)."""
        st = self._fn(*self._args[l], stream_handle)
        if st:
            _lib.check(st)

    def reference_output(self, layer: int) -> torch.Tensor:
        """Self-check of a bench run: the layer's attention output over every
        cached token, all heads (not only this rank's), in plain torch fp32 on
        the device, from the workload's seeded values regenerated in full:
        the pool pages for the first ``ctx`` tokens, the step's K/V row (the
        same every step) for the tokens appended since. Returns [Hq, D]."""
        hkv, d, seed = self.Hkv, self.D, self.seed
        g = torch.Generator(device=self.device)
        pools = []
        for off in (1, 2):
            g.manual_seed(seed * 1000003 + layer * 7 + off)
            chunks = [torch.randn((min(self.pool_pages, p0 + 512) - p0, PAGE, hkv, d), generator=g,
                                  device=self.device).to(torch.bfloat16)
                      for p0 in range(0, self.pool_pages, 512)]
            pools.append(torch.cat(chunks))
        g.manual_seed(seed * 1000003 + layer * 7 + 3)
        q = torch.randn((self.Hq, d), generator=g, device=self.device).to(torch.bfloat16).float()
        k_new = torch.randn((hkv, d), generator=g, device=self.device).to(torch.bfloat16).float()
        v_new = torch.randn((hkv, d), generator=g, device=self.device).to(torch.bfloat16).float()
        total = self.cached(layer)
        table = self.mgr.get_layer(layer).page_table
        ids = torch.tensor([[e.k_block_id, e.v_block_id] for e in table], dtype=torch.long, device=self.device)
        pos = torch.arange(total, device=self.device)
        rows = []
        for w, new in ((0, k_new), (1, v_new)):
            r = pools[w][ids[pos // PAGE, w], pos % PAGE].float()  # [total, Hkv, D]
            r[self.ctx:] = new
            rows.append(r)
        kk, vv = rows
        grp = self.Hq // hkv
        qh = q.view(hkv, grp, d)
        s = torch.einsum("hgd,thd->hgt", qh, kk) * self.scale
        p = torch.softmax(s, dim=-1)
        return torch.einsum("hgt,thd->hgd", p, vv).reshape(self.Hq, d)

    def bytes_per_layer_token(self, total_tokens: int) -> int:
        """Algorithmic HBM bytes of one fused decode launch attending
        total_tokens tokens (the new one included): every K and V row read
        once, Q read, the bf16 output written, the new K/V row read from the
        input and written to its page, the block table read."""
        row = self.hkv_local * self.D * 2
        n_pages = (total_tokens + PAGE - 1) // PAGE
        kv_read = 2 * (total_tokens - 1) * row
        new_kv = 2 * 2 * row
        q = self.hq_local * self.D * 2
        out = self.hq_local * self.D * 2
        table = n_pages * 8
        return kv_read + new_kv + q + out + table


def allgather_heads(local_out, full_out, group=None):
    """All-gather each rank's query-head block of a layer output into
    full_out ([.., Hq, .., D] with the rank-major head order of shard_heads).
    NCCL: one all_gather_into_tensor; other backends (gloo, for CPU tests):
    all_gather into a list."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    flat = full_out.view(world, -1)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(flat, local_out.contiguous().view(-1), group=group)
    else:
        parts = [torch.empty_like(flat[0]) for _ in range(world)]
        dist.all_gather(parts, local_out.contiguous().view(-1), group=group)
        for r in range(world):
            flat[r].copy_(parts[r])
    return full_out
