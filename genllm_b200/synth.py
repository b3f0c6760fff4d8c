"""Seeded synthetic workloads for the paged KV-cache path.

The reference ships no dataset or benchmark inputs for this path; every
config is synthetic (bf16 N(0,1) values, seeded fragmented block tables).
Both the parity tests and bench.py build their inputs here so that the CUDA
path and the CPU checkers see identical bytes.

A *fragmented case* reproduces a cache that has been filled and partly
recycled: every physical page of a ``pool_pages`` pool is handed out, the
ones not in the table are returned to the free list, and the table is a
seeded permutation. The K and V pools use independent permutations (the
reference keeps separate K and V id streams, PageEntry{k_block_id,
v_block_id}, include/core/page_attention.h:47-50).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

PAGE_SLOTS = 16  # PAGE_BLOCK_SIZE, include/core/page_attention.h:9


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even, exponent-0 inputs flushed to
    signed zero (the reference's conversion, include/utils/bfloat16.hpp:18-41)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    sign = u >> 31
    e = (u >> 23) & 0xFF
    m = u & 0x7FFFFF
    low = u & 0xFFFF
    up = ((low > 0x8000) | ((low == 0x8000) & ((m & 0x10000) != 0))).astype(np.uint32)
    hm = (m >> 16) + up
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


def randn_bf16(rng: np.random.Generator, shape) -> np.ndarray:
    return bf16_bits(rng.standard_normal(shape, dtype=np.float32))


@dataclass
class FragmentedCase:
    n_q_heads: int
    n_kv_heads: int
    head_dim: int
    n_prior: int           # tokens already in the cache
    n_new: int             # tokens appended by the step (1 = decode)
    pool_pages: int
    k_ids: np.ndarray      # int32 [ceil(n_prior/16)] physical K page per logical page
    v_ids: np.ndarray
    k_free_order: np.ndarray  # ids returned to the K free list, in order
    v_free_order: np.ndarray
    k_pool: np.ndarray     # uint16 [pool_pages][16][Hkv][D]
    v_pool: np.ndarray
    q: np.ndarray          # uint16 [Hq][S][D]
    k_new: np.ndarray      # uint16 [Hkv][S][D]
    v_new: np.ndarray
    scale: float

    @property
    def n_pages(self) -> int:
        return len(self.k_ids)

    @property
    def total(self) -> int:
        return self.n_prior + self.n_new


def fragmented_case(seed: int, n_q_heads: int, n_kv_heads: int, head_dim: int, n_prior: int,
                    pool_pages: int, n_new: int = 1, fill_pools: bool = True,
                    poison_unused: bool = False, page_order: str = "random") -> FragmentedCase:
    """Build the inputs of one paged-attention step.

    Config 1 of the path (Qwen3-0.6B layer): ``fragmented_case(0, 16, 8, 128,
    1024, 256)``. With ``poison_unused`` the slots no table entry covers hold
    NaN bit patterns, so a kernel that reads past the valid tokens shows up.

    ``page_order`` sets the physical ids behind the logical pages: "random"
    (a shuffled pool), "asc" (0, 1, 2, ...), "desc" (the highest ids first,
    as the LIFO free list hands them out after a reset; the step's new pages
    then come back ascending), "broken" (descending with some runs of 8
    interrupted: two ids swapped in one run, V alone swapped in another) and
    "kv_mismatch" (K descending, V ascending).
    """
    rng = np.random.default_rng(seed)
    n_pages = (n_prior + PAGE_SLOTS - 1) // PAGE_SLOTS
    if n_pages > pool_pages:
        raise ValueError("pool too small for the prior tokens")
    kp = rng.permutation(pool_pages).astype(np.int32)
    vp = rng.permutation(pool_pages).astype(np.int32)
    if page_order != "random":
        up = np.arange(pool_pages, dtype=np.int32)
        if page_order == "asc":
            kp, vp = up.copy(), up.copy()
        elif page_order in ("desc", "broken"):
            kp, vp = up[::-1].copy(), up[::-1].copy()
            if page_order == "broken":
                if pool_pages > 12:
                    kp[[11, 12]] = kp[[12, 11]]
                    vp[[11, 12]] = vp[[12, 11]]
                if pool_pages > 20:
                    vp[[19, 20]] = vp[[20, 19]]
        elif page_order == "kv_mismatch":
            kp, vp = up[::-1].copy(), up.copy()
        else:
            raise ValueError(f"unknown page_order {page_order!r}")
    shape = (pool_pages, PAGE_SLOTS, n_kv_heads, head_dim)
    if fill_pools:
        k_pool = randn_bf16(rng, shape)
        v_pool = randn_bf16(rng, shape)
        if poison_unused:
            nan = np.uint16(0x7FC1)
            used_k = np.zeros(pool_pages, bool); used_k[kp[:n_pages]] = True
            used_v = np.zeros(pool_pages, bool); used_v[vp[:n_pages]] = True
            k_pool[~used_k] = nan
            v_pool[~used_v] = nan
            tail = n_prior - (n_pages - 1) * PAGE_SLOTS if n_pages else PAGE_SLOTS
            if n_pages and tail < PAGE_SLOTS:
                k_pool[kp[n_pages - 1], tail:] = nan
                v_pool[vp[n_pages - 1], tail:] = nan
    else:
        k_pool = np.zeros(0, np.uint16)
        v_pool = np.zeros(0, np.uint16)
    q = randn_bf16(rng, (n_q_heads, n_new, head_dim))
    k_new = randn_bf16(rng, (n_kv_heads, n_new, head_dim))
    v_new = randn_bf16(rng, (n_kv_heads, n_new, head_dim))
    return FragmentedCase(n_q_heads, n_kv_heads, head_dim, n_prior, n_new, pool_pages,
                          kp[:n_pages].copy(), vp[:n_pages].copy(), kp[n_pages:].copy(),
                          vp[n_pages:].copy(), k_pool, v_pool, q, k_new, v_new,
                          float(1.0 / np.sqrt(head_dim)))


@dataclass
class QkRopeCase:
    """Inputs of the QK-norm + RoPE step that feeds the attention op, as the
    reference's Qwen3 block produces them (src/model/Qwen3.cpp:130-154):
    q_flat [S][Hq*D] and k_flat / v_flat [S][Hkv*D] bf16 (the projections'
    outputs), per-head RMSNorm weights [D] fp32, eps, RoPE theta and the
    position of the first token."""
    q_flat: np.ndarray
    k_flat: np.ndarray
    v_flat: np.ndarray
    q_norm_w: np.ndarray
    k_norm_w: np.ndarray
    eps: float
    theta: float
    start_pos: int
    n_q_heads: int
    n_kv_heads: int
    head_dim: int

    @property
    def seq_len(self) -> int:
        return self.q_flat.shape[0]


def qk_rope_case(seed: int, n_q_heads: int, n_kv_heads: int, seq_len: int, start_pos: int,
                 head_dim: int = 128, eps: float = 1e-6, theta: float = 1e6) -> QkRopeCase:
    rng = np.random.default_rng(seed)
    q = randn_bf16(rng, (seq_len, n_q_heads * head_dim))
    k = randn_bf16(rng, (seq_len, n_kv_heads * head_dim))
    v = randn_bf16(rng, (seq_len, n_kv_heads * head_dim))
    wq = (1.0 + 0.25 * rng.standard_normal(head_dim)).astype(np.float32)
    wk = (1.0 + 0.25 * rng.standard_normal(head_dim)).astype(np.float32)
    return QkRopeCase(q, k, v, wq, wk, eps, theta, start_pos, n_q_heads, n_kv_heads, head_dim)


def heads_major(flat: np.ndarray, n_heads: int) -> np.ndarray:
    """[S][H*D] -> [H][S][D]: the reference's reshape_permute {0, 2, 1, 3}."""
    S = flat.shape[0]
    return np.ascontiguousarray(flat.reshape(S, n_heads, -1).transpose(1, 0, 2))



def kv_format_values(seed: int, n_kv_heads: int, n_tokens: int, head_dim: int = 128,
                     special: bool = True) -> tuple[np.ndarray, np.ndarray]:
    """K and V [Hkv][n_tokens][D] bf16 bits for the format export / import
    cases: N(0, 1) values with a different magnitude per 16-token block
    (2^-20 .. 2^20), and with ``special`` the edge cases of the fp8 block
    scale: an all-zero block, +-inf and NaN among finite values, a block of
    bf16 subnormals and one of the largest finite bf16 values."""
    rng = np.random.default_rng(seed)
    n_blocks = (n_tokens + 15) // 16
    out = []
    for _ in range(2):
        x = rng.standard_normal((n_kv_heads, n_tokens, head_dim), dtype=np.float32)
        mag = np.exp2(rng.integers(-20, 21, size=(n_kv_heads, n_blocks))).astype(np.float32)
        x *= np.repeat(mag, 16, axis=1)[:, :n_tokens, None]
        b = bf16_bits(x)
        if special and n_tokens >= 16:
            h = n_kv_heads - 1
            blk = lambda i: slice(16 * (i % n_blocks), min(n_tokens, 16 * (i % n_blocks) + 16))
            b[0, blk(1)] = 0                                  # all-zero block
            b[h, blk(2)][0, :3] = [0x7F80, 0xFF80, 0x7FC0]    # +inf, -inf, NaN
            b[0, blk(3)] = (rng.integers(1, 0x80, b[0, blk(3)].shape) |
                            (rng.integers(0, 2, b[0, blk(3)].shape) << 15)).astype(np.uint16)  # subnormals
            b[h, blk(4)][:, ::7] = 0x7F7F                     # largest finite bf16
        out.append(b)
    return out[0], out[1]
