// prefill_tc.cu — chunked-prefill paged attention on the 5th-generation
// tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// The reference has no tensor-core path: its CUDA op runs a warp per (head,
// query) over a serial page loop (src/backend/cuda/attention.cu:401-489),
// and the CPU op folds one token at a time into an online softmax
// (src/backend/cpu/attention.cpp:156-215). Here a chunk of S queries of one
// query head attends causally over every cached page:
//
//   * CTA = 128 queries x 1 query head (grid ceil(S/128) x Hq [x KV split]),
//     11 warps: two softmax groups of 4 warps, a K-load warp, a V-load warp
//     and an MMA warp;
//   * Q tile [128 x 128] and each KV tile (128 keys = 8 pages of 16 slots)
//     arrive by TMA in the 128-byte-swizzled K-major layout (one box per
//     page and 64-dim half, or one box per 8-page run of consecutive ids);
//     K and V tiles sit in 3-stage rings;
//   * the KV tiles alternate between the two softmax groups; group g owns
//     S/P buffer g (TMEM columns [128 g, +128)) and O accumulator g
//     ([256 + 128 g, +128)), one thread per query row;
//   * S = Q K^T: 8 tcgen05.mma (M128 N128 K16, bf16 -> fp32), both operands
//     in shared memory, issued by one thread, completion by tcgen05.commit;
//   * each group thread loads its S row from TMEM, applies the causal /
//     length mask, updates an fp32 online softmax (log2 domain, lazy
//     rescaling) and stores P over S in TMEM as bf16 hi + lo terms, so that
//     O_g += P V (16 tcgen05.mma, V an MN-major operand) keeps fp32-level
//     accuracy; while one group computes, the tensor cores run the other's
//     MMAs;
//   * the groups' (m, l, O) are merged, then the CTAs of a KV-split cluster
//     reduce-scatter their partials through distributed shared memory, and
//     each stores its share of the rows (fp32/bf16/fp16).
//
// Keys past the cached length in the last tile are masked in S, and their V
// rows are zeroed in shared memory (0 x NaN from stale slots would poison
// the MMA). Every mbarrier wait is bounded (kErrTimeout).
#include <climits>

#include "device.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace gkv {
namespace {

constexpr int kBM = 128;  // queries per CTA
constexpr int kBN = 128;  // keys per KV tile (8 pages)
constexpr int kPagesPerTile = kBN / kPageSlots;
constexpr uint32_t kHalf = 128 * 128;          // one 64-dim half of a 128-row tile: 16 KiB
constexpr uint32_t kTile = 2 * kHalf;          // 32 KiB
constexpr uint32_t kOffQ = 0;
constexpr int kStages = 3;                     // K and V tiles in flight
constexpr uint32_t kOffK = kOffQ + kTile;
constexpr uint32_t kOffV = kOffK + kStages * kTile;
constexpr uint32_t kOffBar = kOffV + kStages * kTile;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;  // + barriers, TMEM slot, alignment slack
static_assert((9 + 4 * kStages) * 8 + 4 <= 256, "barriers and the TMEM slot fit their 256 bytes");
// (m, l) rows of the two softmax groups at the end: the last 4 KiB of the
// last V stage.
constexpr uint32_t kOffEx = kOffV + kStages * kTile - 4096;
// Cluster reduce-scatter: a CTA's partials (O rows [128][128] fp32 at 0,
// then (m, l, -, -) per row at kRecvO), one receive slot per other CTA of the
// cluster (up to 2; each at most 64 rows of O then their (m, l, -, -)), and
// the staged output rows (at most 128 x 512 bytes).
constexpr uint32_t kRecvO = 128 * kHeadDim * 4;
constexpr uint32_t kRowBytes = kHeadDim * 4 + 16;  // bytes received per row and sender
constexpr uint32_t kRecvSlotO = 64 * kHeadDim * 4;
constexpr uint32_t kRecvSlot = kRecvSlotO + 64 * 16;
constexpr uint32_t kOffRecv = kRecvO + 128 * 16;
constexpr uint32_t kOffStage = (kOffRecv + 2 * kRecvSlot + 1023) / 1024 * 1024;
static_assert(kOffStage + 128 * kHeadDim * 4 <= kOffEx, "staged output rows clear of the (m, l) exchange");
static_assert(kRecvSlot % 16 == 0 && kOffRecv % 16 == 0, "bulk copy addresses are multiples of 16 bytes");
// TMEM columns: S/P of the two groups' tiles [0, 256) (buffer = tile & 1 =
// group), O of group 0 [256, 384), O of group 1 [384, 512).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;

struct TcParams {
    const int2* table;
    void* out;
    uint32_t* err;
    int32_t out_dtype;
    int32_t n_q_heads;
    int32_t n_kv_heads;
    int32_t seq_len;
    int32_t total;
    int32_t n_pages;
    int32_t pool_pages;
    int32_t causal;
    int32_t runs;    // k_run / v_run maps usable
    int32_t contig;  // 1: K/V are contiguous [B*Hkv][S][128] (k_run / v_run map them), no table
    // KV tiles with index >= new_tile0 hold only this chunk's tokens and are
    // copied from the chunk's K/V inputs ([Hkv][S][128], k_new / v_new) at
    // row (tile - new_tile0) * 128 instead of from the pages (INT_MAX: none).
    int32_t new_tile0;
    // 1: every input this launch reads was complete before the previous
    // kernel (the chunk's append) started, so the launch does not wait for
    // it before reading, only before it completes (the next chunk reads the
    // pages that append writes).
    int32_t wait_at_end;
    float qscale;    // softmax scale * log2(e)
};

constexpr int kConsumerThreads = 256;               // 8 warps: two groups of one thread per query row
constexpr int kLoadWarp = kConsumerThreads / 32;   // issues the K loads (warp + 1: the V loads)
constexpr int kMmaWarp = kLoadWarp + 2;            // issues the tcgen05 MMAs
constexpr int kThreadsTc = kConsumerThreads + 96;
constexpr float kRescaleLog2 = 8.f;  // lazy-rescale threshold (log2 units)

#ifdef GKV_PROBE_TIMELINE
// Measurement builds only: per-tile phase clocks of threads 0 and 128 (the
// two softmax groups), of the MMA warp and of the K-load warp, in one CTA.
__device__ long long g_probe_pf[2 * 128 * 16];
__device__ long long g_probe_mma[128 * 4];
__device__ long long g_probe_ld[128 * 8];
// Per CTA: entry, setup done, first S ready, exit, every MMA done, groups
// merged, partials merged, output stored, cluster barrier passed, partial
// copies issued, own rows' partials received, output rows staged, staging
// synchronised, reciprocal ready.
__device__ unsigned long long g_probe_ee[1024 * 16];
#define PROBE_EE(k)                                                                                          \
    if (tid == 0) {                                                                                          \
        const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;                      \
        if (cta < 1024) g_probe_ee[cta * 16 + (k)] = global_timer_ns();                                      \
    }
#define PROBE_LD(k)                                                                                  \
    if (blockIdx.x == gridDim.x - 1 && blockIdx.y == 0 && blockIdx.z == 1 && j < 128) g_probe_ld[j * 8 + (k)] = clock64();
#define PROBE_MMA(k)                                                                                 \
    if (blockIdx.x == gridDim.x - 1 && blockIdx.y == 0 && blockIdx.z == 1 && j < 128) g_probe_mma[j * 4 + (k)] = clock64();
#define PROBE_PF(k)                                                                                  \
    if ((tid & 127) == 0 && blockIdx.x == gridDim.x - 1 && blockIdx.y == 0 && blockIdx.z == 1 && j < 128) \
        g_probe_pf[((tid >> 7) * 128 + j) * 16 + (k)] = clock64();
#else
#define PROBE_PF(k)
#define PROBE_MMA(k)
#define PROBE_LD(k)
#define PROBE_EE(k)
#endif

// How a tile's 8 pages are copied: 0 = page by page; 1 = one run of
// ascending consecutive ids (K and V alike); 2 = one run of descending ids
// (what the LIFO free list hands out after a reset), whose copy lands the
// pages in reverse order. Lanes 0-7 of the calling warp hold entry `lane` of
// the tile; every lane gets the same answer. The load warps evaluate the same
// rule on their private copy of the entries (tile_mode_regs), so producers
// and consumers agree on the layout of every stage.
__device__ __forceinline__ int tile_mode_warp(int2 e, int lane, int pool_pages, int runs) {
    const int x0 = __shfl_sync(0xFFFFFFFFu, e.x, 0), y0 = __shfl_sync(0xFFFFFFFFu, e.y, 0);
    const bool in = lane < kPagesPerTile;
    const bool asc = __all_sync(0xFFFFFFFFu, !in || (e.x == x0 + lane && e.y == y0 + lane));
    const bool desc = __all_sync(0xFFFFFFFFu, !in || (e.x == x0 - lane && e.y == y0 - lane));
    if (!runs) return 0;
    if (asc && x0 >= 0 && y0 >= 0 && x0 + kPagesPerTile <= pool_pages && y0 + kPagesPerTile <= pool_pages) return 1;
    if (desc && x0 - (kPagesPerTile - 1) >= 0 && y0 - (kPagesPerTile - 1) >= 0 && x0 < pool_pages && y0 < pool_pages)
        return 2;
    return 0;
}
__device__ __forceinline__ int tile_mode_regs(const int2 (&e)[kPagesPerTile], int pool_pages, int runs) {
    const int x0 = e[0].x, y0 = e[0].y;
    bool asc = true, desc = true;
#pragma unroll
    for (int i = 1; i < kPagesPerTile; ++i) {
        asc = asc && e[i].x == x0 + i && e[i].y == y0 + i;
        desc = desc && e[i].x == x0 - i && e[i].y == y0 - i;
    }
    if (!runs) return 0;
    if (asc && x0 >= 0 && y0 >= 0 && x0 + kPagesPerTile <= pool_pages && y0 + kPagesPerTile <= pool_pages) return 1;
    if (desc && x0 - (kPagesPerTile - 1) >= 0 && y0 - (kPagesPerTile - 1) >= 0 && x0 < pool_pages && y0 < pool_pages)
        return 2;
    return 0;
}
// Key (within the tile) held by smem row / S column c of a tile copied in `mode`.
__device__ __forceinline__ int tile_key(int c, int mode) {
    return mode == 2 ? (((kPagesPerTile - 1 - (c >> 4)) << 4) | (c & 15)) : c;
}

// Output conversion of the epilogue: two fp32 values -> packed bf16 (lo in
// the low half) by the hardware's round-to-nearest-even. For normal values
// these are the reference's bits (include/utils/bfloat16.hpp:18-41 rounds to
// nearest even); it differs only where the reference flushes a zero-exponent
// input to a signed zero (a difference below 2^-126) and in the payload of a
// NaN. Anything longer costs here: the epilogue runs once per CTA from a
// cold instruction cache, and its time grew with the code size (a per-value
// special-case check took ~1 us more per tile).
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}
__device__ __noinline__ uint4 half8_rn(float4 x, float4 y) {
    auto h2 = [](float u, float v) {
        return (uint32_t)__half_as_ushort(__float2half_rn(u)) | ((uint32_t)__half_as_ushort(__float2half_rn(v)) << 16);
    };
    return make_uint4(h2(x.x, x.y), h2(x.z, x.w), h2(y.x, y.y), h2(y.z, y.w));
}

__global__ void __launch_bounds__(kThreadsTc, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                      const __grid_constant__ CUtensorMap v_map, const __grid_constant__ CUtensorMap k_run,
                      const __grid_constant__ CUtensorMap v_run, const __grid_constant__ CUtensorMap k_new,
                      const __grid_constant__ CUtensorMap v_new, const TcParams a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bar_q = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint64_t* bar_k = bar_q + 1;             // [kStages] K tile landed
    uint64_t* bar_v = bar_k + kStages;       // [kStages] V tile landed
    uint64_t* bar_kfree = bar_v + kStages;   // [kStages] Q K^T of the stage's tile done
    uint64_t* bar_vfree = bar_kfree + kStages;  // [kStages] P V of the stage's tile done
    uint64_t* bar_s = bar_vfree + kStages;   // [2] S of a tile in its TMEM buffer (buffer = tile & 1)
    uint64_t* bar_o = bar_s + 2;             // [2] P V into O of a group done
    uint64_t* bar_p = bar_o + 2;             // [2] a group's 4 warps: P of its tile written (S read)
    uint64_t* bar_fin = bar_p + 2;           // every MMA of the CTA done
    uint64_t* bar_recv = bar_fin + 1;        // KV split: the other CTAs' partials of this CTA's rows landed
    constexpr int kNumBars = 9 + 4 * kStages;  // q, k, v, kfree, vfree, s[2], o[2], p[2], fin, recv
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_q + kNumBars);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    // Longest work first: CTAs start in the order of their linear index (x
    // fastest), which is mapped to (query tile, head) with the heads
    // innermost and the query tiles descending, so that under a causal mask
    // the CTAs with the most KV tiles start first and the last wave holds
    // the shortest ones.
    const int lin = blockIdx.y * gridDim.x + blockIdx.x;
    const int hq = lin % gridDim.y;
    const int q0 = (gridDim.x - 1 - lin / gridDim.y) * kBM;
    const int G = a.n_q_heads / a.n_kv_heads;
    // Paged: blockIdx.y is the query head. Contiguous (non-paged attention
    // over B sequences): blockIdx.y = b * Hq + head, and the K/V rows of
    // (b, kv head) sit at index b * Hkv + head / G of the tensor map.
    const int h = a.contig ? (hq / a.n_q_heads) * a.n_kv_heads + (hq % a.n_q_heads) / G : hq / G;
    const int S = a.seq_len;
    const int first_q_abs = a.total - S + q0;
    const int last_q_abs = min(a.total - 1, first_q_abs + kBM - 1);
    const int kv_end = a.causal ? last_q_abs + 1 : a.total;
    const int n_tiles_all = (kv_end + kBN - 1) / kBN;
    // KV split across the CTAs of a cluster (grid z = cluster size): this CTA
    // takes tiles [j0, j0 + n_tiles); the CTAs then reduce-scatter their
    // partials, each finalising a share of the rows.
    const int rank = blockIdx.z, n_split = gridDim.z;
    const int j0 = rank * n_tiles_all / n_split;
    const int n_tiles = (rank + 1) * n_tiles_all / n_split - j0;

    PROBE_EE(0);
    // Page ids of tile j: 8 independent table loads (one latency, not 8),
    // fetched by the issuing thread a tile before they are needed.
    auto load_ids = [&](int j, int2 (&e)[kPagesPerTile]) {
#pragma unroll
        for (int i = 0; i < kPagesPerTile; ++i) {
            int lp = (j0 + j) * kPagesPerTile + i;
            if (lp >= a.n_pages) lp = a.n_pages - 1;  // beyond the cache: rows are masked / zeroed
            // The chunk's own tiles come from its inputs; their entries may
            // still be in the append's hands.
            e[i] = j0 + j >= a.new_tile0 ? make_int2(0, 0) : a.table[lp];
        }
    };
    // The load warps fetch the first tile's page ids before the setup below
    // when nothing the previous kernel writes is read (wait_at_end): the
    // table load's latency then overlaps TMEM allocation and barrier setup.
    int2 ids_pre[kPagesPerTile];
    const bool pre = (warp == kLoadWarp || warp == kLoadWarp + 1) && (tid & 31) == 0 && n_tiles > 0 && !a.contig &&
                     a.wait_at_end;
    if (pre) load_ids(0, ids_pre);
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        for (int b = 0; b < kNumBars; ++b) mbar_init(bar_q + b, 1);
        mbar_init(&bar_p[0], 4);
        mbar_init(&bar_p[1], 4);
        fence_mbar_init();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // Launched as a programmatic dependent: the setup above overlapped the
    // previous kernel (the chunk's append). Unless the launch takes the
    // chunk's own tiles from its inputs (wait_at_end), nothing that kernel
    // writes (pages, table) or that came before it (Q) is read until it has
    // completed.
    if (!a.wait_at_end) asm volatile("griddepcontrol.wait;" ::: "memory");
    // Once this thread's tiles are done: let the next launch start (a kernel
    // that does not wait for this one is never launched as its programmatic
    // dependent). Reading the chunk's own tiles from its inputs, wait first
    // for the previous kernel (the chunk's append): the output stores, which
    // follow, must not overtake the previous chunk's, and the grid must not
    // complete before that append has (the next chunk reads its pages).
    // Every thread waiting before it triggers also makes "all of this grid
    // triggered" imply "the append before it completed", which is what lets
    // the next chunk's prefill start during this one's tail.
    auto launch_next = [&] {
        if (a.wait_at_end) asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    };
    PROBE_EE(1);
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;  // this warp's TMEM lanes

    const uint32_t sQ = smem_addr(smem + kOffQ);
    const uint32_t sK = smem_addr(smem + kOffK);
    const uint32_t sV = smem_addr(smem + kOffV);
    // Q is read once; K and V tiles are read again by the CTAs of the other
    // query tiles and heads of the group, so they keep normal L2 priority.
    const uint64_t pol = l2_policy_evict_first();
    uint64_t pol_kv;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol_kv));

    // Stage tile j's K (which = 0) or V (which = 1) into stage j % kStages.
    // Eight pages with consecutive ids are one run: two copies (one per
    // 64-dim half) with box {64, 1, 128} instead of 8 pages x 2 halves of box
    // {64, 1, 16}. A TMA copy costs its issuing thread about the same whatever
    // its size, so runs cut the load warps' issue time per tile by 8x. A
    // descending run lands its pages in reverse order (tile_key).
    auto issue = [&](int j, int which, const int2 (&ids)[kPagesPerTile]) {
        const int st = j % kStages;
        uint64_t* bar = which ? &bar_v[st] : &bar_k[st];
        mbar_arrive_expect_tx(bar, kTile);
        if (a.contig) {  // 128 consecutive key rows (past S: zero-filled by the copy)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf)
                tma_load_3d(smem + (which ? kOffV : kOffK) + st * kTile + hf * kHalf, which ? &v_run : &k_run, bar,
                            hf * 64, (j0 + j) * kBN, h, pol_kv);
            return;
        }
        if (j0 + j >= a.new_tile0) {  // the chunk's own keys, from its inputs (past S: zero-filled)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf)
                tma_load_3d(smem + (which ? kOffV : kOffK) + st * kTile + hf * kHalf, which ? &v_new : &k_new, bar,
                            hf * 64, (j0 + j - a.new_tile0) * kBN, h, pol_kv);
            return;
        }
        const int mode = tile_mode_regs(ids, a.pool_pages, a.runs);
        if (mode != 0) {
            const int first = which ? ids[0].y : ids[0].x;
            const int low = mode == 1 ? first : first - (kPagesPerTile - 1);
#pragma unroll
            for (int hf = 0; hf < 2; ++hf)
                tma_load_3d(smem + (which ? kOffV : kOffK) + st * kTile + hf * kHalf, which ? &v_run : &k_run, bar,
                            hf * 64, h, low * kPageSlots, pol_kv);
            return;
        }
#pragma unroll
        for (int i = 0; i < kPagesPerTile; ++i) {
            int2 e = ids[i];
            if (e.x < 0 || e.x >= a.pool_pages || e.y < 0 || e.y >= a.pool_pages) {
                atomicOr(a.err, kErrBadPage);
                e = make_int2(0, 0);
            }
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                if (which == 0)
                    tma_load_3d(smem + kOffK + st * kTile + hf * kHalf + i * 2048, &k_map, bar, hf * 64, h,
                                e.x * kPageSlots, pol_kv);
                else
                    tma_load_3d(smem + kOffV + st * kTile + hf * kHalf + i * 2048, &v_map, bar, hf * 64, h,
                                e.y * kPageSlots, pol_kv);
            }
        }
    };

    constexpr uint32_t kIdescQK = tc::idesc_bf16_f32(128, 128, false, false);
    constexpr uint32_t kIdescPV = tc::idesc_bf16_f32(128, 128, false, true);

    bool ok = true;
    // The consumer warps' own barrier (the load and MMA warps never join it).
    auto consumer_sync = [] { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory"); };
    // A wait that times out clears `ok`; later waits are then skipped, but
    // every thread still reaches every __syncthreads, so nothing can hang.
    auto wait = [&](uint64_t* bar, uint32_t parity) {
        if (ok && !mbar_wait_bounded(bar, parity)) ok = false;
    };
    // The MMA warp runs converged; one elected lane issues. Descriptors are
    // built once and stepped by adding the byte offset / 16 to their address
    // field (smem addresses stay below 256 KiB, so the 14-bit field cannot
    // carry). A tight issue sequence keeps the tensor pipe fed: each
    // m128n128k16 MMA takes 64 cycles, about what loose issue code spends
    // between two MMAs.
    const uint64_t desc_q0 = tc::smem_desc_sw128(sQ, 16, 1024);
    const uint64_t desc_k0 = tc::smem_desc_sw128(sK, 16, 1024);
    const uint64_t desc_v0 = tc::smem_desc_sw128(sV, kHalf, 1024);
    // S(j) = Q K(j)^T into TMEM columns [(j & 1) * 128, +128), both operands
    // from shared memory (K-major, 128-byte swizzle).
    auto issue_qk = [&](int j) {
        const int sb = j & 1, st = j % kStages;
        wait(&bar_k[st], (j / kStages) & 1);
        PROBE_MMA(3);
        tc::fence_after_sync();
        if (tc::elect_one()) {
            const uint64_t dk = desc_k0 + ((st * kTile) >> 4);
            const uint32_t d = tmem + sb * 128;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const uint32_t off = (((kk >> 2) * kHalf) + (kk & 3) * 32) >> 4;
                tc::mma_bf16(d, desc_q0 + off, dk + off, kIdescQK, kk > 0);
            }
            tc::commit(&bar_s[sb]);
            tc::commit(&bar_kfree[st]);
        }
        __syncwarp();
    };

    // P(j) V(j) into the O columns of group j & 1, both bf16 terms of P, with
    // P read from TMEM (where it replaced S(j)).
    auto issue_pv = [&](int j) {
        const int g = j & 1, st = j % kStages;
        wait(&bar_v[st], (j / kStages) & 1);
        tc::fence_after_sync();
        if (tc::elect_one()) {
            const uint64_t dv = desc_v0 + ((st * kTile) >> 4);
            const uint32_t p = tmem + g * 128;
            const uint32_t o = tmem + kColO + g * 128;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                tc::mma_bf16_ts(o, p + kk * 8, dv + ((kk * 2048) >> 4), kIdescPV, j >= 2 || kk > 0);
                tc::mma_bf16_ts(o, p + 64 + kk * 8, dv + ((kk * 2048) >> 4), kIdescPV, true);
            }
            tc::commit(&bar_o[g]);
            tc::commit(&bar_vfree[st]);
        }
        __syncwarp();
    };

    // Warp-specialised software pipeline with two softmax groups. The KV
    // tiles of the CTA alternate between group 0 (warps 0-3, even tiles) and
    // group 1 (warps 4-7, odd tiles); each group keeps its own running max,
    // sum and O accumulator for all 128 query rows (one thread per row), so
    // one group's softmax runs while the tensor cores compute the other
    // group's P V and next Q K^T. The groups' (m, l, O) are merged at the end.
    // One load warp issues K(j) once QK(j-3) has freed its stage, another V(j)
    // once PV(j-3) has; the MMA warp issues QK(0), QK(1), then per tile PV(j)
    // once group j & 1 has written P(j), followed by QK(j+2) into the TMEM
    // buffer P(j) occupied once PV(j) is done.
    if (warp == kMmaWarp) {
        if (n_tiles > 0) {
            wait(bar_q, 0);
            tc::fence_after_sync();
            issue_qk(0);
            if (n_tiles > 1) issue_qk(1);
            for (int j = 0; j < n_tiles && ok; ++j) {
                wait(&bar_p[j & 1], (j >> 1) & 1);
                PROBE_MMA(0);
                tc::fence_after_sync();
                if (!ok) break;
                issue_pv(j);
                if (j + 2 < n_tiles) {
                    wait(&bar_o[j & 1], (j >> 1) & 1);  // QK(j+2) overwrites P(j) in TMEM
                    PROBE_MMA(1);
                    tc::fence_after_sync();
                    issue_qk(j + 2);
                    PROBE_MMA(2);
                }
            }
            // Tracks every MMA this thread issued: both groups' O are final.
            if (tc::elect_one()) tc::commit(bar_fin);
            __syncwarp();
            if (!ok) atomicOr(a.err, kErrTimeout);
        }
        __syncwarp();
        launch_next();
        if (n_split > 1)  // the consumers' cluster barrier (every CTA's MMAs done)
            asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
        tc::fence_before_sync();
        __syncthreads();
        return;
    }
    if (warp == kLoadWarp || warp == kLoadWarp + 1) {
        const int lane = tid & 31;
        if (lane == 0) {
            const int which = warp - kLoadWarp;  // 0: K, 1: V
            if (which == 0) {
                mbar_arrive_expect_tx(bar_q, kTile);
                tma_load_3d(smem + kOffQ, &q_map, bar_q, 0, q0, hq, pol);
                tma_load_3d(smem + kOffQ + kHalf, &q_map, bar_q, 64, q0, hq, pol);
            }
            uint64_t* freed = which ? bar_vfree : bar_kfree;
            int2 ids[kPagesPerTile], nxt[kPagesPerTile];
            if (pre) {
#pragma unroll
                for (int i = 0; i < kPagesPerTile; ++i) ids[i] = ids_pre[i];
            } else if (n_tiles > 0 && !a.contig) {
                load_ids(0, ids);
            }
            for (int j = 0; j < n_tiles && ok; ++j) {
                if (j + 1 < n_tiles && !a.contig) load_ids(j + 1, nxt);
                if (which == 0) { PROBE_LD(0); }
                if (j >= kStages) wait(&freed[j % kStages], (j / kStages - 1) & 1);
                if (which == 0) { PROBE_LD(1); }
                if (!ok) break;
                issue(j, which, ids);
                if (which == 0) { PROBE_LD(2); }
#pragma unroll
                for (int i = 0; i < kPagesPerTile; ++i) ids[i] = nxt[i];
            }
            if (which == 0 && n_tiles == 0) wait(bar_q, 0);  // the Q load must land before the CTA exits
            if (!ok) atomicOr(a.err, kErrTimeout);
        }
        __syncwarp();
        launch_next();
        if (n_split > 1)  // the consumers' cluster barrier (every CTA's MMAs done)
            asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
        tc::fence_before_sync();
        __syncthreads();
        return;
    }

    const int r = tid & 127;  // query row of this thread
    const int g = tid >> 7;   // softmax group: KV tiles g, g + 2, ...
    const int q_abs = first_q_abs + r;
    const int lim = a.causal ? min(q_abs, a.total - 1) : a.total - 1;  // last visible key
    float m_run = -INFINITY, l_run = 0.f;
    // Lanes 0-7 of every consumer warp hold the page entries of the group's
    // next tile (fetched a tile ahead) to derive its copy mode.
    const int lane = tid & 31;
    auto entry = [&](int j) {
        // No table (contiguous K/V, or the chunk's own tiles from its
        // inputs): the tile is in key order (mode 0).
        if (a.contig || j0 + j >= a.new_tile0) return make_int2(-1, -1);
        int lp = (j0 + j) * kPagesPerTile + (lane & (kPagesPerTile - 1));
        if (lp >= a.n_pages) lp = a.n_pages - 1;
        return a.table[lp];
    };
    int2 next_e = g < n_tiles ? entry(g) : make_int2(0, 0);
    const uint32_t t_s = tmem + lane_base + g * 128;           // this group's S / P buffer, this warp's lanes
    const uint32_t t_o = tmem + lane_base + kColO + g * 128;   // this group's O

    for (int j = g; j < n_tiles; j += 2) {
        const int2 cur_e = next_e;  // page entries of tile j (lanes 0-7)
        if (j + 2 < n_tiles) next_e = entry(j + 2);
        PROBE_PF(0);
        const int key0 = (j0 + j) * kBN;
        // S(j) is ready; its commit also tracks P V of this group's previous
        // tile (issued before QK(j)), so O may be rescaled without a wait.
        wait(&bar_s[g], (j >> 1) & 1);
        if (j == 0) { PROBE_EE(2); }
        tc::fence_after_sync();
        float s[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tc::ld32(t_s + c * 32, *reinterpret_cast<float(*)[32]>(&s[c * 32]));
        tc::wait_ld_into(*reinterpret_cast<float(*)[32]>(&s[0]));
        tc::reg_dep(*reinterpret_cast<float(*)[32]>(&s[32]));
        tc::reg_dep(*reinterpret_cast<float(*)[32]>(&s[64]));
        tc::reg_dep(*reinterpret_cast<float(*)[32]>(&s[96]));
        PROBE_PF(1);

        // Row max over the tile (scores unscaled: qscale > 0 keeps the order).
        const int n_ok = max(0, min(kBN, lim - key0 + 1));  // keys [0, n_ok) of the tile are visible
        if (!__all_sync(0xFFFFFFFFu, n_ok >= kBN)) {
            const int mode = tile_mode_warp(cur_e, lane, a.pool_pages, a.runs);
#pragma unroll
            for (int c = 0; c < 128; ++c)
                if (tile_key(c, mode) >= n_ok) s[c] = -INFINITY;
        }
        float mx4[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
        for (int c = 4; c < 128; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], s[c]);
        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
        PROBE_PF(2);
        // Lazy rescaling: the reference max m_run moves only when the tile's
        // max exceeds it by more than kRescaleLog2 (P then stays <= 2^8, exact
        // in the fp32 accumulators and the hi/lo split); O and l are rescaled
        // only then.
        const float m_tile = mx * a.qscale;
        const bool move = m_tile > m_run + kRescaleLog2;
        const float m_new = move ? m_tile : m_run;
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = move ? exp2_approx(m_run - m_use) : 1.f;
        // P = 2^(s * qscale - m), split into bf16 hi + bf16 lo, both by
        // truncation (the upper 16 bits; no conversion instructions): hi holds
        // P to 2^-7 relative, lo = P - hi (exact in fp32) to 2^-7 of itself,
        // so hi + lo carries P to 2^-14, where a single bf16 P would lose 2^-9
        // per probability. Packed two keys per 32-bit word, lower key in the
        // low half, as the MMA reads A from TMEM. Four partial sums keep the
        // dependent FADD chain short. Four passes of 32 keys; each pass's
        // stores to TMEM run while the next pass computes.
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
        const float neg_m = -m_use;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
            uint32_t hw[16], lw[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float p0 = exp2_approx(fmaf(s[c4 * 32 + 2 * i], a.qscale, neg_m));
                const float p1 = exp2_approx(fmaf(s[c4 * 32 + 2 * i + 1], a.qscale, neg_m));
                sum4[i & 3] += p0 + p1;
                const uint32_t b0 = __float_as_uint(p0), b1 = __float_as_uint(p1);
                hw[i] = __byte_perm(b0, b1, 0x7632);
                const float r0 = p0 - __uint_as_float(b0 & 0xFFFF0000u), r1 = p1 - __uint_as_float(b1 & 0xFFFF0000u);
                lw[i] = __byte_perm(__float_as_uint(r0), __float_as_uint(r1), 0x7632);
            }
            // P(j) overwrites S(j) in TMEM: hi in the buffer's columns
            // [0, 64), lo in [64, 128).
            tc::st16(t_s + c4 * 16, hw);
            tc::st16(t_s + 64 + c4 * 16, lw);
        }
        const float sum = (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
        PROBE_PF(4);
        l_run = l_run * alpha + sum;
        m_run = m_new;

        if (j >= 2 && __any_sync(0xFFFFFFFFu, move)) {
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                float o[32];
                tc::ld32(t_o + c * 32, o);
                tc::wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) o[i] *= alpha;
                tc::st32(t_o + c * 32, o);
            }
        }
        tc::wait_st();
        PROBE_PF(5);
        // Past the cache in the last tile: zero V's rows once it has landed
        // (P is 0 there, but stale rows could hold NaN or Inf).
        const int valid_rows = min(kBN, a.total - key0);
        if (valid_rows < kBN) {  // CTA-uniform
            const int vst = j % kStages;
            wait(&bar_v[vst], (j / kStages) & 1);
            const int mode = tile_mode_warp(cur_e, lane, a.pool_pages, a.runs);
            if (tile_key(r, mode) >= valid_rows) {
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    uint4* v0 = reinterpret_cast<uint4*>(smem + kOffV + vst * kTile + hf * kHalf + r * 128);
#pragma unroll
                    for (int c = 0; c < 8; ++c) v0[c] = make_uint4(0, 0, 0, 0);
                }
            }
            fence_proxy_async_smem();
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_p[g]);
        PROBE_PF(7);
    }

    // Merge the two groups: thread (r, g) produces dims [64 g, +64) of row r
    // from both groups' O columns and (m, l) rows exchanged through shared
    // memory (the tail of the last V stage, idle once every MMA is done and
    // clear of the cluster merge's receive area).
    if (n_tiles > 0) wait(bar_fin, 0);
    PROBE_EE(4);
    tc::fence_after_sync();
    float2* ex = reinterpret_cast<float2*>(smem + kOffEx);
    ex[g * 128 + r] = make_float2(m_run, l_run);
    consumer_sync();
    const float2 oth = ex[(1 - g) * 128 + r];
    const float m0 = g == 0 ? m_run : oth.x, l0 = g == 0 ? l_run : oth.y;
    const float m1 = g == 0 ? oth.x : m_run, l1 = g == 0 ? oth.y : l_run;
    const float Mg = fmaxf(m0, m1);
    const float Mgs = Mg == -INFINITY ? 0.f : Mg;
    const float f0 = exp2_approx(m0 - Mgs), f1 = exp2_approx(m1 - Mgs);
    const int hc = g;  // which 64 of the 128 output dims this thread owns
    float o[64];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        float a0[32], a1[32];
        tc::ld32(tmem + lane_base + kColO + hc * 64 + c * 32, a0);
        tc::ld32(tmem + lane_base + kColO + 128 + hc * 64 + c * 32, a1);
        tc::wait_ld();  // warp-collective: executed even on the error path
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            // Group 1 has no tile when n_tiles < 2 (its O was never written);
            // neither group has one when n_tiles == 0.
            const float x0 = n_tiles > 0 ? a0[i] * f0 : 0.f;
            o[c * 32 + i] = n_tiles > 1 ? fmaf(a1[i], f1, x0) : x0;
        }
    }
    m_run = Mg;
    l_run = (n_tiles > 0 ? l0 * f0 : 0.f) + (n_tiles > 1 ? l1 * f1 : 0.f);
    PROBE_EE(5);
    launch_next();
    // Reduce-scatter over the cluster: CTA k finalises and stores query rows
    // [k * 128 / n, (k + 1) * 128 / n). Each CTA writes the partials of the
    // rows it does not own into its own (idle) shared memory and sends each
    // other CTA that CTA's rows with bulk copies into its receive slot,
    // completing on the receiver's bar_recv. Per-thread st.shared::cluster
    // stores of the same bytes ran at ~10 B/clk; a leader receiving every
    // row took 1.7 us for the copy alone.
    const int row_lo = rank * kBM / n_split, row_hi = (rank + 1) * kBM / n_split;
    const bool own = r >= row_lo && r < row_hi;
    float l_fin = l_run;
    if (n_split > 1) {
        // Partials: O rows [128][128] fp32 at offset 0, 16-byte pieces
        // XOR-permuted by the row's low 3 bits (rows are 512 bytes apart; the
        // 8 threads of a shared-memory phase then hit distinct banks), and
        // (m, l, -, -) per row at kRecvO.
        if (!own) {
            float4* mine = reinterpret_cast<float4*>(smem + r * kHeadDim * 4 + hc * 64 * 4);
#pragma unroll
            for (int i = 0; i < 16; ++i) mine[i ^ (r & 7)] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
            if (hc == 0) reinterpret_cast<float4*>(smem + kRecvO)[r] = make_float4(m_run, l_run, 0.f, 0.f);
            fence_proxy_async_smem();
        }
        if (tid == 0) mbar_arrive_expect_tx(bar_recv, (uint32_t)((n_split - 1) * (row_hi - row_lo)) * kRowBytes);
        // Every CTA's MMAs are done (its shared memory may be overwritten) and
        // its partials are written.
        tc::fence_before_sync();
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
        PROBE_EE(8);
        if (tid == 0) {
            for (int d = 0; d < n_split; ++d) {
                if (d == rank) continue;
                const int lo = d * kBM / n_split, n = (d + 1) * kBM / n_split - lo;
                const uint32_t slot = kOffRecv + (uint32_t)(rank < d ? rank : rank - 1) * kRecvSlot;
                uint32_t dst_o, dst_ml, bar;
                asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(dst_o) : "r"(smem_addr(smem + slot)), "r"(d));
                asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                             : "=r"(dst_ml)
                             : "r"(smem_addr(smem + slot + kRecvSlotO)), "r"(d));
                asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(bar) : "r"(smem_addr(bar_recv)), "r"(d));
                // The O rows in 4 pieces (several copies in flight), then (m, l).
                const uint32_t ob = (uint32_t)n * kHeadDim * 4, piece = (ob / 4 + 15) / 16 * 16;
                for (uint32_t off = 0; off < ob; off += piece) {
                    const uint32_t bytes = ob - off < piece ? ob - off : piece;
                    asm volatile(
                        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                            dst_o + off),
                        "r"(smem_addr(smem + (uint32_t)lo * kHeadDim * 4 + off)), "r"(bytes), "r"(bar)
                        : "memory");
                }
                asm volatile(
                    "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                        dst_ml),
                    "r"(smem_addr(smem + kRecvO + (uint32_t)lo * 16)), "r"((uint32_t)n * 16), "r"(bar)
                    : "memory");
            }
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            PROBE_EE(9);
            // The sources must stay valid until the copies have read them.
            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        }
        // Waited for even after an earlier timeout: the CTA must not exit
        // while copies into its shared memory are in flight.
        if (!mbar_wait_bounded(bar_recv, 0)) ok = false;
        PROBE_EE(10);
        if (own) {
            const int lr = r - row_lo;  // row within the received slots
            float M = m_run;
            for (int k = 0; k < n_split - 1; ++k)
                M = fmaxf(M, reinterpret_cast<const float4*>(smem + kOffRecv + k * kRecvSlot + kRecvSlotO)[lr].x);
            const float Ms = M == -INFINITY ? 0.f : M;
            const float f0 = exp2_approx(m_run - Ms);
            l_fin = l_run * f0;
#pragma unroll
            for (int i = 0; i < 64; ++i) o[i] *= f0;
            for (int k = 0; k < n_split - 1; ++k) {
                const float4 ml = reinterpret_cast<const float4*>(smem + kOffRecv + k * kRecvSlot + kRecvSlotO)[lr];
                const float f = exp2_approx(ml.x - Ms);
                l_fin = fmaf(ml.y, f, l_fin);
                // The sender's layout: row lo + lr of its buffer, pieces
                // permuted by that row's (= r's) low 3 bits.
                const float4* src =
                    reinterpret_cast<const float4*>(smem + kOffRecv + k * kRecvSlot + lr * kHeadDim * 4 + hc * 64 * 4);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float4 v = src[i ^ (r & 7)];
                    o[4 * i] = fmaf(v.x, f, o[4 * i]);
                    o[4 * i + 1] = fmaf(v.y, f, o[4 * i + 1]);
                    o[4 * i + 2] = fmaf(v.z, f, o[4 * i + 2]);
                    o[4 * i + 3] = fmaf(v.w, f, o[4 * i + 3]);
                }
            }
        }
    }
#ifdef GKV_PROBE_TIMELINE
#pragma unroll
    for (int i = 0; i < 64; ++i) asm volatile("" ::"f"(o[i]));
#endif
    PROBE_EE(6);
    const float inv = 1.f / l_fin;
    // This CTA's output rows through shared memory (clear of the partials
    // and the receive slots): each thread alone holds 64 elements of one row,
    // and rows are 256 or 512 bytes apart, so direct stores would touch a
    // new line per lane. The normalised fp32 rows are staged first (pieces
    // permuted as above); then a compact loop converts to the output dtype
    // with consecutive threads on consecutive 16-byte pieces of the output.
    // This code runs once per CTA from a cold instruction cache, so it is
    // kept short: a fully unrolled conversion of the 64 register values cost
    // ~2 us per CTA, and time grew with the code size of the conversion
    // rather than with its instruction count.
    uint8_t* stile = smem + kOffStage;
    if (own) {
        float4* mine = reinterpret_cast<float4*>(stile + (r - row_lo) * kHeadDim * 4 + hc * 64 * 4);
#pragma unroll
        for (int i = 0; i < 16; ++i)
            mine[i ^ (r & 7)] = make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv, o[4 * i + 3] * inv);
    }
    PROBE_EE(11);
    consumer_sync();
    PROBE_EE(12);
    {
        const int rows = min(row_hi, S - q0) - row_lo;  // this CTA's rows inside the chunk
        const float4* st4 = reinterpret_cast<const float4*>(stile);
        const size_t row0 = (size_t)hq * S + q0 + row_lo;
        if (ok && rows > 0 && a.out_dtype == 0) {
            float4* gout = reinterpret_cast<float4*>(static_cast<float*>(a.out) + row0 * kHeadDim);
#pragma unroll 1
            for (int c = tid; c < rows * 32; c += kConsumerThreads) {
                const int lr = c >> 5;
                gout[c] = st4[lr * 32 + ((c & 31) ^ ((lr + row_lo) & 7))];
            }
        } else if (ok && rows > 0) {
            // Output piece c (8 elements) = fp32 pieces 2p, 2p + 1 of its row.
            uint4* gout = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + row0 * kHeadDim);
            const bool bf = a.out_dtype == 30;
#pragma unroll 1
            for (int c = tid; c < rows * 16; c += kConsumerThreads) {
                const int lr = c >> 4, p = c & 15, sw = (lr + row_lo) & 7;
                const float4 x = st4[lr * 32 + ((2 * p) ^ sw)];
                const float4 y = st4[lr * 32 + ((2 * p + 1) ^ sw)];
                gout[c] = bf ? make_uint4(bf16x2_rn(x.x, x.y), bf16x2_rn(x.z, x.w), bf16x2_rn(y.x, y.y), bf16x2_rn(y.z, y.w))
                             : half8_rn(x, y);
            }
        }
    }
    PROBE_EE(7);
    if (!ok) atomicOr(a.err, kErrTimeout);
    tc::fence_before_sync();
    __syncthreads();
    PROBE_EE(3);
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

namespace {
// Launch prefill_tc_kernel over `rows` query rows of `heads` (query heads, or
// sequences x query heads), splitting the KV range over a cluster of up to 3
// CTAs while the query tiles alone would leave SMs idle.
cudaError_t launch_tc(const CUtensorMap& q_map, const PoolMaps& maps, const CUtensorMap* new_maps, const TcParams& a,
                      int rows, int heads, int num_sms, cudaStream_t stream) {
    static unsigned long long configured = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 64 || !(configured & (1ull << dev))) {
        e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured |= 1ull << dev;
    }
    const int tiles = ((rows + kBM - 1) / kBM) * heads;
    int n_split = num_sms / (tiles > 0 ? tiles : 1);
    if (n_split > 3) n_split = 3;
    if (n_split < 1) n_split = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((rows + kBM - 1) / kBM, heads, n_split);
    cfg.blockDim = dim3(kThreadsTc);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = n_split;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, prefill_tc_kernel, q_map, maps.k, maps.v, maps.k_run, maps.v_run,
                              new_maps ? new_maps[0] : maps.k, new_maps ? new_maps[1] : maps.v, a);
}
}  // namespace

cudaError_t launch_prefill_tc(const PoolView& pool, const CUtensorMap& q_map, const PoolMaps& maps,
                              const int2* table, const PrefillLaunch& p, uint32_t* err, int num_sms,
                              cudaStream_t stream) {
    TcParams a;
    a.table = table;
    a.out = p.out;
    a.err = err;
    a.out_dtype = p.out_dtype;
    a.n_q_heads = p.n_q_heads;
    a.n_kv_heads = pool.n_kv_heads;
    a.seq_len = p.seq_len;
    a.total = p.total;
    a.n_pages = p.n_pages;
    a.pool_pages = pool.pool_pages;
    a.causal = p.causal;
    a.runs = maps.runs ? 1 : 0;
    a.contig = 0;
    // The chunk's own tiles from its inputs: only when the chunk starts on a
    // tile boundary (every tile is then all old or all new keys).
    const int32_t n_prior = p.total - p.seq_len;
    const bool from_inputs = p.kv_new != nullptr && n_prior % kBN == 0;
    a.new_tile0 = from_inputs ? n_prior / kBN : INT_MAX;
    a.wait_at_end = from_inputs ? 1 : 0;
    a.qscale = p.scale * 1.4426950408889634f;
    return launch_tc(q_map, maps, from_inputs ? p.kv_new : nullptr, a, p.seq_len, p.n_q_heads, num_sms, stream);
}

cudaError_t launch_flash_tc(const CUtensorMap& q_map, const CUtensorMap& k_map, const CUtensorMap& v_map,
                            const FlashLaunch& f, uint32_t* err, int num_sms, cudaStream_t stream) {
    TcParams a;
    a.table = nullptr;
    a.out = f.out;
    a.err = err;
    a.out_dtype = f.out_dtype;
    a.n_q_heads = f.n_q_heads;
    a.n_kv_heads = f.n_kv_heads;
    a.seq_len = f.seq_len;
    a.total = f.seq_len;  // self-attention over the chunk: query s sits at position s
    a.n_pages = 0;
    a.pool_pages = 0;
    a.causal = f.causal;
    a.runs = 0;
    a.contig = 1;
    a.new_tile0 = INT_MAX;
    a.wait_at_end = 0;
    a.qscale = f.scale * 1.4426950408889634f;
    const PoolMaps maps{k_map, v_map, k_map, v_map, false};
    return launch_tc(q_map, maps, nullptr, a, f.seq_len, f.batch * f.n_q_heads, num_sms, stream);
}

}  // namespace gkv

#ifdef GKV_PROBE_TIMELINE
extern "C" int gkv_probe_read_prefill(long long* out, int n) {
    return (int)cudaMemcpyFromSymbol(out, gkv::g_probe_pf, sizeof(long long) * n);
}
extern "C" int gkv_probe_read_prefill_ee(unsigned long long* out, int n) {
    return (int)cudaMemcpyFromSymbol(out, gkv::g_probe_ee, sizeof(unsigned long long) * n);
}
extern "C" int gkv_probe_read_prefill_ld(long long* out, int n) {
    return (int)cudaMemcpyFromSymbol(out, gkv::g_probe_ld, sizeof(long long) * n);
}
extern "C" int gkv_probe_read_prefill_mma(long long* out, int n) {
    return (int)cudaMemcpyFromSymbol(out, gkv::g_probe_mma, sizeof(long long) * n);
}
#endif
