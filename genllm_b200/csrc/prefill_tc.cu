// prefill_tc.cu — chunked-prefill paged attention on the 5th-generation
// tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// The reference has no tensor-core path: its CUDA op runs a warp per (head,
// query) over a serial page loop (src/backend/cuda/attention.cu:401-489),
// and the CPU op folds one token at a time into an online softmax
// (src/backend/cpu/attention.cpp:156-215). Here a chunk of S queries of one
// query head attends causally over every cached page:
//
//   * CTA = 128 queries x 1 query head (grid ceil(S/128) x Hq), 8 warps; warp
//     w owns TMEM lanes [32(w%4), +32): two threads per query row, each with
//     64 of the 128 key columns of a tile (they exchange their partial max /
//     sum through spare TMEM columns);
//   * Q tile [128 x 128] and each KV tile (128 keys = 8 pages of 16 slots)
//     arrive by TMA in the 128-byte-swizzled K-major layout: per page and
//     per 64-dim half one box {64 dims, 1 head, 16 slots} of the pool's 3-D
//     map; K and V tiles are double-buffered;
//   * S = Q K^T: 8 tcgen05.mma (M128 N128 K16, bf16 -> fp32) into TMEM
//     columns [0, 128), issued by one thread, completion by tcgen05.commit;
//   * each thread loads its S row from TMEM, applies the causal / length
//     mask, and updates an fp32 online softmax (log2 domain); the
//     probabilities go to shared memory as bf16 in the swizzled K-major
//     layout; O in TMEM columns [128, 256) is rescaled in place when the
//     running max moves;
//   * O += P V: 16 tcgen05.mma with V as an MN-major operand — P enters as
//     bf16 hi + lo terms so that the products keep fp32-level accuracy;
//   * the epilogue divides by the row sum and stores fp32/bf16/fp16 rows.
//
// Keys past the cached length in the last tile are masked in S, and their V
// rows are zeroed in shared memory (0 x NaN from stale slots would poison
// the MMA). Every mbarrier wait is bounded (kErrTimeout).
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
static_assert((6 + 4 * kStages) * 8 + 4 <= 256, "barriers and the TMEM slot fit their 256 bytes");
// TMEM columns: S/P of two tiles [0, 256), O [256, 384), Q as the A operand
// of Q K^T [384, 448) (bf16 pairs), max/sum exchange [448, 452).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256, kColQ = 384, kColX = 448;

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
    float qscale;    // softmax scale * log2(e)
};

constexpr int kConsumerThreads = 256;               // 8 warps: 2 threads per query row
constexpr int kLoadWarp = kConsumerThreads / 32;   // issues the K loads (warp + 1: the V loads)
constexpr int kMmaWarp = kLoadWarp + 2;            // issues the tcgen05 MMAs
constexpr int kThreadsTc = kConsumerThreads + 96;
constexpr float kRescaleLog2 = 8.f;  // lazy-rescale threshold (log2 units)

#ifdef GKV_PROBE_TIMELINE
// Measurement builds only: per-tile phase clocks of threads 0 and 128 of the
// first CTA of the grid.
__device__ long long g_probe_pf[2 * 128 * 16];
__device__ long long g_probe_mma[128 * 4];
__device__ long long g_probe_ld[128 * 8];
__device__ unsigned long long g_probe_ee[1024 * 4];  // per CTA: entry, setup done, first S ready, exit
#define PROBE_EE(k)                                                                                          \
    if (tid == 0) {                                                                                          \
        const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;                      \
        if (cta < 1024) g_probe_ee[cta * 4 + (k)] = global_timer_ns();                                      \
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

__global__ void __launch_bounds__(kThreadsTc, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                      const __grid_constant__ CUtensorMap v_map, const __grid_constant__ CUtensorMap k_run,
                      const __grid_constant__ CUtensorMap v_run, const TcParams a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bar_q = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint64_t* bar_k = bar_q + 1;             // [kStages] K tile landed
    uint64_t* bar_v = bar_k + kStages;       // [kStages] V tile landed
    uint64_t* bar_kfree = bar_v + kStages;   // [kStages] Q K^T of the stage's tile done
    uint64_t* bar_vfree = bar_kfree + kStages;  // [kStages] P V of the stage's tile done
    uint64_t* bar_s = bar_vfree + kStages;   // [2] S of a tile in its TMEM buffer
    uint64_t* bar_o = bar_s + 2;             // P V of a tile done (in issue order)
    uint64_t* bar_p = bar_o + 1;             // consumers: P of a tile written (and S of it read)
    uint64_t* bar_qt = bar_p + 1;            // consumers: Q copied into TMEM
    constexpr int kNumBars = 6 + 4 * kStages;  // q, k, v, kfree, vfree, s[2], o, p, qt
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_q + kNumBars);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int q0 = blockIdx.x * kBM;
    const int hq = blockIdx.y;
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
    // takes tiles [j0, j0 + n_tiles) and the leader merges the results.
    const int rank = blockIdx.z, n_split = gridDim.z;
    const int j0 = rank * n_tiles_all / n_split;
    const int n_tiles = (rank + 1) * n_tiles_all / n_split - j0;

    PROBE_EE(0);
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        for (int b = 0; b < kNumBars; ++b) mbar_init(bar_q + b, 1);
        fence_mbar_init();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    PROBE_EE(1);
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;  // this warp's TMEM lanes
    const uint32_t t_o = tmem + lane_base + kColO;           // this warp's lanes of O

    const uint32_t sK = smem_addr(smem + kOffK);
    const uint32_t sV = smem_addr(smem + kOffV);
    // Q is read once; K and V tiles are read again by the CTAs of the other
    // query tiles and heads of the group, so they keep normal L2 priority.
    const uint64_t pol = l2_policy_evict_first();
    uint64_t pol_kv;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol_kv));

    // Page ids of tile j: 8 independent table loads (one latency, not 8),
    // fetched by the issuing thread a tile before they are needed.
    auto load_ids = [&](int j, int2 (&e)[kPagesPerTile]) {
#pragma unroll
        for (int i = 0; i < kPagesPerTile; ++i) {
            int lp = (j0 + j) * kPagesPerTile + i;
            if (lp >= a.n_pages) lp = a.n_pages - 1;  // beyond the cache: rows are masked / zeroed
            e[i] = a.table[lp];
        }
    };
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
    // The consumer warps' own barrier (the load warp never joins it).
    auto consumer_sync = [] { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory"); };
    // A wait that times out clears `ok`; later waits are then skipped, but
    // every thread still reaches every __syncthreads, so nothing can hang.
    auto wait = [&](uint64_t* bar, uint32_t parity) {
        if (ok && !mbar_wait_bounded(bar, parity)) ok = false;
    };
    // S(j) = Q K(j)^T into TMEM columns [(j & 1) * 128, +128), Q read from
    // TMEM: only K streams from shared memory, whose bandwidth bounds an
    // N = 128 MMA with both operands there.
    // The MMA warp runs converged; one elected lane issues. Descriptors are
    // built once and stepped by adding the byte offset / 16 to their address
    // field (smem addresses stay below 256 KiB, so the 14-bit field cannot
    // carry). A tight issue sequence keeps the tensor pipe fed: each
    // m128n128k16 MMA takes 64 cycles, about what loose issue code spends
    // between two MMAs.
    const uint64_t desc_k0 = tc::smem_desc_sw128(sK, 16, 1024);
    const uint64_t desc_v0 = tc::smem_desc_sw128(sV, kHalf, 1024);
    auto issue_qk = [&](int j) {
        const int sb = j & 1, st = j % kStages;
        wait(&bar_k[st], (j / kStages) & 1);
        PROBE_LD(6);
        tc::fence_after_sync();
        if (tc::elect_one()) {
            const uint64_t dk = desc_k0 + ((st * kTile) >> 4);
            const uint32_t d = tmem + sb * 128;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
                tc::mma_bf16_ts(d, tmem + kColQ + kk * 8, dk + ((((kk >> 2) * kHalf) + (kk & 3) * 32) >> 4), kIdescQK,
                                kk > 0);
            tc::commit(&bar_s[sb]);
            tc::commit(&bar_kfree[st]);
        }
        __syncwarp();
    };

    // P(j) V(j) into the O columns [256, 384), both bf16 terms of P, with P
    // read from TMEM (where it replaced S(j)).
    auto issue_pv = [&](int j) {
        const int sb = j & 1, st = j % kStages;
        if (tc::elect_one()) {
            const uint64_t dv = desc_v0 + ((st * kTile) >> 4);
            const uint32_t p = tmem + sb * 128;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                tc::mma_bf16_ts(tmem + kColO, p + kk * 8, dv + ((kk * 2048) >> 4), kIdescPV, j > 0 || kk > 0);
                tc::mma_bf16_ts(tmem + kColO, p + 64 + kk * 8, dv + ((kk * 2048) >> 4), kIdescPV, true);
            }
            tc::commit(bar_o);
            tc::commit(&bar_vfree[st]);
        }
        __syncwarp();
    };

    // Warp-specialised software pipeline. The consumer warps (0-7) run the
    // softmax of tile j while the tensor cores compute S of tile j+1 (two S
    // buffers in TMEM). One load warp issues K(j) once QK(j-3) has freed its
    // stage, another V(j) once PV(j-3) has; the MMA warp
    // issues QK(0), QK(1), then per tile PV(j) once the consumers have written
    // P(j), followed by QK(j+2) into the TMEM buffer P(j) occupied.
    if (warp == kMmaWarp) {
        if (n_tiles > 0) {
            wait(bar_qt, 0);
            tc::fence_after_sync();
            issue_qk(0);
            if (n_tiles > 1) issue_qk(1);
            for (int j = 0; j < n_tiles && ok; ++j) {
                wait(bar_p, j & 1);
                PROBE_MMA(0);
                tc::fence_after_sync();
                if (!ok) break;
                issue_pv(j);
                if (j + 2 < n_tiles) {
                    wait(bar_o, j & 1);  // QK(j+2) overwrites P(j) in TMEM
                    PROBE_MMA(1);
                    tc::fence_after_sync();
                    issue_qk(j + 2);
                    PROBE_MMA(2);
                }
            }
            if (!ok) atomicOr(a.err, kErrTimeout);
        }
        __syncwarp();
        if (n_split > 1) {  // the consumers' two cluster barriers
            asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
            asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
        }
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
            if (n_tiles > 0 && !a.contig) load_ids(0, ids);
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
        if (n_split > 1) {  // the consumers' two cluster barriers
            asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
            asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
        }
        tc::fence_before_sync();
        __syncthreads();
        return;
    }

    const int r = tid & 127;  // query row of this thread
    const int hc = tid >> 7;  // which 64 of the 128 key columns (and O columns)
    const uint32_t t_x = tmem + lane_base + kColX;  // exchange columns: [kColX + 2 hc, +2)
    if (n_tiles > 0) {
        // Q into TMEM: this thread's row r, dims [64 hc, +64) from the
        // swizzled smem tile, two dims per column (lower dim in the low half).
        wait(bar_q, 0);
        uint32_t qw[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint4 v = *reinterpret_cast<const uint4*>(smem + kOffQ + hc * kHalf + r * 128 + ((c ^ (r & 7)) << 4));
            qw[4 * c] = v.x;
            qw[4 * c + 1] = v.y;
            qw[4 * c + 2] = v.z;
            qw[4 * c + 3] = v.w;
        }
        tc::st32(tmem + lane_base + kColQ + hc * 32, *reinterpret_cast<const float(*)[32]>(qw));
        tc::wait_st();
        tc::fence_before_sync();
        consumer_sync();
        if (tid == 0) mbar_arrive(bar_qt);
    }
    const int q_abs = first_q_abs + r;
    const int lim = a.causal ? min(q_abs, a.total - 1) : a.total - 1;  // last visible key
    float m_run = -INFINITY, l_run = 0.f;
    // Lanes 0-7 of every consumer warp hold the next tile's page entries
    // (fetched a tile ahead) to derive its copy mode.
    const int lane = tid & 31;
    auto entry = [&](int j) {
        if (a.contig) return make_int2(-1, -1);  // no table: every tile is in key order (mode 0)
        int lp = (j0 + j) * kPagesPerTile + (lane & (kPagesPerTile - 1));
        if (lp >= a.n_pages) lp = a.n_pages - 1;
        return a.table[lp];
    };
    int2 next_e = n_tiles > 0 ? entry(0) : make_int2(0, 0);

    // S(j) is loaded from TMEM at the end of tile j-1, so the load latency
    // overlaps the loop turn-around.
    float s[64];
    auto load_s = [&](int j) {
        wait(&bar_s[j & 1], (j >> 1) & 1);
        if (j == 0) { PROBE_EE(2); }
        tc::fence_after_sync();
#pragma unroll
        for (int c = 0; c < 2; ++c)
            tc::ld32(tmem + lane_base + (j & 1) * 128 + hc * 64 + c * 32, *reinterpret_cast<float(*)[32]>(&s[c * 32]));
    };
    if (n_tiles > 0) load_s(0);

    for (int j = 0; j < n_tiles; ++j) {
        const int st = j & 1;
        const int2 cur_e = next_e;  // page entries of tile j (lanes 0-7)
        if (j + 1 < n_tiles) next_e = entry(j + 1);
        PROBE_PF(0);
        const int key0 = (j0 + j) * kBN;
        tc::wait_ld_into(*reinterpret_cast<float(*)[32]>(&s[0]));
        tc::reg_dep(*reinterpret_cast<float(*)[32]>(&s[32]));
        PROBE_PF(1);

        // Row max over the tile: local over this thread's 64 keys, then one
        // exchange with the row's other thread through spare TMEM columns.
        // Scores stay unscaled here (qscale > 0 keeps the order).
        const int n_ok = max(0, min(kBN, lim - key0 + 1));  // keys [0, n_ok) of the tile are visible
        if (!__all_sync(0xFFFFFFFFu, n_ok >= kBN)) {
            const int mode = tile_mode_warp(cur_e, lane, a.pool_pages, a.runs);
#pragma unroll
            for (int c = 0; c < 64; ++c)
                if (tile_key(hc * 64 + c, mode) >= n_ok) s[c] = -INFINITY;
        }
        float mx = s[0];
#pragma unroll
        for (int c = 1; c < 64; ++c) mx = fmaxf(mx, s[c]);
        PROBE_PF(2);
        tc::st2(t_x + 2 * hc, mx, 0.f);
        tc::wait_st();
        tc::fence_before_sync();
        consumer_sync();
        tc::fence_after_sync();
        PROBE_PF(3);
        float mx2, unused;
        tc::ld2(t_x + 2 * (1 - hc), mx2, unused);
        tc::wait_ld();
        // Lazy rescaling: the reference max m_run moves only when the tile's
        // max exceeds it by more than kRescaleLog2 (P then stays <= 2^8, exact
        // in the fp32 accumulators and the hi/lo split); O and l are rescaled
        // only then, so most tiles never wait for the previous P V.
        const float m_tile = fmaxf(mx, mx2) * a.qscale;
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
        // dependent FADD chain short.
        // Two passes of 32 keys; each pass's stores to TMEM run while the
        // next pass computes.
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
        const float neg_m = -m_use;
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
            uint32_t hw[16], lw[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float p0 = exp2_approx(fmaf(s[h2 * 32 + 2 * i], a.qscale, neg_m));
                const float p1 = exp2_approx(fmaf(s[h2 * 32 + 2 * i + 1], a.qscale, neg_m));
                sum4[i & 3] += p0 + p1;
                const uint32_t b0 = __float_as_uint(p0), b1 = __float_as_uint(p1);
                hw[i] = __byte_perm(b0, b1, 0x7632);
                const float r0 = p0 - __uint_as_float(b0 & 0xFFFF0000u), r1 = p1 - __uint_as_float(b1 & 0xFFFF0000u);
                lw[i] = __byte_perm(__float_as_uint(r0), __float_as_uint(r1), 0x7632);
            }
            // P(j) overwrites S(j) in TMEM: hi in the buffer's columns
            // [0, 64), lo in [64, 128); this thread's 64 keys are 32 columns
            // of each.
            tc::st16(tmem + lane_base + st * 128 + hc * 32 + h2 * 16, hw);
            tc::st16(tmem + lane_base + st * 128 + 64 + hc * 32 + h2 * 16, lw);
        }
        const float sum = (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
        PROBE_PF(4);
        l_run = l_run * alpha + sum;  // this thread's share of the row sum
        m_run = m_new;

        if (j > 0 && __any_sync(0xFFFFFFFFu, move)) {
            // P V of tile j-1 must be done before O is rescaled. (The stage's
            // previous P V is done already: V(j-1) was loaded into the stage
            // after it, so the barrier's parity identifies PV(j-1).)
            wait(&bar_vfree[(j - 1) % kStages], ((j - 1) / kStages) & 1);
            tc::fence_after_sync();
            {
#pragma unroll
                for (int c = hc * 2; c < hc * 2 + 2; ++c) {
                    float o[32];
                    tc::ld32(t_o + c * 32, o);
                    tc::wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] *= alpha;
                    tc::st32(t_o + c * 32, o);
                }
            }
        }
        tc::wait_st();
        PROBE_PF(5);
        // V(j) must have landed; zero its rows past the cache (P is 0 there,
        // but stale rows could hold NaN or Inf).
        const int vst = j % kStages;
        wait(&bar_v[vst], (j / kStages) & 1);
        PROBE_PF(6);
        const int valid_rows = min(kBN, a.total - key0);
        if (valid_rows < kBN) {  // CTA-uniform
            const int mode = tile_mode_warp(cur_e, lane, a.pool_pages, a.runs);
            if (tile_key(r, mode) >= valid_rows) {
                uint4* v0 = reinterpret_cast<uint4*>(smem + kOffV + vst * kTile + hc * kHalf + r * 128);
#pragma unroll
                for (int c = 0; c < 8; ++c) v0[c] = make_uint4(0, 0, 0, 0);
            }
            fence_proxy_async_smem();
        }
        tc::fence_before_sync();
        consumer_sync();
        PROBE_PF(7);
        if (tid == 0) mbar_arrive(bar_p);
        PROBE_PF(8);
        if (j + 1 < n_tiles) load_s(j + 1);
    }

    if (n_tiles > 0) wait(bar_o, (n_tiles - 1) & 1);
    tc::fence_after_sync();
    float o[64];
#pragma unroll
    for (int c = 0; c < 2; ++c) tc::ld32(t_o + hc * 64 + c * 32, *reinterpret_cast<float(*)[32]>(&o[c * 32]));
    tc::wait_ld();  // warp-collective: executed even on the error path
    if (n_tiles == 0) {
#pragma unroll
        for (int i = 0; i < 64; ++i) o[i] = 0.f;
    }
    {
        // Each thread holds the sum over its own 64 keys of every tile.
        tc::st2(t_x + 2 * hc, l_run, 0.f);
        tc::wait_st();
        tc::fence_before_sync();
        consumer_sync();
        tc::fence_after_sync();
        float l2, unused;
        tc::ld2(t_x + 2 * (1 - hc), l2, unused);
        tc::wait_ld();
        l_run += l2;
    }
    float l_fin = l_run;
    if (n_split > 1) {
        // Merge through distributed shared memory: the other CTAs of the
        // cluster send (m, l, O row half) into the leader's (now idle) buffers.
        tc::fence_before_sync();
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
        constexpr uint32_t kRecvO = 128 * kHeadDim * 4;  // 64 KiB per sending CTA
        constexpr uint32_t kRecvMl = 3 * kRecvO;
        const uint32_t row_off = r * kHeadDim * 4 + hc * 64 * 4;
        if (rank > 0) {
            const uint32_t local = smem_addr(smem + (rank - 1) * kRecvO + row_off);
            uint32_t remote;
            asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(remote) : "r"(local));
#pragma unroll
            for (int i = 0; i < 16; ++i)
                asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(remote + i * 16), "f"(o[4 * i]),
                             "f"(o[4 * i + 1]), "f"(o[4 * i + 2]), "f"(o[4 * i + 3])
                             : "memory");
            if (hc == 0) {
                const uint32_t lml = smem_addr(smem + kRecvMl + ((rank - 1) * 128 + r) * 8);
                uint32_t rml;
                asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(rml) : "r"(lml));
                asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(rml), "f"(m_run), "f"(l_run) : "memory");
            }
        }
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
        if (rank == 0) {
            float M = m_run;
            for (int k = 1; k < n_split; ++k) M = fmaxf(M, reinterpret_cast<const float2*>(smem + kRecvMl)[(k - 1) * 128 + r].x);
            const float Ms = M == -INFINITY ? 0.f : M;
            const float f0 = exp2_approx(m_run - Ms);
            l_fin = l_run * f0;
#pragma unroll
            for (int i = 0; i < 64; ++i) o[i] *= f0;
            for (int k = 1; k < n_split; ++k) {
                const float2 ml = reinterpret_cast<const float2*>(smem + kRecvMl)[(k - 1) * 128 + r];
                const float f = exp2_approx(ml.x - Ms);
                l_fin = fmaf(ml.y, f, l_fin);
                const float4* src = reinterpret_cast<const float4*>(smem + (k - 1) * kRecvO + row_off);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float4 v = src[i];
                    o[4 * i] = fmaf(v.x, f, o[4 * i]);
                    o[4 * i + 1] = fmaf(v.y, f, o[4 * i + 1]);
                    o[4 * i + 2] = fmaf(v.z, f, o[4 * i + 2]);
                    o[4 * i + 3] = fmaf(v.w, f, o[4 * i + 3]);
                }
            }
        }
    }
    const float inv = 1.f / l_fin;
    // Output tile [128 queries][128 dims] through shared memory (the V stage
    // buffers, idle now and clear of the merge's receive area), then stored
    // with consecutive threads on consecutive 16-byte pieces of a row: each
    // thread alone holds 64 elements of one row, and rows are 256 or 512
    // bytes apart, so direct stores would touch a new line per lane.
    if (rank == 0) {
        const int es = a.out_dtype == 0 ? 4 : 2;
        uint8_t* stile = smem + kOffV;
        uint8_t* mine = stile + r * kHeadDim * es + hc * 64 * es;
        if (es == 4) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
                reinterpret_cast<float4*>(mine)[i] =
                    make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv, o[4 * i + 3] * inv);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                uint32_t w[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float v0 = o[8 * i + 2 * k] * inv, v1 = o[8 * i + 2 * k + 1] * inv;
                    uint32_t b0, b1;
                    if (a.out_dtype == 30) {
                        b0 = bf16_bits_ref(v0);
                        b1 = bf16_bits_ref(v1);
                    } else {
                        b0 = __half_as_ushort(__float2half_rn(v0));
                        b1 = __half_as_ushort(__float2half_rn(v1));
                    }
                    w[k] = b0 | (b1 << 16);
                }
                reinterpret_cast<uint4*>(mine)[i] = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
        consumer_sync();
        const int row_chunks = kHeadDim * es / 16;  // 16-byte pieces per row
        const int rows = min(kBM, S - q0);
        uint8_t* gout = static_cast<uint8_t*>(a.out) + ((size_t)hq * S + q0) * kHeadDim * es;
        if (ok) {
            for (int c = tid; c < rows * row_chunks; c += kConsumerThreads)
                reinterpret_cast<uint4*>(gout)[c] = reinterpret_cast<const uint4*>(stile)[c];
        }
    }
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
cudaError_t launch_tc(const CUtensorMap& q_map, const PoolMaps& maps, const TcParams& a, int rows, int heads,
                      int num_sms, cudaStream_t stream) {
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
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = n_split;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, prefill_tc_kernel, q_map, maps.k, maps.v, maps.k_run, maps.v_run, a);
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
    a.qscale = p.scale * 1.4426950408889634f;
    return launch_tc(q_map, maps, a, p.seq_len, p.n_q_heads, num_sms, stream);
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
    a.qscale = f.scale * 1.4426950408889634f;
    const PoolMaps maps{k_map, v_map, k_map, v_map, false};
    return launch_tc(q_map, maps, a, f.seq_len, f.batch * f.n_q_heads, num_sms, stream);
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
