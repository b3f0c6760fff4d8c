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
constexpr uint32_t kOffK = kOffQ + kTile;      // 2 stages
constexpr uint32_t kOffV = kOffK + 2 * kTile;  // 2 stages
constexpr uint32_t kOffP = kOffV + 2 * kTile;   // P as bf16 hi part
constexpr uint32_t kOffPlo = kOffP + kTile;     // and lo part (P - hi), for fp32-level PV accuracy
constexpr uint32_t kOffBar = kOffPlo + kTile;
constexpr uint32_t kSmemBytes = kOffBar + 128 + 1024;  // + 8 barriers, TMEM slot, alignment slack
constexpr uint32_t kTmemCols = 512;            // S: two buffers [0, 256), O: [256, 384)

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
    float qscale;  // softmax scale * log2(e)
};

constexpr int kConsumerThreads = 256;               // 8 warps: 2 threads per query row
constexpr int kLoadWarp = kConsumerThreads / 32;   // issues the TMA loads
constexpr int kMmaWarp = kLoadWarp + 1;            // issues the tcgen05 MMAs
constexpr int kThreadsTc = kConsumerThreads + 64;

#ifdef GKV_PROBE_TIMELINE
// Measurement builds only: per-tile phase clocks of threads 0 and 128 of the
// first CTA of the grid.
__device__ long long g_probe_pf[2 * 128 * 8];
#define PROBE_PF(k)                                                                                  \
    if ((tid & 127) == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && j < 128)        \
        g_probe_pf[((tid >> 7) * 128 + j) * 8 + (k)] = clock64();
#else
#define PROBE_PF(k)
#endif

__global__ void __launch_bounds__(kThreadsTc, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                      const __grid_constant__ CUtensorMap v_map, const TcParams a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bar_q = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint64_t* bar_k = bar_q + 1;  // [2] K tile landed
    uint64_t* bar_v = bar_q + 3;  // [2] V tile landed
    uint64_t* bar_s = bar_q + 5;  // [2] S = Q K^T of a tile done
    uint64_t* bar_o = bar_q + 7;  // P V of a tile done (consumers)
    uint64_t* bar_vfree = bar_q + 8;  // [2] P V of a tile done (load warp: V buffer free)
    uint64_t* bar_p = bar_q + 10;     // consumers: P of a tile written (and S of it read)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_q + 11);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int q0 = blockIdx.x * kBM;
    const int hq = blockIdx.y;
    const int G = a.n_q_heads / a.n_kv_heads;
    const int h = hq / G;
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

    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        for (int b = 0; b < 11; ++b) mbar_init(bar_q + b, 1);
        fence_mbar_init();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;  // this warp's TMEM lanes
    const uint32_t t_o = tmem + lane_base + 256;             // O columns [256, 384)

    const uint32_t sQ = smem_addr(smem + kOffQ);
    const uint32_t sK = smem_addr(smem + kOffK);
    const uint32_t sV = smem_addr(smem + kOffV);
    const uint32_t sP = smem_addr(smem + kOffP);
    const uint32_t sPlo = smem_addr(smem + kOffPlo);
    const uint64_t pol = l2_policy_evict_first();

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
    // Stage tile j's K (which = 0) or V (which = 1) into buffer (j & 1): 8
    // pages x 2 halves, one TMA box {64, 1, 16} each.
    auto issue = [&](int j, int which, const int2 (&ids)[kPagesPerTile]) {
        const int st = j & 1;
        uint64_t* bar = which ? &bar_v[st] : &bar_k[st];
        mbar_arrive_expect_tx(bar, kTile);
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
                                e.x * kPageSlots, pol);
                else
                    tma_load_3d(smem + kOffV + st * kTile + hf * kHalf + i * 2048, &v_map, bar, hf * 64, h,
                                e.y * kPageSlots, pol);
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
    // S(j) = Q K(j)^T into TMEM columns [(j & 1) * 128, +128).
    auto issue_qk = [&](int j) {
        const int st = j & 1;
        wait(&bar_k[st], (j >> 1) & 1);
        tc::fence_after_sync();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
            tc::mma_bf16(tmem + st * 128, tc::smem_desc_sw128(sQ + off, 16, 1024),
                         tc::smem_desc_sw128(sK + st * kTile + off, 16, 1024), kIdescQK, kk > 0);
        }
        tc::commit(&bar_s[st]);
    };

    // P(j) V(j) into the O columns [256, 384), both bf16 terms of P.
    auto issue_pv = [&](int j) {
        const int st = j & 1;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const uint32_t po = (kk >> 2) * kHalf + (kk & 3) * 32;
            const uint64_t db = tc::smem_desc_sw128(sV + st * kTile + kk * 2048, kHalf, 1024);
            tc::mma_bf16(tmem + 256, tc::smem_desc_sw128(sP + po, 16, 1024), db, kIdescPV, j > 0 || kk > 0);
            tc::mma_bf16(tmem + 256, tc::smem_desc_sw128(sPlo + po, 16, 1024), db, kIdescPV, true);
        }
        tc::commit(bar_o);
        tc::commit(&bar_vfree[st]);
    };

    // Warp-specialised software pipeline. The consumer warps (0-7) run the
    // softmax of tile j while the tensor cores compute S of tile j+1 (two S
    // buffers in TMEM). The load warp issues K(j) once QK(j-2) is done and
    // V(j) once PV(j-2) is done; the MMA warp issues QK(0), QK(1), then per
    // tile PV(j) once the consumers have written P(j), followed by QK(j+2)
    // into the S buffer the consumers just finished reading.
    if (warp == kMmaWarp) {
        if ((tid & 31) == 0 && n_tiles > 0) {
            wait(bar_q, 0);
            issue_qk(0);
            if (n_tiles > 1) issue_qk(1);
            for (int j = 0; j < n_tiles && ok; ++j) {
                wait(bar_p, j & 1);
                tc::fence_after_sync();
                if (!ok) break;
                issue_pv(j);
                if (j + 2 < n_tiles) issue_qk(j + 2);
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
    if (warp == kLoadWarp) {
        if ((tid & 31) == 0) {
            mbar_arrive_expect_tx(bar_q, kTile);
            tma_load_3d(smem + kOffQ, &q_map, bar_q, 0, q0, hq, pol);
            tma_load_3d(smem + kOffQ + kHalf, &q_map, bar_q, 64, q0, hq, pol);
            int2 ids[kPagesPerTile], nxt[kPagesPerTile];
            if (n_tiles > 0) load_ids(0, ids);
            for (int j = 0; j < n_tiles && ok; ++j) {
                const int st = j & 1;
                if (j + 1 < n_tiles) load_ids(j + 1, nxt);
                if (j >= 2) wait(&bar_s[st], ((j - 2) >> 1) & 1);
                if (!ok) break;
                issue(j, 0, ids);
                if (j >= 2) wait(&bar_vfree[st], ((j - 2) >> 1) & 1);
                if (!ok) break;
                issue(j, 1, ids);
#pragma unroll
                for (int i = 0; i < kPagesPerTile; ++i) ids[i] = nxt[i];
            }
            if (n_tiles == 0) wait(bar_q, 0);  // the Q load must land before the CTA exits
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
    const uint32_t t_x = tmem + lane_base + 384;  // exchange columns: [384 + 2 hc, +2)
    const int q_abs = first_q_abs + r;
    const int lim = a.causal ? min(q_abs, a.total - 1) : a.total - 1;  // last visible key
    float m_run = -INFINITY, l_run = 0.f;

    for (int j = 0; j < n_tiles; ++j) {
        const int st = j & 1;
        PROBE_PF(0);
        wait(&bar_s[st], (j >> 1) & 1);
        PROBE_PF(1);
        tc::fence_after_sync();
        const int key0 = (j0 + j) * kBN;

        float s[64];
#pragma unroll
        for (int c = 0; c < 2; ++c)
            tc::ld32(tmem + lane_base + st * 128 + hc * 64 + c * 32, *reinterpret_cast<float(*)[32]>(&s[c * 32]));
        tc::wait_ld();

        // Local max and sum over this thread's 64 columns, one exchange with
        // the row's other thread, then a common max.
        const int n_ok = max(0, min(kBN, lim - key0 + 1)) - hc * 64;
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
            const float v = c < n_ok ? s[c] * a.qscale : -INFINITY;
            s[c] = v;
            mx = fmaxf(mx, v);
        }
        const float ml_use = mx == -INFINITY ? 0.f : mx;
        float sum = 0.f;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
            const float p = exp2_approx(s[c] - ml_use);
            s[c] = p;
            sum += p;
        }
        PROBE_PF(2);
        tc::st2(t_x + 2 * hc, mx, sum);
        tc::wait_st();
        tc::fence_before_sync();
        consumer_sync();
        tc::fence_after_sync();
        PROBE_PF(3);
        float mx2, sum2;
        tc::ld2(t_x + 2 * (1 - hc), mx2, sum2);
        tc::wait_ld();
        const float m_new = fmaxf(m_run, fmaxf(mx, mx2));
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = exp2_approx(m_run - m_use);
        const float f_me = exp2_approx(mx - m_use), f_other = exp2_approx(mx2 - m_use);
#pragma unroll
        for (int c = 0; c < 64; ++c) s[c] *= f_me;
        l_run = l_run * alpha + sum * f_me + sum2 * f_other;
        m_run = m_new;

        if (j > 0) {
            // P V of tile j-1 must be done before P and O are touched.
            wait(bar_o, (j - 1) & 1);
            PROBE_PF(4);
            tc::fence_after_sync();
            if (__any_sync(0xFFFFFFFFu, alpha != 1.f)) {
#pragma unroll
                for (int c = hc * 2; c < hc * 2 + 2; ++c) {
                    float o[32];
                    tc::ld32(t_o + c * 32, o);
                    tc::wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] *= alpha;
                    tc::st32(t_o + c * 32, o);
                }
                tc::wait_st();
            }
        }

        // P into the swizzled K-major layout (row r, 16-byte chunk c of each
        // 64-key half at position c ^ (r & 7)) as two bf16 terms, hi = bf16(P)
        // and lo = bf16(P - hi): P.V = hi.V + lo.V keeps fp32-level accuracy
        // where a single bf16 P would lose 2^-9 relative per probability.
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
            const int c = hc * 8 + c8;
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float x0 = s[c8 * 8 + 2 * i], x1 = s[c8 * 8 + 2 * i + 1];
                const __nv_bfloat162 h2 = __floats2bfloat162_rn(x0, x1);
                const float2 hf2 = __bfloat1622float2(h2);
                const __nv_bfloat162 l2 = __floats2bfloat162_rn(x0 - hf2.x, x1 - hf2.y);
                hw[i] = *reinterpret_cast<const uint32_t*>(&h2);
                lw[i] = *reinterpret_cast<const uint32_t*>(&l2);
            }
            const int hf = c >> 3, cc = c & 7;
            const uint32_t off = hf * kHalf + r * 128 + ((cc ^ (r & 7)) * 16);
            *reinterpret_cast<uint4*>(smem + kOffP + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4*>(smem + kOffPlo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        PROBE_PF(5);
        // V(j) must have landed; zero its rows past the cache.
        wait(&bar_v[st], (j >> 1) & 1);
        PROBE_PF(6);
        const int valid_rows = min(kBN, a.total - key0);
        if (r >= valid_rows) {
            uint4* v0 = reinterpret_cast<uint4*>(smem + kOffV + st * kTile + hc * kHalf + r * 128);
#pragma unroll
            for (int c = 0; c < 8; ++c) v0[c] = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
        tc::fence_before_sync();
        consumer_sync();
        PROBE_PF(7);
        if (tid == 0) mbar_arrive(bar_p);
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
    const int q = q0 + r;
    if (rank == 0 && ok && q < S) {
        const size_t base = ((size_t)hq * S + q) * kHeadDim + hc * 64;
        if (a.out_dtype == 0) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + base);
#pragma unroll
            for (int i = 0; i < 16; ++i)
                dst[i] = make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv, o[4 * i + 3] * inv);
        } else {
#pragma unroll
            for (int i = 0; i < 64; ++i) store_out(a.out, base + i, o[i] * inv, a.out_dtype);
        }
    }
    if (!ok) atomicOr(a.err, kErrTimeout);
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

cudaError_t launch_prefill_tc(const PoolView& pool, const CUtensorMap& q_map, const CUtensorMap& k_map,
                              const CUtensorMap& v_map, const int2* table, const PrefillLaunch& p, uint32_t* err,
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
    a.qscale = p.scale * 1.4426950408889634f;
    // Split the KV range over a cluster of up to 3 CTAs while the query tiles
    // alone would leave SMs idle.
    const int tiles = ((p.seq_len + kBM - 1) / kBM) * p.n_q_heads;
    int n_split = num_sms / (tiles > 0 ? tiles : 1);
    if (n_split > 3) n_split = 3;
    if (n_split < 1) n_split = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.seq_len + kBM - 1) / kBM, p.n_q_heads, n_split);
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
    return cudaLaunchKernelEx(&cfg, prefill_tc_kernel, q_map, k_map, v_map, a);
}

}  // namespace gkv

#ifdef GKV_PROBE_TIMELINE
extern "C" int gkv_probe_read_prefill(long long* out, int n) {
    return (int)cudaMemcpyFromSymbol(out, gkv::g_probe_pf, sizeof(long long) * n);
}
#endif
