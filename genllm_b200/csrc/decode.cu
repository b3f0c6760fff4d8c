// decode.cu — fused paged-attention decode step for sm_100a.
//
// One launch does what the reference spreads over 2*Hkv synchronous
// cudaMemcpy calls, a cudaMalloc/H2D/cudaFree of the page ids and a
// warp-per-head kernel with a serial page loop (src/core/page_attention.cpp:
// 104-139, src/backend/cuda/attention.cu:401-580):
//
//   * grid (n_splits, Hkv): a CTA owns ONE kv head and a contiguous range of
//     logical pages, and all G = Hq/Hkv query heads of that kv head, so every
//     KV byte is read from HBM exactly once (GQA grouping);
//   * each of its 4 warps runs its own TMA pipeline: R stages of one
//     (page, head) K tile and V tile (16 slots x 128 x bf16 = 4 KiB each),
//     loaded with cp.async.bulk.tensor (3-D map over the pool, box
//     {128, 1, 16}, evict-first L2 policy) and completed on an mbarrier;
//   * QK^T: a lane owns 4 of the 128 dims; per chunk of CH slots the CH*G
//     partial dot products are reduced across the warp with a butterfly
//     reduce-scatter (CH*G - 1 shuffles instead of 5 per score);
//   * fp32 online softmax (log2 domain) and PV with the probabilities
//     broadcast through shared memory;
//   * the step's new token (position n_prior) is taken from the K/V inputs,
//     patched into the staged tile and written to its page in the pool by
//     the warp that owns that page (the fused append);
//   * warps merge in shared memory, CTAs write (m, l, acc) partials, and the
//     last CTA of each kv head (atomic ticket) merges the splits and stores
//     the output.
//
// Page-id bounds are checked: a bad id is skipped and flags kErrBadPage.
// Every mbarrier wait is bounded (kErrTimeout).
#include "device.cuh"
#include "kernels.h"

namespace gkv {
namespace {

constexpr int kWarps = 4;       // consumer warps per CTA, each an independent pipeline
constexpr int kStages = 3;      // TMA stages per warp
constexpr int kTileBytes = kPageSlots * kHeadDim * 2;  // one (page, head) tile: 4 KiB
constexpr int kStageBytes = 2 * kTileBytes;            // K + V
constexpr int kTileRegion = kWarps * kStages * kStageBytes;
constexpr int kSmemBytes = kTileRegion + kWarps * kStages * 8 + kWarps * 32 * 4;
static_assert(kWarps * 32 == kHeadDim, "the merge maps one thread to one head dim");
static_assert(kWarps * 8 * (kHeadDim + 2) * 4 <= kTileRegion, "merge buffers reuse the tiles");

struct DecodeParams {
    const uint16_t* q;
    const uint16_t* k_new;
    const uint16_t* v_new;
    uint16_t* k_base;
    uint16_t* v_base;
    int2* table;
    void* out;
    float* part_acc;
    float2* part_ml;
    uint32_t* counters;
    uint32_t* err;
    int32_t out_dtype;
    int32_t n_kv_heads;
    int32_t pool_pages;
    int32_t n_prior;
    int32_t total;
    int32_t n_pages;
    int32_t n_splits;
    int32_t pages_per_split;
    int32_t new_first;
    int32_t new_n;
    float qscale;  // softmax scale * log2(e)
    int2 new_ids[kMaxNewPagesPerLaunch];
};

__device__ __forceinline__ int2 page_entry(const DecodeParams& a, int lp) {
    const int r = lp - a.new_first;
    if (r >= 0 && r < a.new_n) return a.new_ids[r];
    return a.table[lp];
}

__device__ __forceinline__ bool entry_ok(const DecodeParams& a, int2 e) {
    return e.x >= 0 && e.x < a.pool_pages && e.y >= 0 && e.y < a.pool_pages;
}

// Butterfly reduce-scatter of NV per-lane partials (NV = 16 or 32): afterwards
// lane l holds the full warp sum of value index (l >> (5 - log2 NV)).
template <int NV>
__device__ __forceinline__ float reduce_scatter(float (&v)[NV], int lane) {
    int n = NV;
#pragma unroll
    for (int mask = 16; mask >= 1; mask >>= 1) {
        if (n > 1) {
            const bool upper = (lane & mask) != 0;
#pragma unroll
            for (int i = 0; i < NV / 2; ++i) {
                if (i < n / 2) {
                    const float send = upper ? v[i] : v[i + n / 2];
                    const float keep = upper ? v[i + n / 2] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, mask);
                }
            }
            n >>= 1;
        } else {
            v[0] += __shfl_xor_sync(0xFFFFFFFFu, v[0], mask);
        }
    }
    return v[0];
}

template <int G>
__global__ void __launch_bounds__(kWarps * 32, 2)
    paged_decode_kernel(const __grid_constant__ CUtensorMap k_map,
                        const __grid_constant__ CUtensorMap v_map, const DecodeParams a) {
    constexpr int CH = (32 / G) < kPageSlots ? (32 / G) : kPageSlots;  // slots per chunk
    constexpr int NV = CH * G;                                         // 16 or 32
    constexpr int LOG_NV = NV == 32 ? 5 : 4;
    constexpr int SH = 5 - LOG_NV;          // lane l holds value index l >> SH
    constexpr int LOG_G = G == 1 ? 0 : G == 2 ? 1 : G == 4 ? 2 : 3;
    constexpr int SMASK0 = 1 << (SH + LOG_G);  // first lane mask spanning the slot bits

    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kTileRegion);
    float* pbuf_all = reinterpret_cast<float*>(bars + kWarps * kStages);
    __shared__ uint32_t s_ticket;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int h = blockIdx.y;
    const int split = blockIdx.x;
    const int Hkv = a.n_kv_heads;

    uint8_t* my_tiles = smem + warp * kStages * kStageBytes;
    uint64_t* my_bars = bars + warp * kStages;
    float* pbuf = pbuf_all + warp * 32;

    const int p0 = split * a.pages_per_split;
    const int p1 = min(a.n_pages, p0 + a.pages_per_split);
    const int first = p0 + warp;
    const int cnt = first < p1 ? (p1 - first + kWarps - 1) / kWarps : 0;

    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < kStages; ++s) mbar_init(&my_bars[s], 1);
        fence_mbar_init();
    }
    __syncwarp();

    const uint64_t policy = l2_policy_evict_first();
    auto issue = [&](int k) {  // lane 0: stage page `k` of this warp
        const int lp = first + k * kWarps;
        const int2 e = page_entry(a, lp);
        uint64_t* bar = &my_bars[k % kStages];
        uint8_t* dst = my_tiles + (k % kStages) * kStageBytes;
        fence_proxy_async_smem();
        if (entry_ok(a, e)) {
            mbar_arrive_expect_tx(bar, kStageBytes);
            tma_load_3d(dst, &k_map, bar, 0, h, e.x * kPageSlots, policy);
            tma_load_3d(dst + kTileBytes, &v_map, bar, 0, h, e.y * kPageSlots, policy);
        } else {
            atomicOr(a.err, kErrBadPage);
            mbar_arrive(bar);
        }
    };

    if (lane == 0) {
        const int pre = cnt < kStages ? cnt : kStages;
        for (int k = 0; k < pre; ++k) issue(k);
    }

    // This lane's 4 dims of each grouped query head, pre-scaled to log2 units.
    float qf[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const uint2 raw =
            *reinterpret_cast<const uint2*>(a.q + (size_t)(h * G + g) * kHeadDim + lane * 4);
        qf[g][0] = bf16_lo(raw.x) * a.qscale;
        qf[g][1] = bf16_hi(raw.x) * a.qscale;
        qf[g][2] = bf16_lo(raw.y) * a.qscale;
        qf[g][3] = bf16_hi(raw.y) * a.qscale;
    }

    float m[G], l[G], acc[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
        acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;
    }

    const int my_v = lane >> SH;
    const int my_s = my_v / G;
    const int my_g = my_v % G;
    bool timed_out = false;
    int consumed = 0;

    for (int k = 0; k < cnt; ++k) {
        const int st = k % kStages;
        const uint32_t parity = (k / kStages) & 1;
        const int lp = first + k * kWarps;
        const int2 e = page_entry(a, lp);
        const bool ok = entry_ok(a, e);
        if (!mbar_wait_bounded(&my_bars[st], parity)) {
            timed_out = true;
            break;
        }
        consumed = k + 1;
        uint16_t* kt = reinterpret_cast<uint16_t*>(my_tiles + st * kStageBytes);
        uint16_t* vt = kt + kPageSlots * kHeadDim;
        const int base = lp * kPageSlots;
        const int nvalid = min(kPageSlots, a.total - base);

        // Fused append: the step's token lands in this page.
        if (a.k_new != nullptr && a.n_prior >= base && a.n_prior < base + kPageSlots) {
            const int slot = a.n_prior - base;
            const uint2 kk = *reinterpret_cast<const uint2*>(a.k_new + (size_t)h * kHeadDim + lane * 4);
            const uint2 vv = *reinterpret_cast<const uint2*>(a.v_new + (size_t)h * kHeadDim + lane * 4);
            *reinterpret_cast<uint2*>(kt + slot * kHeadDim + lane * 4) = kk;
            *reinterpret_cast<uint2*>(vt + slot * kHeadDim + lane * 4) = vv;
            if (ok) {
                const size_t row = ((size_t)slot * Hkv + h) * kHeadDim + lane * 4;
                *reinterpret_cast<uint2*>(a.k_base + (size_t)e.x * kPageSlots * Hkv * kHeadDim + row) = kk;
                *reinterpret_cast<uint2*>(a.v_base + (size_t)e.y * kPageSlots * Hkv * kHeadDim + row) = vv;
            }
            __syncwarp();
        }

        if (ok) {
#pragma unroll
            for (int c = 0; c < kPageSlots / CH; ++c) {
                const int s0 = c * CH;
                if (s0 >= nvalid) break;
                float part[NV];
#pragma unroll
                for (int s = 0; s < CH; ++s) {
                    const uint2 raw = *reinterpret_cast<const uint2*>(kt + (s0 + s) * kHeadDim + lane * 4);
                    const float k0 = bf16_lo(raw.x), k1 = bf16_hi(raw.x);
                    const float k2 = bf16_lo(raw.y), k3 = bf16_hi(raw.y);
#pragma unroll
                    for (int g = 0; g < G; ++g)
                        part[s * G + g] = fmaf(qf[g][3], k3, fmaf(qf[g][2], k2, fmaf(qf[g][1], k1, qf[g][0] * k0)));
                }
                float sc = reduce_scatter<NV>(part, lane);
                if (s0 + my_s >= nvalid) sc = -INFINITY;

                float cmax = sc;
#pragma unroll
                for (int mask = SMASK0; mask <= 16; mask <<= 1)
                    cmax = fmaxf(cmax, __shfl_xor_sync(0xFFFFFFFFu, cmax, mask));
                float mnew[G];
                float m_own = 0.f;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    mnew[g] = fmaxf(m[g], __shfl_sync(0xFFFFFFFFu, cmax, g << SH));
                    if (g == my_g) m_own = mnew[g];
                }
                const float p = (sc == -INFINITY) ? 0.f : exp2_approx(sc - m_own);
                float psum = p;
#pragma unroll
                for (int mask = SMASK0; mask <= 16; mask <<= 1)
                    psum += __shfl_xor_sync(0xFFFFFFFFu, psum, mask);
                if ((lane & ((1 << SH) - 1)) == 0) pbuf[my_v] = p;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float alpha = (mnew[g] == -INFINITY) ? 1.f : exp2_approx(m[g] - mnew[g]);
                    l[g] = l[g] * alpha + __shfl_sync(0xFFFFFFFFu, psum, g << SH);
                    acc[g][0] *= alpha;
                    acc[g][1] *= alpha;
                    acc[g][2] *= alpha;
                    acc[g][3] *= alpha;
                    m[g] = mnew[g];
                }
                __syncwarp();
#pragma unroll
                for (int s = 0; s < CH; ++s) {
                    if (s0 + s < nvalid) {
                        const uint2 raw = *reinterpret_cast<const uint2*>(vt + (s0 + s) * kHeadDim + lane * 4);
                        const float v0 = bf16_lo(raw.x), v1 = bf16_hi(raw.x);
                        const float v2 = bf16_lo(raw.y), v3 = bf16_hi(raw.y);
#pragma unroll
                        for (int g = 0; g < G; ++g) {
                            const float pg = pbuf[s * G + g];
                            acc[g][0] = fmaf(pg, v0, acc[g][0]);
                            acc[g][1] = fmaf(pg, v1, acc[g][1]);
                            acc[g][2] = fmaf(pg, v2, acc[g][2]);
                            acc[g][3] = fmaf(pg, v3, acc[g][3]);
                        }
                    }
                }
                __syncwarp();
            }
        }
        __syncwarp();
        if (lane == 0 && k + kStages < cnt) issue(k + kStages);
    }

    if (timed_out) {
        // Drain this warp's copies still in flight (bounded) before exiting.
        if (lane == 0) atomicOr(a.err, kErrTimeout);
        const int issued = cnt < consumed + kStages ? cnt : consumed + kStages;
        for (int k = consumed; k < issued; ++k)
            (void)mbar_wait_bounded(&my_bars[k % kStages], (k / kStages) & 1);
    }

    // ---- merge the warps of this CTA -----------------------------------
    __syncthreads();
    float* w_acc = reinterpret_cast<float*>(smem);  // [kWarps][G][128]
    float* w_m = w_acc + kWarps * G * kHeadDim;     // [kWarps][G]
    float* w_l = w_m + kWarps * G;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        *reinterpret_cast<float4*>(&w_acc[(warp * G + g) * kHeadDim + lane * 4]) =
            make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
        if (lane == 0) {
            w_m[warp * G + g] = m[g];
            w_l[warp * G + g] = l[g];
        }
    }
    __syncthreads();

    const int d = threadIdx.x;  // kWarps * 32 == kHeadDim threads: one dim each
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, w_m[w * G + g]);
        const float Ms = (M == -INFINITY) ? 0.f : M;
        float L = 0.f, A = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float f = exp2_approx(w_m[w * G + g] - Ms);
            L = fmaf(w_l[w * G + g], f, L);
            A = fmaf(w_acc[(w * G + g) * kHeadDim + d], f, A);
        }
        const int hq = h * G + g;
        if (a.n_splits == 1) {
            store_out(a.out, (size_t)hq * kHeadDim + d, A / L, a.out_dtype);
        } else {
            const size_t row = (size_t)hq * a.n_splits + split;
            a.part_acc[row * kHeadDim + d] = A;
            if (d == 0) a.part_ml[row] = make_float2(M, L);
        }
    }
    if (a.n_splits == 1) return;

    // ---- last CTA of this kv head merges the splits -----------------------
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_ticket = atomicAdd(&a.counters[h], 1u);
    __syncthreads();
    if (s_ticket != (uint32_t)(a.n_splits - 1)) return;
    __threadfence();
#pragma unroll 1
    for (int g = 0; g < G; ++g) {
        const int hq = h * G + g;
        const float2* ml = a.part_ml + (size_t)hq * a.n_splits;
        const float* pa = a.part_acc + (size_t)hq * a.n_splits * kHeadDim + d;
        float M = -INFINITY;
        for (int s = 0; s < a.n_splits; ++s) M = fmaxf(M, __ldcg(&ml[s].x));
        const float Ms = (M == -INFINITY) ? 0.f : M;
        float L = 0.f, A = 0.f;
        for (int s = 0; s < a.n_splits; ++s) {
            const float2 e = __ldcg(&ml[s]);
            const float f = exp2_approx(e.x - Ms);
            L = fmaf(e.y, f, L);
            A = fmaf(__ldcg(&pa[(size_t)s * kHeadDim]), f, A);
        }
        store_out(a.out, (size_t)hq * kHeadDim + d, A / L, a.out_dtype);
    }
    if (threadIdx.x == 0) a.counters[h] = 0u;  // ready for the next launch
}

template <int G>
cudaError_t launch_g(const CUtensorMap& km, const CUtensorMap& vm, const DecodeParams& p,
                     dim3 grid, cudaStream_t stream) {
    // The shared-memory opt-in is per device; remember which devices have it.
    static unsigned long long configured = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 64 || !(configured & (1ull << dev))) {
        e = cudaFuncSetAttribute(paged_decode_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kSmemBytes);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured |= 1ull << dev;
    }
    paged_decode_kernel<G><<<grid, kWarps * 32, kSmemBytes, stream>>>(km, vm, p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_decode(const PoolView& pool, const CUtensorMap& k_map, const CUtensorMap& v_map,
                          int2* table, const NewPages& np, const Scratch& scratch,
                          const DecodeLaunch& d, int num_sms, cudaStream_t stream) {
    const int Hkv = pool.n_kv_heads;
    const int G = d.n_q_heads / Hkv;
    DecodeParams p;
    p.q = d.q;
    p.k_new = d.k_new;
    p.v_new = d.v_new;
    p.k_base = pool.k_base;
    p.v_base = pool.v_base;
    p.table = table;
    p.out = d.out;
    p.part_acc = scratch.part_acc;
    p.part_ml = scratch.part_ml;
    p.counters = scratch.counters;
    p.err = scratch.err;
    p.out_dtype = d.out_dtype;
    p.n_kv_heads = Hkv;
    p.pool_pages = pool.pool_pages;
    p.n_prior = d.n_prior;
    p.total = d.total;
    p.n_pages = d.n_pages;
    p.qscale = d.scale * 1.4426950408889634f;
    p.new_first = np.first;
    p.new_n = np.n;
    for (int i = 0; i < np.n; ++i) p.new_ids[i] = np.ids[i];

    // Splits: two resident CTAs per SM over all kv heads, at least one page
    // per warp, and within the partials capacity.
    int n_splits = d.n_splits;
    if (n_splits <= 0) {
        n_splits = (2 * num_sms + Hkv - 1) / Hkv;
        const int by_pages = (d.n_pages + kWarps - 1) / kWarps;
        if (n_splits > by_pages) n_splits = by_pages;
    }
    if (n_splits * d.n_q_heads > kMaxPartialRows) n_splits = kMaxPartialRows / d.n_q_heads;
    if (n_splits < 1) n_splits = 1;
    int pps = (d.n_pages + n_splits - 1) / n_splits;
    if (pps < 1) pps = 1;
    n_splits = (d.n_pages + pps - 1) / pps;  // no empty splits
    if (n_splits < 1) n_splits = 1;
    p.n_splits = n_splits;
    p.pages_per_split = pps;

    dim3 grid(n_splits, Hkv);
    switch (G) {
        case 1: return launch_g<1>(k_map, v_map, p, grid, stream);
        case 2: return launch_g<2>(k_map, v_map, p, grid, stream);
        case 4: return launch_g<4>(k_map, v_map, p, grid, stream);
        case 8: return launch_g<8>(k_map, v_map, p, grid, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace gkv
