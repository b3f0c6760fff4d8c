// decode.cu — fused paged-attention decode step for sm_100a.
//
// One step does what the reference spreads over 2*Hkv synchronous
// cudaMemcpy calls, a cudaMalloc/H2D/cudaFree of the page ids and a
// warp-per-head kernel with a serial page loop (src/core/page_attention.cpp:
// 104-139, src/backend/cuda/attention.cu:401-580). Two launches:
//
// paged_decode_kernel — one CTA per SM, each owning a contiguous range of
// logical pages (split-K over the context):
//   * a producer warp stages pages by TMA (no multicast): per page, per
//     kv head, per 64-dim half one box {64 dims, 1 head, 16 slots} of the
//     pool's 3-D map, 128-byte swizzle; a stage holds 8 (page, head) tiles of
//     K and of V (64 KiB), three stages in flight; full/empty mbarriers;
//   * 8 consumer warps, warp w on head (w % Hkv) of page (w / Hkv) of each
//     stage, so all heads of a page are fetched together (whole page
//     regions, DRAM-friendly) and every KV byte is read from HBM once;
//   * per (page, head): S^T = K Q^T with mma.sync m16n8k16 (bf16 in, fp32
//     accumulate; M = 16 slots, N = the G grouped query heads padded to 8,
//     K = 128 dims in 8 steps, operands by ldmatrix from the swizzled tile),
//     fp32 online softmax per head with 3-step warp shuffles (log2 domain),
//     then O^T += V^T P^T (M = 16 dims x 8 tiles, K = 16 slots, ldmatrix.trans);
//   * the step's new token (position n_prior) is taken from the K/V inputs,
//     patched into the staged tile and written to its page in the pool by the
//     warp that owns that (page, head): the fused append;
//   * warps merge in shared memory; each CTA writes an (m, l, acc) partial per
//     query head.
// paged_decode_combine_kernel — launched with programmatic dependent launch,
// one CTA per query head merges the splits and stores the output.
//
// Page ids are bounds-checked (a bad id is skipped and sets kErrBadPage);
// every mbarrier wait is bounded (kErrTimeout).
#include <cstdlib>

#include <algorithm>
#include <atomic>

#include "device.cuh"
#include "kernels.h"
#include "qk_rope.cuh"

namespace gkv {
namespace {

// A stage holds kConsumerWarps (page, head) tiles of K and of V, one per
// consumer warp; a producer warp keeps the ring of stages filled.
constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
#ifdef GKV_PROBE_STAGES
constexpr int kStages = GKV_PROBE_STAGES;
#else
constexpr int kStages = 3;
#endif
constexpr uint32_t kTileHalf = kPageSlots * 128;     // 16 slots x 128 B (64 dims): 2 KiB
constexpr uint32_t kTile = 2 * kTileHalf;            // one (page, head) K or V tile: 4 KiB
constexpr uint32_t kStageKV = kConsumerWarps * kTile;  // 32 KiB of K (or V) per stage
constexpr uint32_t kStageBytes = 2 * kStageKV;        // 64 KiB
constexpr uint32_t kOffBar = kStages * kStageBytes;
constexpr uint32_t kOffP = kOffBar + 2 * kStages * 8;            // full barriers, slot counters; then per-warp P^T hi/lo buffers
constexpr int kMaxSplitPages = 1024;                              // page ids cached per CTA
constexpr uint32_t kOffIds = kOffP + kConsumerWarps * 512;
constexpr uint32_t kSmemBytes = kOffIds + kMaxSplitPages * 8 + 1024;  // + alignment slack
static_assert(kConsumerWarps * 36 * 32 * 4 <= kStages * kStageBytes, "merge buffers fit");

struct DecodeParams {
    const uint16_t* q;
    const uint16_t* k_new;
    const uint16_t* v_new;
    uint16_t* k_base;
    uint16_t* v_base;
    int2* table;
    float* part_acc;   // [n_splits][Hq][128]
    float2* part_ml;   // [n_splits][Hq]
    uint32_t* err;
    const uint32_t* done;  // non-null: wait until *done reaches done_expect before reading the table or pages
    uint32_t done_expect;
    // Split merge fused into this grid (null: the combine kernel merges).
    // merge[0] counts arriving CTAs, merge[1] finished mergers; both zero
    // between launches. The last n_merge CTAs to arrive merge the splits.
    uint32_t* merge;
    void* out;
    int32_t out_dtype;
    uint32_t* done_post;  // non-null (with merge): the last merger stores done_seq here
    uint32_t done_seq;
    uint32_t* arrive;     // non-null (combine kernel merges): count of CTAs whose partials are written
    int32_t late_trigger;  // 1: release the next launch only after this grid's wait for its predecessor
    int32_t l2_prefetch_stages;  // stages past the ring brought into L2 while the ring is full
    int32_t n_kv_heads;
    int32_t group;     // G = Hq / Hkv
    int32_t pool_pages;
    int32_t n_prior;
    int32_t total;
    int32_t n_pages;
    int32_t pages_per_split;
    int32_t pages_per_stage;  // P = 8 / Hkv (floored)
    int32_t new_first;
    int32_t new_n;
    int32_t qk_on;  // 1: q / k_new are pre-norm projections: QK-norm + RoPE here (position n_prior)
    QkNorm qk;
    const DeviceStep* step;  // non-null: the step fields above come from here (captured steps)
    int32_t inputs_ready;    // 1: previous launch is another layer's combine of the same step (see kernel)
    float qscale;  // softmax scale * log2(e)
#ifdef GKV_PROBE_TIMELINE
    int32_t probe_slot;
#endif
    int2 new_ids[kMaxNewPagesPerLaunch];
};

// The step fields, from the launch parameters or (captured steps) from the
// device step block, which a copy before the step wrote: safe to read before
// griddepcontrol.wait.
struct StepFields {
    int n_prior, total, n_pages, pages_per_split, new_first, new_n;
    int2 new0;
};

__device__ __forceinline__ StepFields step_fields(const DecodeParams& a) {
    if (a.step) {
        const DeviceStep* s = a.step;
        return {__ldg(&s->n_prior), __ldg(&s->total), __ldg(&s->n_pages), __ldg(&s->pages_per_split),
                __ldg(&s->new_first), __ldg(&s->new_n), __ldg(&s->new_id)};
    }
    return {a.n_prior, a.total, a.n_pages, a.pages_per_split, a.new_first, a.new_n, a.new_ids[0]};
}

__device__ __forceinline__ int2 page_entry(const DecodeParams& a, const StepFields& sf, int lp) {
    const int r = lp - sf.new_first;
    if (r == 0 && sf.new_n > 0) return sf.new0;
    if (r > 0 && r < sf.new_n) return a.new_ids[r];  // more than one new page: never a captured step
    return a.table[lp];
}

__device__ __forceinline__ bool entry_ok(const DecodeParams& a, int2 e) {
    return e.x >= 0 && e.x < a.pool_pages && e.y >= 0 && e.y < a.pool_pages;
}

// Byte offset of (slot row r, 16-byte chunk c of the 128 dims) inside a
// (page, head) tile stored as two 128-byte-swizzled 64-dim halves of
// 16 rows x 128 B, `hs` bytes apart (kTileHalf when a tile is contiguous,
// Hkv * kTileHalf when a page's heads are interleaved half by half).
__device__ __forceinline__ uint32_t tile_off(int r, int c, uint32_t hs) {
    return (uint32_t)((c >> 3) * hs + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// Wait (bounded) until the completion word of the table reaches `expect`:
// every earlier decode step of this table has completed, so its appended
// rows and published table entries can be read. Acquire at GPU scope, then
// a proxy fence so that the TMA (async proxy) reads come after it.
__device__ __forceinline__ void wait_done(const uint32_t* done, uint32_t expect, uint32_t* err) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(done) : "memory");
    if ((int32_t)(v - expect) < 0) {
        const uint64_t t0 = global_timer_ns();
        for (uint32_t i = 0;; ++i) {
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(done) : "memory");
            if ((int32_t)(v - expect) >= 0) break;
            if ((i & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
                atomicOr(err, kErrTimeout);
                break;
            }
        }
    }
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}


// One merge unit of the fused split merge: query head h, 64-dim half hf.
// 18 groups of 16 threads; group gi folds splits gi, gi + 18, ... with an
// online rescale (each thread 4 dims, float4 loads from L2: the partials are
// this grid's own stores), then group 0 folds the 18 group results from
// shared memory and stores the output.
constexpr int kMergeGroups = kThreads / 16;  // 18
constexpr int kMergeBatch = 9;               // splits per group in flight at once
static_assert(kMergeGroups * 68 * 4 <= kStages * kStageBytes, "merge buffers fit");

__device__ __noinline__ void merge_unit(const float* part_acc, const float2* part_ml, void* out, int out_dtype,
                                       float* sbuf, int n_splits, int Hq, int h, int hf) {
    const int gi = threadIdx.x >> 4, li = threadIdx.x & 15;
    const int d = hf * 64 + li * 4;
    float M = -INFINITY, L = 0.f;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int b = 0; b * kMergeBatch * kMergeGroups < n_splits; ++b) {
        float2 ml[kMergeBatch];
        float4 av[kMergeBatch];
#pragma unroll
        for (int i = 0; i < kMergeBatch; ++i) {
            const int sp = gi + (b * kMergeBatch + i) * kMergeGroups;
            const bool in = sp < n_splits;
            const size_t row = (size_t)sp * Hq + h;
            ml[i] = in ? __ldcg(part_ml + row) : make_float2(-INFINITY, 0.f);
            av[i] = in ? __ldcg(reinterpret_cast<const float4*>(part_acc + row * kHeadDim + d))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float mb = M;
#pragma unroll
        for (int i = 0; i < kMergeBatch; ++i) mb = fmaxf(mb, ml[i].x);
        const float ms = mb == -INFINITY ? 0.f : mb;
        const float r = exp2_approx(M - ms);
        L *= r;
        A.x *= r; A.y *= r; A.z *= r; A.w *= r;
#pragma unroll
        for (int i = 0; i < kMergeBatch; ++i) {
            const float f = exp2_approx(ml[i].x - ms);
            L = fmaf(ml[i].y, f, L);
            A.x = fmaf(av[i].x, f, A.x);
            A.y = fmaf(av[i].y, f, A.y);
            A.z = fmaf(av[i].z, f, A.z);
            A.w = fmaf(av[i].w, f, A.w);
        }
        M = mb;
        if ((li & 7) == 0) {  // two 128-byte lines per (split, head, half), read by this group alone
#pragma unroll
            for (int i = 0; i < kMergeBatch; ++i) {
                const int sp = gi + (b * kMergeBatch + i) * kMergeGroups;
                if (sp < n_splits) l2_discard_line(part_acc + ((size_t)sp * Hq + h) * kHeadDim + d);
            }
        }
    }
    // sbuf: [group][m, l, 2 spare, 64 dims] (68 floats: 16-byte aligned rows)
    float* mine = sbuf + gi * 68;
    if (li == 0) {
        mine[0] = M;
        mine[1] = L;
    }
    *reinterpret_cast<float4*>(mine + 4 + li * 4) = A;
    __syncthreads();
    if (gi == 0) {
        float Mt = -INFINITY;
#pragma unroll
        for (int k = 0; k < kMergeGroups; ++k) Mt = fmaxf(Mt, sbuf[k * 68]);
        const float ms = Mt == -INFINITY ? 0.f : Mt;
        float Lt = 0.f;
        float4 At = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < kMergeGroups; ++k) {
            const float* o = sbuf + k * 68;
            const float f = exp2_approx(o[0] - ms);
            const float4 v = *reinterpret_cast<const float4*>(o + 4 + li * 4);
            Lt = fmaf(o[1], f, Lt);
            At.x = fmaf(v.x, f, At.x);
            At.y = fmaf(v.y, f, At.y);
            At.z = fmaf(v.z, f, At.z);
            At.w = fmaf(v.w, f, At.w);
        }
        const size_t base = (size_t)h * kHeadDim + d;
        store_out(out, base + 0, At.x / Lt, out_dtype);
        store_out(out, base + 1, At.y / Lt, out_dtype);
        store_out(out, base + 2, At.z / Lt, out_dtype);
        store_out(out, base + 3, At.w / Lt, out_dtype);
    }
    __syncthreads();
}

#ifdef GKV_PROBE_TIMELINE
__device__ unsigned long long g_probe_tl[8 * 4096 * 8];
__device__ unsigned long long g_probe_st[8 * 2048 * 16];  // stage-ready times seen by consumer warp 0
#define PROBE_T(k) \
    if (threadIdx.x == 0) g_probe_tl[(a.probe_slot * 4096 + blockIdx.x) * 8 + (k)] = global_timer_ns();
#else
#define PROBE_T(k)
#endif

// kPageBox: one TMA box {64 dims, 16 slots, Hkv heads} per page and 64-dim
// half (4 copies per page; the stage holds a page as [half][head][slot]);
// otherwise one box {64 dims, 1 head, 16 slots} per (page, head, half) (32
// copies per page at Hkv = 8; the stage holds [head][half][slot]).
template <bool kPageBox>
__global__ void __launch_bounds__(kThreads, 2)  // 96 registers: a combine CTA fits beside it
    paged_decode_kernel(const __grid_constant__ CUtensorMap k_map, const __grid_constant__ CUtensorMap v_map,
                        const DecodeParams a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint64_t* empty = full + kStages;

    PROBE_T(0);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int split = blockIdx.x;
    const int Hkv = a.n_kv_heads;
    const int G = a.group;
    const int P = a.pages_per_stage;
    const StepFields sf = step_fields(a);
    const int p0 = split * sf.pages_per_split;
    const int p1 = min(sf.n_pages, p0 + sf.pages_per_split);
    const int n_stages = p1 > p0 ? (p1 - p0 + P - 1) / P : 0;

    // Programmatic dependent launch: the split-combine kernel that follows may
    // be scheduled now (it waits for this grid's completion itself).
    if (!a.late_trigger) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // This grid may start before the previous decode step of the same table
    // has completed (the combine kernels release their successor at entry):
    // its table entries and appended rows are read only once its completion
    // word says so.
    if (a.done != nullptr) {
        if (threadIdx.x == 0) wait_done(a.done, a.done_expect, a.err);
        __syncthreads();
    }

    // Publish this step's new block-table entries (this launch reads them
    // from its parameters; later launches read the table).
    if (split == 0 && (int)threadIdx.x < sf.new_n)
        a.table[sf.new_first + threadIdx.x] = threadIdx.x == 0 ? sf.new0 : a.new_ids[threadIdx.x];

    // Stage i of this split: its np pages, every kv head, both 64-dim halves of
    // K and V, one TMA box {64, 1, 16} each, completing on full[i % kStages].
    const uint64_t pol = l2_policy_evict_first();
    auto issue_stage = [&](int i, auto&& entry_of) {
        const int st = i % kStages;
        uint8_t* sk = smem + st * kStageBytes;
        uint8_t* sv = sk + kStageKV;
        const int np = min(P, p1 - (p0 + i * P));
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&full[st], (uint32_t)(np * Hkv) * 2u * kTile);
        for (int pi = 0; pi < np; ++pi) {
            int2 e = entry_of(i * P + pi);
            if (e.x < 0) e = make_int2(0, 0);  // loaded but never used (the consumer skips it)
            if constexpr (kPageBox) {
                const uint32_t t = (uint32_t)(pi * Hkv) * kTile;
                for (int hf = 0; hf < 2; ++hf) {
                    const uint32_t o = t + (uint32_t)(hf * Hkv) * kTileHalf;
                    tma_load_3d(sk + o, &k_map, &full[st], hf * 64, e.x * kPageSlots, 0, pol);
                    tma_load_3d(sv + o, &v_map, &full[st], hf * 64, e.y * kPageSlots, 0, pol);
                }
            } else {
                for (int h = 0; h < Hkv; ++h) {
                    const uint32_t t = (uint32_t)(pi * Hkv + h) * kTile;
                    for (int hf = 0; hf < 2; ++hf) {
                        tma_load_3d(sk + t + hf * kTileHalf, &k_map, &full[st], hf * 64, h, e.x * kPageSlots, pol);
                        tma_load_3d(sv + t + hf * kTileHalf, &v_map, &full[st], hf * 64, h, e.y * kPageSlots, pol);
                    }
                }
            }
        }
    };
    // Stage i's pages into L2 (no shared memory, no barrier).
    auto prefetch_stage = [&](int i, auto&& entry_of) {
        const int np = min(P, p1 - (p0 + i * P));
        for (int pi = 0; pi < np; ++pi) {
            const int2 e = entry_of(i * P + pi);
            if (e.x < 0) continue;
            if constexpr (kPageBox) {
                for (int hf = 0; hf < 2; ++hf) {
                    tma_prefetch_3d(&k_map, hf * 64, e.x * kPageSlots, 0);
                    tma_prefetch_3d(&v_map, hf * 64, e.y * kPageSlots, 0);
                }
            } else {
                for (int h = 0; h < Hkv; ++h)
                    for (int hf = 0; hf < 2; ++hf) {
                        tma_prefetch_3d(&k_map, hf * 64, h, e.x * kPageSlots);
                        tma_prefetch_3d(&v_map, hf * 64, h, e.y * kPageSlots);
                    }
            }
        }
    };
    // A page id, bounds-checked: a bad id becomes {-1, -1} (loaded as page 0,
    // skipped by the consumer) and sets the error bit.
    auto checked = [&](int i) {
        int2 e = page_entry(a, sf, p0 + i);
        if (!entry_ok(a, e)) {
            atomicOr(a.err, kErrBadPage);
            e = make_int2(-1, -1);
        }
        return e;
    };

    int2* ids = reinterpret_cast<int2*>(smem + kOffIds);
    if (threadIdx.x == kConsumerWarps * 32) {
        // Producer: barriers, then stage 0 straight from the table while the
        // other threads cache the split's ids (saves one table round trip
        // on the first data).
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_mbar_init();
        if (a.done != nullptr) asm volatile("fence.proxy.async.global;" ::: "memory");
        if (n_stages > 0) issue_stage(0, checked);
    }
    for (int i = threadIdx.x; i < p1 - p0; i += kThreads) ids[i] = checked(i);
    __syncthreads();
    PROBE_T(1);

    if (warp == kConsumerWarps) {
        // ---------------- producer ----------------
        if (lane == 0) {
            for (int i = 1; i < n_stages; ++i) {
                const int st = i % kStages;
                if (i >= kStages && !mbar_wait_bounded(&empty[st], ((i / kStages) - 1) & 1))
                    atomicOr(a.err, kErrTimeout);
                issue_stage(i, [&](int k) { return ids[k]; });
                if (i == kStages - 1) {
                    // The ring is full. Until the consumers may start (their
                    // griddepcontrol.wait, which on the per-layer path waits
                    // for the previous kernels to complete) nothing frees
                    // it: bring the next stages' pages into L2 meanwhile, so
                    // that their loads later come from L2 rather than HBM.
                    const int pf_end = min(n_stages, kStages + a.l2_prefetch_stages);
                    for (int j = kStages; j < pf_end; ++j) prefetch_stage(j, [&](int k) { return ids[k]; });
                }
            }
        }
    } else {
        // ---------------- consumers ----------------
        const int head = warp % Hkv;
        const int pslot = warp / Hkv;           // page within a stage
        const uint32_t hs = kPageBox ? (uint32_t)Hkv * kTileHalf : kTileHalf;  // 64-dim halves apart
        const bool active = pslot < P;
        const int g = lane >> 2;                // fragment row group
        const int t = lane & 3;                 // fragment column pair
        uint8_t* pbuf = smem + kOffP + warp * 512;  // P^T staging: hi and lo [8 heads][16 slots] bf16

        // This launch may overlap the tail of the previous kernel on the stream
        // (programmatic dependent launch): the page stream above reads only
        // cached pages, but Q and the new K/V row are that kernel's outputs.
        // QK-norm weights and this position's RoPE rows are not the previous
        // kernel's outputs: they are loaded before the wait, whose latency
        // covers theirs.
        RowParamsG8 rq;
        if (a.qk_on) {
            const size_t pos = (size_t)sf.n_prior * kHeadDim;
            rq = load_row_params_g8(a.qk.q_w, a.qk.cos + pos, a.qk.sin + pos, lane & 7);
        }
        // Inside a multi-layer step whose layers are distinct, the layers
        // after the first read inputs that were complete before the step's
        // first launch: no wait here (one thread waits at the end instead, so
        // that this grid still completes after the previous kernel).
        if (!a.inputs_ready) asm volatile("griddepcontrol.wait;" ::: "memory");
        if (a.late_trigger) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        PROBE_T(5);
        // B operand of S^T = K Q^T: Q^T fragments (k = dims, n = grouped query head).
        uint32_t qb[8][2];
        if (a.qk_on) {
            // QK-norm + RoPE of this warp's G query rows, each through a
            // 256-byte staging row (the warp's P buffer, idle until the first
            // page) from which each lane takes its fragment.
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) qb[kk][0] = qb[kk][1] = 0u;
            if (active) {
                // One query row per 8-lane group, four rows at once
                // (norm_rope_row_g8), then each row through a staging row of
                // the warp's 512-byte P buffer (idle until the first page),
                // two at a time, from which each lane takes its fragment.
                const int grp = lane >> 3, j = lane & 7;
                const size_t pos = (size_t)sf.n_prior * kHeadDim;
                uint16_t* stage = reinterpret_cast<uint16_t*>(pbuf);
#pragma unroll
                for (int b0 = 0; b0 < 8; b0 += 4) {
                    if (b0 >= G) break;
                    const int n = b0 + grp;
                    const bool row_ok = n < G;
                    const uint16_t* qr = a.q + (size_t)(head * G + (row_ok ? n : 0)) * kHeadDim;
                    float x[4][4];
#pragma unroll
                    for (int it = 0; it < 4; ++it)
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            x[it][k] = __uint_as_float((uint32_t)qr[32 * it + 8 * k + j] << 16);
                    uint16_t o[4][4];
                    norm_rope_row_g8(x, j, rq, a.qk.eps, o);
#pragma unroll
                    for (int half = 0; half < 2; ++half) {  // groups 2 half, 2 half + 1 -> staging rows 0, 1
                        if ((grp >> 1) == half && row_ok) {
#pragma unroll
                            for (int it = 0; it < 4; ++it)
#pragma unroll
                                for (int k = 0; k < 4; ++k) stage[(grp & 1) * kHeadDim + 32 * it + 8 * k + j] = o[it][k];
                        }
                        __syncwarp();
                        const int r0 = b0 + 2 * half;
                        if ((g == r0 || g == r0 + 1) && g < G) {
                            const uint16_t* row = stage + (g - r0) * kHeadDim;
#pragma unroll
                            for (int kk = 0; kk < 8; ++kk) {
                                qb[kk][0] = *reinterpret_cast<const uint32_t*>(row + kk * 16 + 2 * t);
                                qb[kk][1] = *reinterpret_cast<const uint32_t*>(row + kk * 16 + 2 * t + 8);
                            }
                        }
                        __syncwarp();
                    }
                }
            }
        } else {
            const int n = g;
            const bool valid = active && n < G;
            const uint16_t* qr = a.q + (size_t)(head * G + (valid ? n : 0)) * kHeadDim;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                qb[kk][0] = valid ? *reinterpret_cast<const uint32_t*>(qr + kk * 16 + 2 * t) : 0u;
                qb[kk][1] = valid ? *reinterpret_cast<const uint32_t*>(qr + kk * 16 + 2 * t + 8) : 0u;
            }
        }
#ifdef GKV_PROBE_TIMELINE
        asm volatile("" ::"r"(qb[0][0]), "r"(qb[7][1]));
        PROBE_T(6);
#endif
        float acc[8][4];
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // heads 2t, 2t+1

        // ldmatrix row addressing (lane -> matrix mi, row within it).
        const int mi = lane >> 3;
        const int lr = lane & 7;

        for (int i = 0; i < n_stages; ++i) {
            const int st = i % kStages;
            const bool ok_wait = mbar_wait_bounded(&full[st], (i / kStages) & 1);
            if (i == 0) { PROBE_T(2); }
#ifdef GKV_PROBE_TIMELINE
            if (threadIdx.x == 0 && i < 16) g_probe_st[(a.probe_slot * 2048 + blockIdx.x) * 16 + i] = global_timer_ns();
#endif
            if (!ok_wait && lane == 0) atomicOr(a.err, kErrTimeout);
            const int lp = p0 + i * P + pslot;
            const bool have = active && lp < p1 && ok_wait;
            const int2 e = have ? ids[lp - p0] : make_int2(-1, -1);
#ifdef GKV_PROBE_SKIP_COMPUTE
            const bool use = false;  // measurement build: page stream only
            (void)e;
#else
            const bool use = have && e.x >= 0;
#endif
            if (use) {
                uint8_t* kt = smem + st * kStageBytes +
                              (kPageBox ? (uint32_t)(pslot * Hkv) * kTile + (uint32_t)head * kTileHalf
                                        : (uint32_t)(pslot * Hkv + head) * kTile);
                uint8_t* vt = kt + kStageKV;
                const int base = lp * kPageSlots;
                const int nvalid = min(kPageSlots, sf.total - base);
                // Fused append of this step's token.
                if (a.k_new != nullptr && sf.n_prior >= base && sf.n_prior < base + kPageSlots) {
                    const int slot = sf.n_prior - base;
                    uint2 kk;
                    if (a.qk_on) {  // the post-QK-norm, post-RoPE row is what the page holds
                        float xk[4];
                        load_row4(a.k_new + (size_t)head * kHeadDim, lane, xk);
                        const size_t pos = (size_t)sf.n_prior * kHeadDim;
                        const RowParams rp = load_row_params(a.qk.k_w, a.qk.cos + pos, a.qk.sin + pos, lane);
                        uint16_t o[4];
                        norm_rope_row(xk, rp, a.qk.eps, o);
                        uint16_t* stage = reinterpret_cast<uint16_t*>(pbuf);
#pragma unroll
                        for (int it = 0; it < 4; ++it) stage[lane + 32 * it] = o[it];
                        __syncwarp();
                        kk = *reinterpret_cast<const uint2*>(stage + lane * 4);
                        __syncwarp();
                    } else {
                        kk = *reinterpret_cast<const uint2*>(a.k_new + (size_t)head * kHeadDim + lane * 4);
                    }
                    const uint2 vv = *reinterpret_cast<const uint2*>(a.v_new + (size_t)head * kHeadDim + lane * 4);
                    const uint32_t o = tile_off(slot, lane >> 1, hs) + (lane & 1) * 8;
                    *reinterpret_cast<uint2*>(kt + o) = kk;
                    *reinterpret_cast<uint2*>(vt + o) = vv;
                    const size_t row = ((size_t)slot * Hkv + head) * kHeadDim + lane * 4;
                    *reinterpret_cast<uint2*>(a.k_base + (size_t)e.x * kPageSlots * Hkv * kHeadDim + row) = kk;
                    *reinterpret_cast<uint2*>(a.v_base + (size_t)e.y * kPageSlots * Hkv * kHeadDim + row) = vv;
                }
                // Slots past the cache: zero their V rows (0 x NaN would poison the MMA).
                if (nvalid < kPageSlots) {
                    for (int r = nvalid + (lane >> 3); r < kPageSlots; r += 4) {
                        *reinterpret_cast<uint4*>(vt + r * 128 + (lane & 7) * 16) = make_uint4(0, 0, 0, 0);
                        *reinterpret_cast<uint4*>(vt + hs + r * 128 + (lane & 7) * 16) = make_uint4(0, 0, 0, 0);
                    }
                }
                __syncwarp();

                // S^T[slot][head] = K Q^T
                // Two independent accumulation chains (even / odd k-steps).
                float s[4] = {0.f, 0.f, 0.f, 0.f}, s_odd[4] = {0.f, 0.f, 0.f, 0.f};
                const uint32_t ks = smem_addr(kt);
#pragma unroll
                for (int kk = 0; kk < 8; kk += 2) {
                    uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
                    ldsm_x4(ks + tile_off(lr + (mi & 1) * 8, 2 * kk + (mi >> 1), hs), a0, a1, a2, a3);
                    ldsm_x4(ks + tile_off(lr + (mi & 1) * 8, 2 * kk + 2 + (mi >> 1), hs), b0, b1, b2, b3);
                    mma_bf16_16816(s, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
                    mma_bf16_16816(s_odd, b0, b1, b2, b3, qb[kk + 1][0], qb[kk + 1][1]);
                }
#pragma unroll
                for (int i2 = 0; i2 < 4; ++i2) s[i2] += s_odd[i2];
                // s[0]: (slot g, head 2t) s[1]: (g, 2t+1) s[2]: (g+8, 2t) s[3]: (g+8, 2t+1)
                const bool v_lo = g < nvalid, v_hi = g + 8 < nvalid;
                const float s0 = v_lo ? s[0] * a.qscale : -INFINITY;
                const float s1 = v_lo ? s[1] * a.qscale : -INFINITY;
                const float s2 = v_hi ? s[2] * a.qscale : -INFINITY;
                const float s3 = v_hi ? s[3] * a.qscale : -INFINITY;
                float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
#pragma unroll
                for (int m = 4; m <= 16; m <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xFFFFFFFFu, mx0, m));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xFFFFFFFFu, mx1, m));
                }
                const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);  // finite: slot 0 is always valid
                const float al0 = exp2_approx(m0 - mn0), al1 = exp2_approx(m1 - mn1);
                const float p0v = exp2_approx(s0 - mn0), p1v = exp2_approx(s1 - mn1);
                const float p2v = exp2_approx(s2 - mn0), p3v = exp2_approx(s3 - mn1);
                float su0 = p0v + p2v, su1 = p1v + p3v;
#pragma unroll
                for (int m = 4; m <= 16; m <<= 1) {
                    su0 += __shfl_xor_sync(0xFFFFFFFFu, su0, m);
                    su1 += __shfl_xor_sync(0xFFFFFFFFu, su1, m);
                }
                l0 = l0 * al0 + su0;
                l1 = l1 * al1 + su1;
                m0 = mn0;
                m1 = mn1;
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    acc[mt][0] *= al0;
                    acc[mt][1] *= al1;
                    acc[mt][2] *= al0;
                    acc[mt][3] *= al1;
                }
                // P^T staging as bf16 hi + lo (P = hi + lo to ~2^-17 relative), so the
                // PV products keep fp32-level accuracy: pbuf[0|1][head][slot].
                uint16_t* pb = reinterpret_cast<uint16_t*>(pbuf);
                {
                    const float pv[4] = {p0v, p1v, p2v, p3v};
                    const int hh[4] = {2 * t, 2 * t + 1, 2 * t, 2 * t + 1};
                    const int ss[4] = {g, g, g + 8, g + 8};
#pragma unroll
                    for (int i2 = 0; i2 < 4; ++i2) {
                        const __nv_bfloat16 hi = __float2bfloat16_rn(pv[i2]);
                        const __nv_bfloat16 lo = __float2bfloat16_rn(pv[i2] - __bfloat162float(hi));
                        pb[hh[i2] * 16 + ss[i2]] = __bfloat16_as_ushort(hi);
                        pb[128 + hh[i2] * 16 + ss[i2]] = __bfloat16_as_ushort(lo);
                    }
                }
                __syncwarp();
                const uint32_t ph0 = *reinterpret_cast<const uint32_t*>(pb + g * 16 + 2 * t);
                const uint32_t ph1 = *reinterpret_cast<const uint32_t*>(pb + g * 16 + 2 * t + 8);
                const uint32_t pl0 = *reinterpret_cast<const uint32_t*>(pb + 128 + g * 16 + 2 * t);
                const uint32_t pl1 = *reinterpret_cast<const uint32_t*>(pb + 128 + g * 16 + 2 * t + 8);
                const uint32_t vs = smem_addr(vt);
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4_t(vs + tile_off(lr + (mi >> 1) * 8, 2 * mt + (mi & 1), hs), a0, a1, a2, a3);
                    mma_bf16_16816(acc[mt], a0, a1, a2, a3, ph0, ph1);
                    mma_bf16_16816(acc[mt], a0, a1, a2, a3, pl0, pl1);
                }
                fence_proxy_async_smem();  // generic writes above precede the next TMA into this stage
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }

        // Warps that share a kv head (P > 1 pages per stage) merge in
        // registers through shared memory, in fragment order (lane-major,
        // conflict-free); then the warp of page slot 0 holds the CTA's
        // partial for its head.
        if (P > 1) {
            asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32));  // stage buffers are free
            float* frag = reinterpret_cast<float*>(smem);                 // [warp][36][32]
            float* mine = frag + warp * 36 * 32 + lane;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) mine[(mt * 4 + i) * 32] = acc[mt][i];
            mine[32 * 32] = m0;
            mine[33 * 32] = l0;
            mine[34 * 32] = m1;
            mine[35 * 32] = l1;
            asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32));
            auto peer = [&](int k) { return frag + (k * Hkv + head) * 36 * 32 + lane; };
            if (active && pslot == 0) {
                float M0 = m0, M1 = m1;
                for (int k = 1; k < P; ++k) {
                    const float* o = peer(k);
                    M0 = fmaxf(M0, o[32 * 32]);
                    M1 = fmaxf(M1, o[34 * 32]);
                }
                const float s0 = M0 == -INFINITY ? 0.f : M0, s1 = M1 == -INFINITY ? 0.f : M1;
                float f0 = exp2_approx(m0 - s0), f1 = exp2_approx(m1 - s1);
                l0 *= f0;
                l1 *= f1;
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    acc[mt][0] *= f0;
                    acc[mt][1] *= f1;
                    acc[mt][2] *= f0;
                    acc[mt][3] *= f1;
                }
                for (int k = 1; k < P; ++k) {
                    const float* o = peer(k);
                    const float g0 = exp2_approx(o[32 * 32] - s0), g1 = exp2_approx(o[34 * 32] - s1);
                    l0 = fmaf(o[33 * 32], g0, l0);
                    l1 = fmaf(o[35 * 32], g1, l1);
#pragma unroll
                    for (int mt = 0; mt < 8; ++mt) {
                        acc[mt][0] = fmaf(o[(mt * 4 + 0) * 32], g0, acc[mt][0]);
                        acc[mt][1] = fmaf(o[(mt * 4 + 1) * 32], g1, acc[mt][1]);
                        acc[mt][2] = fmaf(o[(mt * 4 + 2) * 32], g0, acc[mt][2]);
                        acc[mt][3] = fmaf(o[(mt * 4 + 3) * 32], g1, acc[mt][3]);
                    }
                }
                m0 = M0;
                m1 = M1;
            }
        }
        // The CTA's partial for each query head of this warp's kv head.
        if (active && pslot == 0) {
            const int Hq = Hkv * G;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int n = 2 * t + half;
                if (n < G) {
                    const size_t row = (size_t)split * Hq + head * G + n;
                    float* dst = a.part_acc + row * kHeadDim;
                    // Kept in L2 (evict_last) until the merge reads them: the
                    // next decode grid streams pages into L2 meanwhile.
                    const uint64_t keep = l2_policy_evict_last();
#pragma unroll
                    for (int mt = 0; mt < 8; ++mt) {
                        st_f32_hint(dst + mt * 16 + g, acc[mt][half], keep);
                        st_f32_hint(dst + mt * 16 + g + 8, acc[mt][2 + half], keep);
                    }
                    if (g == 0) {
                        const float2 ml = half ? make_float2(m1, l1) : make_float2(m0, l0);
                        st_f32_hint(&a.part_ml[row].x, ml.x, keep);
                        st_f32_hint(&a.part_ml[row].y, ml.y, keep);
                    }
                }
            }
        }
    }
    if (a.merge != nullptr) {
        // ---------------- fused split merge ----------------
        // This CTA's partials (and the appended row / table entries) are
        // ordered before its arrival; the last n_merge CTAs to arrive wait
        // (bounded) for the others, then merge one or more (head, half) units.
        // Splits past the step's count (a captured step's fixed grid) had no
        // pages and take no part.
        const int n_splits = a.step ? __ldg(&a.step->n_splits) : (int)gridDim.x;
        const int n_merge = min(n_splits, 2 * Hkv * G);
        __threadfence();
        __syncthreads();
        __shared__ uint32_t s_ticket;
        if (threadIdx.x == 0 && split < n_splits) s_ticket = atomicAdd(&a.merge[0], 1u);
        __syncthreads();
        PROBE_T(3);
        const uint32_t first = (uint32_t)(n_splits - n_merge);
        if (split < n_splits && s_ticket >= first) {
            if (threadIdx.x == 0) {
                uint32_t v;
                const uint64_t t0 = global_timer_ns();
                for (uint32_t i = 0;; ++i) {
                    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.merge) : "memory");
                    if (v >= (uint32_t)n_splits) break;
                    if ((i & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
                        atomicOr(a.err, kErrTimeout);
                        break;
                    }
                }
            }
            __syncthreads();
            PROBE_T(7);
            const int Hq = Hkv * G;
            float* sbuf = reinterpret_cast<float*>(smem);  // stage buffers are free
            for (int u = (int)(s_ticket - first); u < 2 * Hq; u += n_merge) merge_unit(a.part_acc, a.part_ml, a.out, a.out_dtype, sbuf, n_splits, Hq, u >> 1, u & 1);
            if (threadIdx.x == 0) {
                __threadfence();
                if (atomicAdd(&a.merge[1], 1u) == (uint32_t)n_merge - 1u) {
                    // Every merger has read the partials: reset for the next
                    // launch, and publish this step's completion for the next
                    // decode step of the table.
                    a.merge[0] = 0u;
                    a.merge[1] = 0u;
                    if (a.done_post != nullptr)
                        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(a.done_post), "r"(a.done_seq)
                                     : "memory");
                }
            }
        }
    } else if (a.arrive != nullptr) {
        // The combine waits for this count rather than for the grid to
        // complete (GKV_DECODE_COMBINE_WAIT=count). The CTA's partials,
        // appended row and table entries are ordered before it.
        const int n_splits = a.step ? __ldg(&a.step->n_splits) : (int)gridDim.x;
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0 && split < n_splits) atomicAdd(a.arrive, 1u);
        PROBE_T(3);
    } else {
        __syncthreads();
        PROBE_T(3);
    }
    if (a.inputs_ready && threadIdx.x == 0) asm volatile("griddepcontrol.wait;" ::: "memory");

#ifdef GKV_PROBE_TIMELINE
    __syncthreads();
    PROBE_T(4);
#endif
}

struct CombineParams {
    const float* part_acc;
    const float2* part_ml;
    void* out;
    int32_t out_dtype;
    int32_t n_q_heads;
    int32_t n_splits;
    uint32_t* err;
    GatherLaunch g;
    const DeviceStep* step;  // non-null: n_splits from here (captured steps)
    int32_t early;           // 1: the next launch is another layer's decode: trigger it at entry
    uint32_t* done;          // non-null: post done_seq here once the decode grid completed; trigger at entry
    uint32_t done_seq;
    uint32_t* arrive;        // non-null: [0] decode CTAs arrived (wait for n_splits of them instead of the
                             // grid's completion), [1] combine CTAs done (the last one resets both)
#ifdef GKV_PROBE_TIMELINE
    int32_t probe_slot;
#endif
};

constexpr int kCombineWarps = 8;  // 8 warps x 80 registers fit beside a decode CTA (96 registers) on every SM
constexpr int kCombineDims = 32;  // dims per CTA (one per lane)

// Grid (Hq, 128 / 32): warp w of a CTA folds splits w, w + 8, ... for the
// CTA's 32 dims (one per lane, 128-byte coalesced rows), then the 8 warps
// merge through shared memory.
__global__ void __launch_bounds__(kCombineWarps * 32, 3) paged_decode_combine_kernel(const CombineParams c) {
#ifdef GKV_PROBE_TIMELINE
#define PROBE_C(k) if (threadIdx.x == 0) g_probe_tl[(c.probe_slot * 4096 + 2048 + blockIdx.y * gridDim.x + blockIdx.x) * 8 + (k)] = global_timer_ns();
#else
#define PROBE_C(k)
#endif
    PROBE_C(0);
    // When the next launch is another layer's decode (a multi-layer step
    // whose layers are distinct, and not its last layer), it reads nothing
    // this layer's grids write before its own wait: it may start now, its
    // page stream overlapping this layer's tail.
    // With a completion word, a decode launched next reads nothing before its
    // own wait that this step wrote until the word says this step completed
    // (it checks it), so it may start now whatever layer it belongs to: its
    // page stream overlaps this step's tail, this merge and (multi-GPU) the
    // gather's completion protocol.
    const bool gather = c.g.world > 1;
    const bool early = c.done != nullptr || (c.early && !gather);
    if (early) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int n_splits = c.step ? __ldg(&c.step->n_splits) : c.n_splits;
    if (c.arrive != nullptr) {
        // Wait (bounded) until every decode CTA has written its partials;
        // one thread polls, the others wait at the barrier.
        if (threadIdx.x == 0) {
            const uint64_t t0 = global_timer_ns();
            uint32_t v;
            for (uint32_t i = 0;; ++i) {
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c.arrive) : "memory");
                if (v >= (uint32_t)n_splits) break;
                if ((i & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
                    atomicOr(c.err, kErrTimeout);
                    break;
                }
            }
        }
        __syncthreads();
    } else {
        asm volatile("griddepcontrol.wait;" ::: "memory");  // the decode grid's partials are visible
    }
    PROBE_C(1);
    // Every decode CTA's pool rows and table entries are visible. Publish
    // that for the next decode step of this table (with an arrival count,
    // the last combine CTA does it once it has reset the count).
    if (c.arrive == nullptr && c.done != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0)
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(c.done), "r"(c.done_seq) : "memory");
    // Otherwise only now may the next launch start: a decode step of the
    // same layer reads pages and table entries this step's decode grid
    // wrote, and its page stream begins before it waits for this grid. With
    // the fused gather the trigger comes after this rank's stores and flags
    // are out.
    if (!early && !gather) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int hq = blockIdx.x;
    const int lane = threadIdx.x & 31;
    const int d = blockIdx.y * kCombineDims + lane;
    const int w = threadIdx.x >> 5;
    constexpr int kBatch = 19;  // splits per warp in flight at once (147 splits: one round)
    __shared__ float s_l[kCombineWarps], s_a[kCombineWarps][kCombineDims], s_m[kCombineWarps];
    // One pass with an online rescale: each batch's loads are issued together.
    float M = -INFINITY, L = 0.f, A = 0.f;
    for (int b = 0; b * kBatch * kCombineWarps < n_splits; ++b) {
        float2 ml[kBatch];
        float av[kBatch];
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const int s = w + (b * kBatch + i) * kCombineWarps;
            const bool in = s < n_splits;
            ml[i] = in ? c.part_ml[(size_t)s * c.n_q_heads + hq] : make_float2(-INFINITY, 0.f);
            av[i] = in ? c.part_acc[((size_t)s * c.n_q_heads + hq) * kHeadDim + d] : 0.f;
        }
        float mb = M;
#pragma unroll
        for (int i = 0; i < kBatch; ++i) mb = fmaxf(mb, ml[i].x);
        const float ms = mb == -INFINITY ? 0.f : mb;
        const float r = exp2_approx(M - ms);
        L *= r;
        A *= r;
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const float f = exp2_approx(ml[i].x - ms);
            L = fmaf(ml[i].y, f, L);
            A = fmaf(av[i], f, A);
        }
        M = mb;
        // Each 128-byte line of partials (one split, 32 dims) is read by this
        // warp alone: drop it from L2 without a write-back.
        if (lane == 0) {
#pragma unroll
            for (int i = 0; i < kBatch; ++i) {
                const int s = w + (b * kBatch + i) * kCombineWarps;
                if (s < n_splits) l2_discard_line(c.part_acc + ((size_t)s * c.n_q_heads + hq) * kHeadDim + blockIdx.y * kCombineDims);
            }
        }
    }
    if (lane == 0) {
        s_m[w] = M;
        s_l[w] = L;
    }
    s_a[w][lane] = A;
    __syncthreads();
    if (c.arrive != nullptr && threadIdx.x == 0) {
        // The last combine CTA to get here resets the counts for the next
        // step of this table, then publishes the step's completion.
        if (atomicAdd(c.arrive + 1, 1u) == gridDim.x * gridDim.y - 1u) {
            c.arrive[0] = 0u;
            c.arrive[1] = 0u;
            if (c.done != nullptr)
                asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(c.done), "r"(c.done_seq) : "memory");
        }
    }
    if (w == 0) {
        float Mt = -INFINITY;
#pragma unroll
        for (int k = 0; k < kCombineWarps; ++k) Mt = fmaxf(Mt, s_m[k]);
        const float ms = Mt == -INFINITY ? 0.f : Mt;
        float Lt = 0.f, At = 0.f;
#pragma unroll
        for (int k = 0; k < kCombineWarps; ++k) {
            const float f = exp2_approx(s_m[k] - ms);
            Lt = fmaf(s_l[k], f, Lt);
            At = fmaf(s_a[k][lane], f, At);
        }
        PROBE_C(2);
        const float v = At / Lt;
        if (!gather) {
            store_out(c.out, (size_t)hq * kHeadDim + d, v, c.out_dtype);
        } else {
            for (int r = 0; r < c.g.world; ++r) store_out(c.g.dst[r], (size_t)hq * kHeadDim + d, v, c.out_dtype);
        }
    }
    if (!gather) return;
    // ---- fused head all-gather: completion protocol ----
    // This CTA's peer stores are ordered before its ticket at GPU scope; the
    // last CTA's system-scope fence and release (cumulative over what it
    // observed through the tickets) publish every CTA's stores to the peers.
    // A system-scope fence in every CTA cost ~9 us per layer at 2 GPUs.
    __threadfence();
    __syncthreads();
    __shared__ uint32_t s_last;
    if (threadIdx.x == 0) {
        const uint32_t n_ctas = gridDim.x * gridDim.y;
        s_last = atomicAdd(c.g.ticket, 1u) == n_ctas - 1;
    }
    __syncthreads();
    PROBE_C(3);
    if (!s_last) {
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        return;
    }
    if (threadIdx.x == 0) {
        *c.g.ticket = 0u;
        // One system-scope fence, then plain (relaxed) flag stores: together
        // a release of every block this rank stored. A release store per
        // flag would put a system-scope fence in front of each of them.
        __threadfence_system();
        for (int r = 0; r < c.g.n_flag_dst; ++r)
            asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(c.g.flag_dst[r]), "r"(c.g.epoch) : "memory");
    }
    __syncthreads();
    PROBE_C(4);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // Wait (bounded) until every peer's block for this layer and step arrived.
    if (threadIdx.x < c.g.world) {
        const uint32_t* f = c.g.flag_wait[threadIdx.x];
        const uint64_t t0 = global_timer_ns();
        uint32_t v;
        for (uint32_t i = 0;; ++i) {
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
            if ((int32_t)(v - c.g.epoch) >= 0) break;
            if ((i & 63u) == 63u && global_timer_ns() - t0 > c.g.wait_ns) {
                atomicOr(c.err, kErrTimeout);
                break;
            }
        }
    }
#ifdef GKV_PROBE_TIMELINE
    __syncthreads();
    PROBE_C(5);
#endif
}

// GKV_NO_PDL=1 turns programmatic dependent launch off (plain stream order).
bool overlap_enabled() {
    static const bool on = [] {
        const char* v = getenv("GKV_NO_PDL");
        return !(v && v[0] == '1');
    }();
    return on;
}

// Stages past the shared-memory ring that the producer brings into L2
// while the ring is full (GKV_DECODE_L2_PREFETCH, default 0: measured at 32k,
// the prefetch traffic slows the previous layer's merge by more than the
// early pages save on per-layer calls).
int l2_prefetch_stages() {
    static const int n = [] {
        const char* v = getenv("GKV_DECODE_L2_PREFETCH");
        return v ? atoi(v) : 0;
    }();
    return n;
}

// GKV_DECODE_COMBINE_WAIT=count: the combine waits for the decode CTAs'
// arrival count instead of the decode grid's completion. Off by default:
// measured at 32k, the polling costs more (29.4 vs 28.0 us per layer) than
// the earlier start saves.
bool counted_combine() {
    static const bool on = [] {
        const char* v = getenv("GKV_DECODE_COMBINE_WAIT");
        return v && v[0] == 'c';
    }();
    return on;
}

// GKV_DECODE_BOX=head selects the per-(page, head) boxes; the default is one
// box per page and 64-dim half.
bool page_boxes() {
    static const bool on = [] {
        const char* v = getenv("GKV_DECODE_BOX");
        return !(v && v[0] == 'h');
    }();
    return on;
}

}  // namespace

cudaError_t configure_decode_kernels() {
    static std::atomic<unsigned long long> configured{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 64 || !(configured.load() & (1ull << dev))) {
        // Both kernels ask for the largest shared-memory carveout, so that an
        // SM running combine CTAs can take the next decode CTA without
        // reconfiguring (which would wait for the combine CTAs to drain).
        for (auto* k : {paged_decode_kernel<false>, paged_decode_kernel<true>}) {
            e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
            if (e != cudaSuccess) return e;
            e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
            if (e != cudaSuccess) return e;
        }
        e = cudaFuncSetAttribute(paged_decode_combine_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured.fetch_or(1ull << dev);
    }
    return cudaSuccess;
}

bool decode_split_geometry(int32_t n_pages, int32_t n_kv_heads, int32_t n_q_heads, int32_t n_splits_hint,
                           int num_sms, int32_t* pages_per_split, int32_t* n_splits_out) {
    const int P = kConsumerWarps / n_kv_heads;
    const int n_stages_total = (n_pages + P - 1) / P;
    int n_splits = n_splits_hint > 0 ? n_splits_hint : num_sms;
    if (n_splits > n_stages_total) n_splits = n_stages_total;
    if (n_splits * n_q_heads > kMaxPartialRows) n_splits = kMaxPartialRows / n_q_heads;
    if (n_splits < 1) n_splits = 1;
    int stages_per_split = (n_stages_total + n_splits - 1) / n_splits;
    if (stages_per_split * P > kMaxSplitPages) {  // very long contexts: more splits than SMs
        stages_per_split = kMaxSplitPages / P;
        n_splits = (n_stages_total + stages_per_split - 1) / stages_per_split;
        if (n_splits * n_q_heads > kMaxPartialRows) return false;
    }
    *pages_per_split = stages_per_split * P;
    *n_splits_out = (n_pages + *pages_per_split - 1) / *pages_per_split;
    return true;
}

cudaError_t launch_decode(const PoolView& pool, const DecodeMaps& maps, int2* table,
                          const NewPages& np, const Scratch& scratch, const DecodeLaunch& d, int num_sms,
                          cudaStream_t stream, const GatherLaunch* gather) {
    const int Hkv = pool.n_kv_heads;
    if (Hkv > kConsumerWarps) return cudaErrorInvalidValue;
    cudaError_t e = configure_decode_kernels();
    if (e != cudaSuccess) return e;
    DecodeParams p;
    p.q = d.q;
    p.k_new = d.k_new;
    p.v_new = d.v_new;
    p.k_base = pool.k_base;
    p.v_base = pool.v_base;
    p.table = table;
    p.part_acc = scratch.part_acc;
    p.part_ml = scratch.part_ml;
    p.err = scratch.err;
    p.done = d.post_done ? scratch.done : nullptr;
    p.done_expect = d.done_seq - 1u;
    p.merge = nullptr;
    p.arrive = nullptr;
    p.out = d.out;
    p.out_dtype = d.out_dtype;
    p.done_post = nullptr;
    p.done_seq = d.done_seq;
    p.l2_prefetch_stages = l2_prefetch_stages();
    p.n_kv_heads = Hkv;
    p.group = d.n_q_heads / Hkv;
    p.pool_pages = pool.pool_pages;
    p.n_prior = d.n_prior;
    p.total = d.total;
    p.n_pages = d.n_pages;
    p.pages_per_stage = kConsumerWarps / Hkv;
    p.qscale = d.scale * 1.4426950408889634f;
    p.new_first = np.first;
    p.new_n = np.n;
    p.qk_on = d.qk ? 1 : 0;
    if (d.qk) p.qk = *d.qk;
#ifdef GKV_PROBE_TIMELINE
    static int probe_counter = 0;
    p.probe_slot = probe_counter++ % 8;
#endif
    for (int i = 0; i < np.n; ++i) p.new_ids[i] = np.ids[i];

    // One CTA per SM; each split a whole number of stages.
    int n_splits = 0;
    if (!decode_split_geometry(d.n_pages, Hkv, d.n_q_heads, d.n_splits, num_sms, &p.pages_per_split, &n_splits))
        return cudaErrorInvalidValue;
    p.step = d.step;
    p.inputs_ready = d.prev_is_other_layer ? 1 : 0;
    int grid = n_splits;
    // The split merge runs inside the decode grid (no combine launch) with
    // the table's own counters; the fused multi-GPU gather keeps the combine
    // kernel.
    const bool fused = d.fused_merge && scratch.merge != nullptr && !(gather && gather->world > 1);
    p.late_trigger = 0;
    p.arrive = (!fused && scratch.merge != nullptr && counted_combine()) ? scratch.merge : nullptr;
    if (fused) {
        p.merge = scratch.merge;
        p.done_post = d.post_done ? scratch.done : nullptr;
        // The first layer of an uncaptured multi-layer step: the next layer's
        // decode reads its inputs without waiting, so it may start only once
        // this grid has waited for whatever ran before the step.
        p.late_trigger = d.next_is_other_layer && !d.prev_is_other_layer && !d.step ? 1 : 0;
    }
    if (d.step) {
        // Captured step: the geometry in the step block changes from token
        // to token; the grid is fixed and splits past the step's count find
        // no pages.
        if (d.grid < 1 || d.grid * d.n_q_heads > kMaxPartialRows) return cudaErrorInvalidValue;
        grid = d.grid;
    }

    // Both launches use programmatic dependent launch: the decode grid's page
    // stream may start while the previous kernel on the stream finishes (it
    // waits for that kernel before reading Q / the new K/V row), and the
    // combine's CTAs are placed while the decode grid runs.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = overlap_enabled() ? 1 : 0;
    cudaLaunchConfig_t dcfg = {};
    dcfg.gridDim = dim3(grid);
    dcfg.blockDim = dim3(kThreads);
    dcfg.dynamicSmemBytes = kSmemBytes;
    dcfg.stream = stream;
    dcfg.attrs = attr;
    dcfg.numAttrs = 1;
    const bool pb = page_boxes();
    e = pb ? cudaLaunchKernelEx(&dcfg, paged_decode_kernel<true>, maps.k_page, maps.v_page, p)
           : cudaLaunchKernelEx(&dcfg, paged_decode_kernel<false>, maps.k_head, maps.v_head, p);
    if (e != cudaSuccess) return e;
    if (fused) return cudaSuccess;

    CombineParams c{scratch.part_acc, scratch.part_ml, d.out, d.out_dtype, d.n_q_heads, n_splits, scratch.err, {}};
    if (gather) c.g = *gather;
    c.step = d.step;
    c.early = d.next_is_other_layer ? 1 : 0;
    c.done = d.post_done ? scratch.done : nullptr;
    c.done_seq = d.done_seq;
    c.arrive = p.arrive;
#ifdef GKV_PROBE_TIMELINE
    c.probe_slot = p.probe_slot;
#endif
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(d.n_q_heads, kHeadDim / kCombineDims);
    cfg.blockDim = dim3(kCombineWarps * 32);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, paged_decode_combine_kernel, c);
}

}  // namespace gkv

#ifdef GKV_PROBE_TIMELINE
extern "C" int gkv_probe_read_timeline(unsigned long long* out, int n) {
    return (int)cudaMemcpyFromSymbol(out, gkv::g_probe_tl, sizeof(unsigned long long) * n);
}
extern "C" int gkv_probe_read_stages(unsigned long long* out, int n) {
    return (int)cudaMemcpyFromSymbol(out, gkv::g_probe_st, sizeof(unsigned long long) * n);
}
#endif
