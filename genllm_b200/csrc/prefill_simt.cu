// prefill_simt.cu — multi-query paged attention on CUDA cores.
//
// Used for seq_len > 1 chunks whose shape the tensor-core prefill kernel does
// not take. One warp per (query head, query row); a lane owns 4 of the 128
// dims; pages are walked in order through the device block table and each
// token is folded into an fp32 online softmax, as in the reference CPU op
// (src/backend/cpu/attention.cpp:156-215), with causal masking at
// q_abs = total - seq_len + sq.
#include "device.cuh"
#include "kernels.h"

namespace gkv {
namespace {

struct SimtParams {
    const uint16_t* q;
    const uint16_t* k_base;
    const uint16_t* v_base;
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
    float qscale;
};

__global__ void __launch_bounds__(128) prefill_simt_kernel(const SimtParams a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sq = blockIdx.x * 4 + warp;
    const int hq = blockIdx.y;
    if (sq >= a.seq_len) return;
    const int G = a.n_q_heads / a.n_kv_heads;
    const int h = hq / G;
    const int Hkv = a.n_kv_heads;
    const int q_abs = a.total - a.seq_len + sq;
    const int limit = a.causal ? q_abs : a.total - 1;

    const uint2 qr = *reinterpret_cast<const uint2*>(a.q + ((size_t)hq * a.seq_len + sq) * kHeadDim + lane * 4);
    const float q0 = bf16_lo(qr.x) * a.qscale, q1 = bf16_hi(qr.x) * a.qscale;
    const float q2 = bf16_lo(qr.y) * a.qscale, q3 = bf16_hi(qr.y) * a.qscale;
    float m = -INFINITY, l = 0.f, o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;

    for (int lp = 0; lp < a.n_pages; ++lp) {
        const int base = lp * kPageSlots;
        if (base > limit) break;
        const int2 e = a.table[lp];
        if (e.x < 0 || e.x >= a.pool_pages || e.y < 0 || e.y >= a.pool_pages) {
            if (lane == 0) atomicOr(a.err, kErrBadPage);
            continue;
        }
        const int n = min(min(kPageSlots, a.total - base), limit - base + 1);
        const uint16_t* kp = a.k_base + ((size_t)e.x * kPageSlots * Hkv + h) * kHeadDim + lane * 4;
        const uint16_t* vp = a.v_base + ((size_t)e.y * kPageSlots * Hkv + h) * kHeadDim + lane * 4;
        for (int s = 0; s < n; ++s) {
            const uint2 kr = *reinterpret_cast<const uint2*>(kp + (size_t)s * Hkv * kHeadDim);
            float sc = q0 * bf16_lo(kr.x) + q1 * bf16_hi(kr.x) + q2 * bf16_lo(kr.y) + q3 * bf16_hi(kr.y);
#pragma unroll
            for (int mask = 16; mask >= 1; mask >>= 1) sc += __shfl_xor_sync(0xFFFFFFFFu, sc, mask);
            const float mn = fmaxf(m, sc);
            const float alpha = exp2_approx(m - mn);
            const float p = exp2_approx(sc - mn);
            const uint2 vr = *reinterpret_cast<const uint2*>(vp + (size_t)s * Hkv * kHeadDim);
            o0 = o0 * alpha + p * bf16_lo(vr.x);
            o1 = o1 * alpha + p * bf16_hi(vr.x);
            o2 = o2 * alpha + p * bf16_lo(vr.y);
            o3 = o3 * alpha + p * bf16_hi(vr.y);
            l = l * alpha + p;
            m = mn;
        }
    }
    const float inv = 1.f / l;
    const size_t o = ((size_t)hq * a.seq_len + sq) * kHeadDim + lane * 4;
    store_out(a.out, o + 0, o0 * inv, a.out_dtype);
    store_out(a.out, o + 1, o1 * inv, a.out_dtype);
    store_out(a.out, o + 2, o2 * inv, a.out_dtype);
    store_out(a.out, o + 3, o3 * inv, a.out_dtype);
}

}  // namespace

cudaError_t launch_prefill_simt(const PoolView& pool, const int2* table, const PrefillLaunch& p,
                                uint32_t* err, cudaStream_t stream) {
    SimtParams a;
    a.q = p.q;
    a.k_base = pool.k_base;
    a.v_base = pool.v_base;
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
    dim3 grid((p.seq_len + 3) / 4, p.n_q_heads);
    prefill_simt_kernel<<<grid, 128, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace gkv
