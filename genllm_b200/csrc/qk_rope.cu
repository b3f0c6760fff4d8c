// qk_rope.cu — the step between the Q/K/V projections and the attention op,
// fused into one launch: per-head QK-norm and RoPE of Q and K, and the
// [S][H*128] -> [H][S][128] permute of Q, K and V (the reference runs it as
// three reshape_permute ops, two rms_norm ops and two apply_rope ops,
// src/model/Qwen3.cpp:136-154). One CTA per token, one warp per 128-dim row
// of it; the arithmetic is qk_rope.cuh's, bit-exact with the reference CPU ops.
#include <cuda_runtime.h>

#include "kernels.h"
#include "qk_rope.cuh"

namespace gkv {
namespace {

constexpr int kWarps = 8;
constexpr int kMaxRowsPerToken = 96;  // Hq + Hkv rows of one token staged in shared memory (24 KiB)

struct QkRopeParams {
    const uint16_t* q;  // [S][Hq*128]
    const uint16_t* k;  // [S][Hkv*128]
    const uint16_t* v;
    uint16_t* q_out;    // [Hq][S][128]
    uint16_t* k_out;    // [Hkv][S][128]
    uint16_t* v_out;
    QkNorm n;
    int32_t seq_len;
    int32_t n_q_heads;
    int32_t n_kv_heads;
    int32_t start_pos;
};

// One CTA per token: the token's Q, K and V rows are contiguous in the
// projections ([S][H*128]), so the CTA reads them with 16-byte loads into
// shared memory (V goes straight to its head-major place), then each warp
// normalises and rotates rows of Q and K with the position's cos/sin and the
// norm weights held in registers across its rows, and writes each row back
// as 16-byte stores.
__global__ void __launch_bounds__(kWarps * 32) qk_norm_rope_kernel(const QkRopeParams a) {
    __shared__ __align__(16) uint16_t rows[kMaxRowsPerToken][kHeadDim];
    __shared__ __align__(16) uint16_t outs[kWarps][kHeadDim];
    const int s = blockIdx.x;
    const int S = a.seq_len, Hq = a.n_q_heads, Hkv = a.n_kv_heads;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int kChunks = kHeadDim / 8;  // 16-byte pieces of a row
    // Q and K rows of the token into shared memory; V to its output rows.
    {
        const uint4* q = reinterpret_cast<const uint4*>(a.q + (size_t)s * Hq * kHeadDim);
        const uint4* k = reinterpret_cast<const uint4*>(a.k + (size_t)s * Hkv * kHeadDim);
        const uint4* v = reinterpret_cast<const uint4*>(a.v + (size_t)s * Hkv * kHeadDim);
        uint4* sm = reinterpret_cast<uint4*>(&rows[0][0]);
        for (int i = threadIdx.x; i < Hq * kChunks; i += kWarps * 32) sm[i] = q[i];
        for (int i = threadIdx.x; i < Hkv * kChunks; i += kWarps * 32) {
            sm[Hq * kChunks + i] = k[i];
            const int h = i / kChunks, c = i % kChunks;
            reinterpret_cast<uint4*>(a.v_out + ((size_t)h * S + s) * kHeadDim)[c] = v[i];
        }
    }
    const size_t pos = (size_t)(a.start_pos + s) * kHeadDim;
    __syncthreads();
    const RowParams pq = load_row_params(a.n.q_w, a.n.cos + pos, a.n.sin + pos, lane);
    RowParams pk = pq;
#pragma unroll
    for (int it = 0; it < 4; ++it) pk.w[it] = a.n.k_w[lane + 32 * it];
    uint16_t* ob = outs[warp];
    for (int r = warp; r < Hq + Hkv; r += kWarps) {
        const bool is_q = r < Hq;
        float x[4];
        load_row4(rows[r], lane, x);
        uint16_t o[4];
        norm_rope_row(x, is_q ? pq : pk, a.n.eps, o);
#pragma unroll
        for (int it = 0; it < 4; ++it) ob[lane + 32 * it] = o[it];
        __syncwarp();
        uint16_t* dst = is_q ? a.q_out + ((size_t)r * S + s) * kHeadDim : a.k_out + ((size_t)(r - Hq) * S + s) * kHeadDim;
        if (lane < kChunks) reinterpret_cast<uint4*>(dst)[lane] = reinterpret_cast<const uint4*>(ob)[lane];
        __syncwarp();
    }
}

}  // namespace

cudaError_t launch_qk_norm_rope(const uint16_t* q, const uint16_t* k, const uint16_t* v, int32_t seq_len,
                                int32_t n_q_heads, int32_t n_kv_heads, const QkNorm& n, int32_t start_pos,
                                uint16_t* q_out, uint16_t* k_out, uint16_t* v_out, cudaStream_t stream) {
    QkRopeParams p{q, k, v, q_out, k_out, v_out, n, seq_len, n_q_heads, n_kv_heads, start_pos};
    if (seq_len <= 0) return cudaSuccess;
    if (n_q_heads + n_kv_heads > kMaxRowsPerToken) return cudaErrorInvalidValue;
    // 16-byte accesses: every pointer must be 16-byte aligned.
    for (const void* ptr : {(const void*)q, (const void*)k, (const void*)v, (const void*)q_out, (const void*)k_out,
                            (const void*)v_out})
        if (reinterpret_cast<uintptr_t>(ptr) % 16) return cudaErrorInvalidValue;
    qk_norm_rope_kernel<<<(unsigned)seq_len, kWarps * 32, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace gkv
