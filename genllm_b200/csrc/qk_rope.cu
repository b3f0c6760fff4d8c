// qk_rope.cu — the step between the Q/K/V projections and the attention op,
// fused into one launch: per-head QK-norm and RoPE of Q and K, and the
// [S][H*128] -> [H][S][128] permute of Q, K and V (the reference runs it as
// three reshape_permute ops, two rms_norm ops and two apply_rope ops,
// src/model/Qwen3.cpp:136-154). One warp per 128-dim row; the arithmetic is
// qk_rope.cuh's, bit-exact with the reference CPU ops.
#include <cuda_runtime.h>

#include "kernels.h"
#include "qk_rope.cuh"

namespace gkv {
namespace {

constexpr int kWarps = 8;

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

__global__ void __launch_bounds__(kWarps * 32) qk_norm_rope_kernel(const QkRopeParams a) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
    const int S = a.seq_len, Hq = a.n_q_heads, Hkv = a.n_kv_heads;
    // Rows: all Q heads of every token, then K, then V (head-major per kind).
    const int nq = S * Hq, nk = S * Hkv;
    if (row >= nq + 2 * nk) return;
    int kind, h, s;
    if (row < nq) {
        kind = 0;
        h = row / S;
        s = row - h * S;
    } else if (row < nq + nk) {
        kind = 1;
        h = (row - nq) / S;
        s = row - nq - h * S;
    } else {
        kind = 2;
        h = (row - nq - nk) / S;
        s = row - nq - nk - h * S;
    }
    const int H = kind == 0 ? Hq : Hkv;
    const uint16_t* src = (kind == 0 ? a.q : kind == 1 ? a.k : a.v) + ((size_t)s * H + h) * kHeadDim;
    uint16_t* dst = (kind == 0 ? a.q_out : kind == 1 ? a.k_out : a.v_out) + ((size_t)h * S + s) * kHeadDim;
    if (kind == 2) {  // V: the permute only
        reinterpret_cast<uint2*>(dst)[lane] = reinterpret_cast<const uint2*>(src)[lane];
        return;
    }
    float x[4];
    load_row4(src, lane, x);
    const size_t pos = (size_t)(a.start_pos + s) * kHeadDim;
    const RowParams rp = load_row_params(kind == 0 ? a.n.q_w : a.n.k_w, a.n.cos + pos, a.n.sin + pos, lane);
    uint16_t o[4];
    norm_rope_row(x, rp, a.n.eps, o);
#pragma unroll
    for (int it = 0; it < 4; ++it) dst[lane + 32 * it] = o[it];
}

}  // namespace

cudaError_t launch_qk_norm_rope(const uint16_t* q, const uint16_t* k, const uint16_t* v, int32_t seq_len,
                                int32_t n_q_heads, int32_t n_kv_heads, const QkNorm& n, int32_t start_pos,
                                uint16_t* q_out, uint16_t* k_out, uint16_t* v_out, cudaStream_t stream) {
    QkRopeParams p{q, k, v, q_out, k_out, v_out, n, seq_len, n_q_heads, n_kv_heads, start_pos};
    const long long rows = (long long)seq_len * (n_q_heads + 2 * n_kv_heads);
    if (rows <= 0) return cudaSuccess;
    const unsigned grid = (unsigned)((rows + kWarps - 1) / kWarps);
    qk_norm_rope_kernel<<<grid, kWarps * 32, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace gkv
