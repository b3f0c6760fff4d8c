// qk_rope.cuh — per-head RMSNorm (Qwen3's QK-norm) and RoPE of one 128-dim
// row by one warp, bit-exact with the reference CPU ops:
//   src/backend/cpu/normalization.cpp:39-95  rms_norm (AVX2): four 8-lane
//     fma accumulators over 32-element steps, merged (a0+a1)+(a2+a3), the
//     two 128-bit halves added, two horizontal adds; rms = 1/sqrt(sum/n+eps);
//     (x * rms) * w stored by truncation to bf16;
//   src/backend/cpu/rope.cpp:73-110  ApplyRopeImpl<CPU>: half-split
//     rotation with cos/sin of position pos; as the reference is built
//     (-O3 -mfma, GCC's default contraction for C++) each rotation is one
//     fused multiply-add whose addend is the other product rounded; bf16 RNE
//     store.
// Lane l holds the row's elements l, l+32, l+64, l+96 (index `it`): that is
// the AVX2 accumulator layout (lane = 8 k + j for accumulator k, lane j) and
// puts each RoPE pair (i, i+64) in one lane.
#pragma once
#include <stdint.h>

#include "device.cuh"
#include "kernels.h"

namespace gkv {

// This lane's parameters of a row: the weights of its 4 elements and the
// cos/sin of its two RoPE pairs (i = lane, lane + 32) at the row's position.
struct RowParams {
    float w[4], c[2], s[2];
};
__device__ __forceinline__ RowParams load_row_params(const float* w, const float* cs, const float* sn, int lane) {
    RowParams p;
#pragma unroll
    for (int it = 0; it < 4; ++it) p.w[it] = w[lane + 32 * it];
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        p.c[it] = cs[lane + 32 * it];
        p.s[it] = sn[lane + 32 * it];
    }
    return p;
}

// x: this lane's 4 elements (floats of bf16 inputs). out: bf16 bits of the
// same 4 elements after RMSNorm and RoPE.
__device__ __forceinline__ void norm_rope_row(const float (&x)[4], const RowParams& p, float eps,
                                              uint16_t (&out)[4]) {
    // Sum of squares in the AVX2 order.
    float acc = 0.f;
#pragma unroll
    for (int it = 0; it < 4; ++it) acc = __fmaf_rn(x[it], x[it], acc);
    const float t = __fadd_rn(acc, __shfl_down_sync(0xFFFFFFFFu, acc, 8));  // lanes 0-7: a0+a1, 16-23: a2+a3
    const float a0 = __fadd_rn(t, __shfl_down_sync(0xFFFFFFFFu, t, 16));    // lanes 0-7
    const float s4 = __fadd_rn(a0, __shfl_down_sync(0xFFFFFFFFu, a0, 4));   // lanes 0-3
    const float u = __fadd_rn(s4, __shfl_down_sync(0xFFFFFFFFu, s4, 1));    // lanes 0, 2
    const float tot = __fadd_rn(u, __shfl_down_sync(0xFFFFFFFFu, u, 2));    // lane 0
    const float sum = __shfl_sync(0xFFFFFFFFu, tot, 0);
    // sum / 128 is exact as a product with 2^-7 (both round the same real
    // number); the reciprocal square root keeps the reference's two IEEE steps.
    const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(sum, 0.0078125f), eps)));
    float y[4];
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const float v = __fmul_rn(__fmul_rn(x[it], rms), p.w[it]);
        y[it] = __uint_as_float(__float_as_uint(v) & 0xFFFF0000u);  // truncation to bf16
    }
    // RoPE: pairs (it, it + 2) = elements (i, i + 64), i = lane + 32 it.
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const float c = p.c[it], s = p.s[it];
        out[it] = bf16_bits_ref_fast(__fmaf_rn(y[it], c, -__fmul_rn(y[it + 2], s)));
        out[it + 2] = bf16_bits_ref_fast(__fmaf_rn(y[it], s, __fmul_rn(y[it + 2], c)));
    }
}

// The same arithmetic with a row per 8-lane group (4 rows per warp at once).
// Lane j of the group holds the 16 elements e = 32 it + 8 k + j (it, k in
// 0..3): the AVX2 accumulator (k, j) is then a chain inside one lane, and the
// RoPE pairs (e, e + 64) are (it, it + 2) of the same lane. x/out indexed
// [it][k]; w/cs/sn are the full rows (weights, the position's cos/sin).
// This lane's parameters for norm_rope_row_g8: the weights of its 16
// elements and the cos/sin of its 8 RoPE pairs at the row's position.
struct RowParamsG8 {
    float w[4][4], c[2][4], s[2][4];
};
__device__ __forceinline__ RowParamsG8 load_row_params_g8(const float* w, const float* cs, const float* sn, int j) {
    RowParamsG8 p;
#pragma unroll
    for (int it = 0; it < 4; ++it)
#pragma unroll
        for (int k = 0; k < 4; ++k) p.w[it][k] = w[32 * it + 8 * k + j];
#pragma unroll
    for (int it = 0; it < 2; ++it)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            p.c[it][k] = cs[32 * it + 8 * k + j];
            p.s[it][k] = sn[32 * it + 8 * k + j];
        }
    return p;
}

__device__ __forceinline__ void norm_rope_row_g8(const float (&x)[4][4], int j, const RowParamsG8& p, float eps,
                                                 uint16_t (&out)[4][4]) {
    float acc[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        acc[k] = 0.f;
#pragma unroll
        for (int it = 0; it < 4; ++it) acc[k] = __fmaf_rn(x[it][k], x[it][k], acc[k]);
    }
    const float a0 = __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
    const float s4 = __fadd_rn(a0, __shfl_down_sync(0xFFFFFFFFu, a0, 4, 8));  // j < 4
    const float u = __fadd_rn(s4, __shfl_down_sync(0xFFFFFFFFu, s4, 1, 8));   // j = 0, 2
    const float tot = __fadd_rn(u, __shfl_down_sync(0xFFFFFFFFu, u, 2, 8));   // j = 0
    const float sum = __shfl_sync(0xFFFFFFFFu, tot, 0, 8);
    const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(sum, 0.0078125f), eps)));
    float y[4][4];
#pragma unroll
    for (int it = 0; it < 4; ++it)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float v = __fmul_rn(__fmul_rn(x[it][k], rms), p.w[it][k]);
            y[it][k] = __uint_as_float(__float_as_uint(v) & 0xFFFF0000u);
        }
#pragma unroll
    for (int it = 0; it < 2; ++it)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float c = p.c[it][k], s = p.s[it][k];
            out[it][k] = bf16_bits_ref_fast(__fmaf_rn(y[it][k], c, -__fmul_rn(y[it + 2][k], s)));
            out[it + 2][k] = bf16_bits_ref_fast(__fmaf_rn(y[it][k], s, __fmul_rn(y[it + 2][k], c)));
        }
}

// Load a bf16 row's 4 elements of this lane.
__device__ __forceinline__ void load_row4(const uint16_t* row, int lane, float (&x)[4]) {
#pragma unroll
    for (int it = 0; it < 4; ++it) x[it] = __uint_as_float((uint32_t)row[lane + 32 * it] << 16);
}

}  // namespace gkv
