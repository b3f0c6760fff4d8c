/*
 * qk_rope_oracle.c — CPU restatement of the reference's per-head RMSNorm
 * (QK-norm) and RoPE, the two ops that produce the post-QK-norm, post-RoPE
 * Q and K the paged-attention op appends and attends.
 *
 * TEST INFRASTRUCTURE ONLY (see paged_oracle.h). Paths are relative to the
 * Genllm source tree:
 *   orc_rms_norm_bf16   src/backend/cpu/normalization.cpp:39-95 (rms_norm):
 *                       the AVX2 kernel's exact order — four 8-lane fma
 *                       accumulators over 32-element steps, the pairwise
 *                       merge, the 128-bit halves and two horizontal adds;
 *                       1 / sqrt(sum / n + eps); (x * rms) * w stored by
 *                       truncation to bf16 (store_f32_bf16, :24-31).
 *   orc_apply_rope_bf16 src/backend/cpu/rope.cpp:73-110 (ApplyRopeImpl<CPU>):
 *                       half-split rotation, bf16 RNE store. The reference
 *                       build (CMakeLists.txt: -O3 -mfma, GCC's default
 *                       -ffp-contract=fast for C++) contracts each rotation
 *                       into one fused multiply-add whose addend is the
 *                       other product rounded; this restatement writes that
 *                       form out with fmaf (pinned against the reference ops
 *                       built with those flags, tests/test_oracle.py).
 *   orc_rope_cache      src/backend/cpu/rope.cpp:112-140 (RopeCacheImpl<CPU>):
 *                       double-precision inverse frequencies and angles,
 *                       cos/sin rounded to float, each value written to
 *                       columns i and i + head_dim/2.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "paged_oracle.h"

static float bf16f(uint16_t b) { return orc_bf16_to_f32(b); }

static uint16_t bf16_trunc(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return (uint16_t)(u >> 16);
}

void orc_rms_norm_bf16(const uint16_t* x, const float* w, uint16_t* out, int64_t rows, int64_t dim, float eps) {
    for (int64_t r = 0; r < rows; ++r) {
        const uint16_t* xr = x + r * dim;
        uint16_t* orow = out + r * dim;
        float acc[4][8];
        memset(acc, 0, sizeof acc);
        int64_t j = 0;
        for (; j + 32 <= dim; j += 32)
            for (int k = 0; k < 4; ++k)
                for (int l = 0; l < 8; ++l) {
                    const float v = bf16f(xr[j + 8 * k + l]);
                    acc[k][l] = fmaf(v, v, acc[k][l]);
                }
        float a0[8];
        for (int l = 0; l < 8; ++l) {
            const float s01 = acc[0][l] + acc[1][l];
            const float s23 = acc[2][l] + acc[3][l];
            a0[l] = s01 + s23;
        }
        for (; j + 8 <= dim; j += 8)
            for (int l = 0; l < 8; ++l) {
                const float v = bf16f(xr[j + l]);
                a0[l] = fmaf(v, v, a0[l]);
            }
        /* hsum_ps: 128-bit halves added lane-wise, then two horizontal adds */
        float s4[4];
        for (int k = 0; k < 4; ++k) s4[k] = a0[k] + a0[k + 4];
        float sum_sq = (s4[0] + s4[1]) + (s4[2] + s4[3]);
        for (; j < dim; ++j) { /* scalar tail (dim % 8 != 0), contracted as built */
            const float v = bf16f(xr[j]);
            sum_sq = fmaf(v, v, sum_sq);
        }
        const float rms = 1.0f / sqrtf(sum_sq / (float)dim + eps);
        j = 0;
        for (; j + 8 <= dim; j += 8)
            for (int l = 0; l < 8; ++l) {
                const float y = (bf16f(xr[j + l]) * rms) * w[j + l];
                orow[j + l] = bf16_trunc(y);
            }
        for (; j < dim; ++j) orow[j] = orc_bf16_from_f32((bf16f(xr[j]) * rms) * w[j]);
    }
}

void orc_apply_rope_bf16(const uint16_t* x, uint16_t* out, const float* cos_tab, const float* sin_tab,
                         int64_t n_heads, int64_t seq, int64_t head_dim, int64_t start_pos) {
    const int64_t half = head_dim / 2;
    for (int64_t h = 0; h < n_heads; ++h)
        for (int64_t s = 0; s < seq; ++s) {
            const int64_t pos = start_pos + s;
            const float* c = cos_tab + pos * head_dim;
            const float* sn = sin_tab + pos * head_dim;
            const uint16_t* xr = x + (h * seq + s) * head_dim;
            uint16_t* orow = out + (h * seq + s) * head_dim;
            for (int64_t i = 0; i < half; ++i) {
                const float x0 = bf16f(xr[i]), x1 = bf16f(xr[i + half]);
                const float ci = c[i], si = sn[i];
                orow[i] = orc_bf16_from_f32(fmaf(x0, ci, -(x1 * si)));
                orow[i + half] = orc_bf16_from_f32(fmaf(x0, si, x1 * ci));
            }
        }
}

void orc_rope_cache(float theta, int32_t head_dim, int32_t max_seq, float* cos_out, float* sin_out) {
    const int32_t half = head_dim / 2;
    for (int32_t s = 0; s < max_seq; ++s) {
        const double pos = (double)s;
        for (int32_t i = 0; i < half; ++i) {
            const double inv = 1.0 / pow((double)theta, (2.0 * (double)i) / (double)head_dim);
            const double angle = pos * inv;
            const float cv = (float)cos(angle), sv = (float)sin(angle);
            cos_out[(int64_t)s * head_dim + i] = cv;
            cos_out[(int64_t)s * head_dim + i + half] = cv;
            sin_out[(int64_t)s * head_dim + i] = sv;
            sin_out[(int64_t)s * head_dim + i + half] = sv;
        }
    }
}
