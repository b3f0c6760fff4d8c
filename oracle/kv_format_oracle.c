/*
 * kv_format_oracle.c — CPU restatement of the KV format export / import
 * (pages <-> dense head-major [Hkv][n_tokens][128], bf16 or fp8 e4m3).
 *
 * TEST INFRASTRUCTURE ONLY (see paged_oracle.h). The reference has no export
 * of its cache: the page addressing followed here is its append's
 * (src/core/page_attention.cpp:122-139, page(id) + (slot * Hkv + h) * D),
 * run backwards; the bf16 rounding of the import is the reference's
 * (include/utils/bfloat16.hpp:18-45, orc_bf16_from_f32).
 *
 * The fp8 format is OCP FP8 E4M3 ("OCP 8-bit Floating Point Specification",
 * 2023): bias 7, no infinities, S.1111.111 the only NaN, largest finite 448,
 * subnormal step 2^-9. Encoding rounds to nearest, ties to even, and
 * saturates: finite values and infinities beyond +-448 give +-448; NaN gives
 * 0x7F. The block scale is amax / 448 over the block's finite elements, or
 * 1 where 448 / amax is not finite (amax 0 or below ~2^-119).
 * tests/test_kv_format_oracle.py pins the encoder against torch's own
 * float8_e4m3fn conversion for every in-range input class.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "paged_oracle.h"

uint8_t orc_e4m3_from_f32(float f) {
    if (isnan(f)) return 0x7F;
    const uint8_t sign = signbit(f) ? 0x80 : 0x00;
    const double a = fabs((double)f);
    if (a >= 448.0) return sign | 0x7E;
    if (a < 0x1p-6) {
        /* subnormal range: multiples of 2^-9; a count of 8 is 2^-6 = code 0x08 */
        const double m = nearbyint(a * 0x1p9); /* default rounding: ties to even */
        return sign | (uint8_t)m;
    }
    int e;
    const double fr = frexp(a, &e); /* a = fr * 2^e, fr in [0.5, 1) */
    int ex = e - 1;                 /* a = (2 fr) * 2^ex, 2 fr in [1, 2) */
    double m = nearbyint((2.0 * fr - 1.0) * 8.0);
    if (m == 8.0) {
        m = 0.0;
        ex += 1;
    }
    /* a < 448 keeps (ex, m) at or below (8, 6) */
    return sign | (uint8_t)(((ex + 7) << 3) | (int)m);
}

float orc_e4m3_to_f32(uint8_t b) {
    const int s = b >> 7, e = (b >> 3) & 0xF, m = b & 7;
    float v;
    if (e == 0xF && m == 7) return NAN;
    if (e == 0)
        v = ldexpf((float)m, -9);
    else
        v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
    return s ? -v : v;
}

/* max |x| over the finite elements of n bf16 values (0 if none) */
static float block_amax(const uint16_t* const* rows, int n_rows, int dim) {
    float amax = 0.0f;
    for (int r = 0; r < n_rows; ++r)
        for (int d = 0; d < dim; ++d) {
            const float a = fabsf(orc_bf16_to_f32(rows[r][d]));
            if (isfinite(a) && a > amax) amax = a;
        }
    return amax;
}

void orc_export_kv(const uint16_t* k_pool_base, const uint16_t* v_pool_base, const int32_t* k_ids,
                   const int32_t* v_ids, int32_t n_tokens, int32_t n_kv_heads, int32_t head_dim, int fp8,
                   void* k_out, void* v_out, float* k_scales, float* v_scales) {
    const int32_t n_pages = (n_tokens + ORC_PAGE_SLOTS - 1) / ORC_PAGE_SLOTS;
    const size_t page_elems = (size_t)ORC_PAGE_SLOTS * n_kv_heads * head_dim;
    for (int which = 0; which < 2; ++which) {
        const uint16_t* base = which ? v_pool_base : k_pool_base;
        const int32_t* ids = which ? v_ids : k_ids;
        void* out = which ? v_out : k_out;
        float* scales = which ? v_scales : k_scales;
        for (int32_t lp = 0; lp < n_pages; ++lp) {
            const int valid = n_tokens - lp * ORC_PAGE_SLOTS < ORC_PAGE_SLOTS ? n_tokens - lp * ORC_PAGE_SLOTS
                                                                              : ORC_PAGE_SLOTS;
            const uint16_t* page = base + (size_t)ids[lp] * page_elems;
            for (int32_t h = 0; h < n_kv_heads; ++h) {
                const uint16_t* rows[ORC_PAGE_SLOTS];
                for (int s = 0; s < valid; ++s) rows[s] = page + ((size_t)s * n_kv_heads + h) * head_dim;
                const size_t row0 = (size_t)h * n_tokens + (size_t)lp * ORC_PAGE_SLOTS;
                if (!fp8) {
                    for (int s = 0; s < valid; ++s)
                        memcpy((uint16_t*)out + (row0 + s) * head_dim, rows[s], (size_t)head_dim * 2);
                    continue;
                }
                const float amax = block_amax(rows, valid, head_dim);
                /* 448 / amax not finite (amax 0 or below ~2^-119): scale 1 */
                float inv = 448.0f / amax;
                const int unit = !isfinite(inv);
                const float scale = unit ? 1.0f : amax / 448.0f;
                if (unit) inv = 1.0f;
                for (int s = 0; s < valid; ++s)
                    for (int d = 0; d < head_dim; ++d) {
                        const float y = orc_bf16_to_f32(rows[s][d]) * inv;
                        ((uint8_t*)out)[(row0 + s) * head_dim + d] = orc_e4m3_from_f32(y);
                    }
                scales[(size_t)h * n_pages + lp] = scale;
            }
        }
    }
}

void orc_import_fp8(uint16_t* k_pool_base, uint16_t* v_pool_base, const int32_t* k_ids, const int32_t* v_ids,
                    int32_t n_prior, const uint8_t* k_in, const uint8_t* v_in, const float* k_scales,
                    const float* v_scales, int32_t seq_len, int32_t n_kv_heads, int32_t head_dim) {
    const int32_t n_blocks = (seq_len + ORC_PAGE_SLOTS - 1) / ORC_PAGE_SLOTS;
    const size_t page_elems = (size_t)ORC_PAGE_SLOTS * n_kv_heads * head_dim;
    for (int which = 0; which < 2; ++which) {
        uint16_t* base = which ? v_pool_base : k_pool_base;
        const int32_t* ids = which ? v_ids : k_ids;
        const uint8_t* in = which ? v_in : k_in;
        const float* scales = which ? v_scales : k_scales;
        for (int32_t h = 0; h < n_kv_heads; ++h)
            for (int32_t p = 0; p < seq_len; ++p) {
                const int32_t pos = n_prior + p;
                const float scale = scales[(size_t)h * n_blocks + p / ORC_PAGE_SLOTS];
                uint16_t* dst = base + (size_t)ids[pos / ORC_PAGE_SLOTS] * page_elems +
                                ((size_t)(pos % ORC_PAGE_SLOTS) * n_kv_heads + h) * head_dim;
                const uint8_t* src = in + ((size_t)h * seq_len + p) * head_dim;
                for (int d = 0; d < head_dim; ++d) dst[d] = orc_bf16_from_f32(orc_e4m3_to_f32(src[d]) * scale);
            }
    }
}
