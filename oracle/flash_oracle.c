/*
 * flash_oracle.c — CPU restatement of the reference's non-paged attention op,
 * FlashAttentionImpl<CPU>::execute (src/backend/cpu/attention.cpp:39-120):
 * self-attention over one chunk (K/V hold the same seq_len tokens as Q),
 * batch >= 1, GQA head h -> kv head h / groups, scores dot * scale (dot
 * accumulated in float in d order), causal mask skv > sq, softmax with expf
 * (max, exp-and-sum, divide), out = sum_skv p * v in skv order. Stops before
 * the final store in the output dtype (fp32 out).
 *
 * TEST INFRASTRUCTURE ONLY (see paged_oracle.h).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#include "paged_oracle.h"

void orc_flash_attention_f32(const uint16_t* q, const uint16_t* k, const uint16_t* v, int32_t batch, int32_t Hq,
                             int32_t Hkv, int32_t S, int32_t D, int32_t groups, float scale, int causal,
                             float* out) {
    float* scores = (float*)malloc(sizeof(float) * (size_t)(S > 0 ? S : 1));
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t h = 0; h < Hq; ++h) {
            const int64_t kvh = h / groups;
            for (int64_t sq = 0; sq < S; ++sq) {
                const uint16_t* qr = q + ((b * Hq + h) * S + sq) * D;
                for (int64_t skv = 0; skv < S; ++skv) {
                    const uint16_t* kr = k + ((b * Hkv + kvh) * S + skv) * D;
                    float dot = 0.0f;
                    for (int32_t d = 0; d < D; ++d) dot += orc_bf16_to_f32(qr[d]) * orc_bf16_to_f32(kr[d]);
                    scores[skv] = dot * scale;
                }
                if (causal)
                    for (int64_t skv = sq + 1; skv < S; ++skv) scores[skv] = -INFINITY;
                float mx = -INFINITY;
                for (int64_t skv = 0; skv < S; ++skv)
                    if (scores[skv] > mx) mx = scores[skv];
                float sum = 0.0f;
                for (int64_t skv = 0; skv < S; ++skv) {
                    scores[skv] = expf(scores[skv] - mx);
                    sum += scores[skv];
                }
                for (int64_t skv = 0; skv < S; ++skv) scores[skv] /= sum;
                float* orow = out + ((b * Hq + h) * S + sq) * D;
                for (int32_t d = 0; d < D; ++d) {
                    float val = 0.0f;
                    for (int64_t skv = 0; skv < S; ++skv)
                        val += scores[skv] * orc_bf16_to_f32(v[((b * Hkv + kvh) * S + skv) * D + d]);
                    orow[d] = val;
                }
            }
        }
    free(scores);
}
