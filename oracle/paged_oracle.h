/*
 * paged_oracle.h — CPU restatement of Genllm's paged KV-cache path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the parity tests, smoke() and
 * bench.py's cpu_baseline leg compare the CUDA product against. Nothing in the
 * product (genllm_b200/) links, imports or calls it.
 *
 * Each function restates one piece of the reference (paths are relative to the
 * Genllm source tree):
 *   orc_bf16_from_f32 / orc_bf16_to_f32  include/utils/bfloat16.hpp:18-45
 *   orc_pool_*                           src/core/page_attention.cpp:25-64 (BlockPool)
 *   orc_layer_append_pages               src/core/page_attention.cpp:141-162
 *   orc_layer_append_kv                  src/core/page_attention.cpp:104-139
 *   orc_paged_attention_f32              src/backend/cpu/attention.cpp:156-215
 *
 * Parity is pinned against the reference itself: oracle/_ref (built from the
 * reference's own translation units by oracle/Makefile) is run on the same
 * seeded inputs by tests/test_oracle.py, and tests/golden/ holds vectors made
 * by that build (tests/golden/make_golden.py).
 */
#ifndef GENLLM_PAGED_ORACLE_H
#define GENLLM_PAGED_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_PAGE_SLOTS 16 /* PAGE_BLOCK_SIZE, include/core/page_attention.h:9 */

/* dtype codes: the reference's GGML DataType values (include/utils/utils.hpp) */
#define ORC_F32 0
#define ORC_F16 1
#define ORC_BF16 30

uint16_t orc_bf16_from_f32(float f);
float orc_bf16_to_f32(uint16_t b);
float orc_f16_to_f32(uint16_t h);

/* BlockPool: LIFO free list over ids [0, capacity). */
typedef struct orc_pool {
    int32_t capacity;
    int32_t num_blocks; /* ids handed out so far (high-water mark) */
    int32_t n_free;
    int32_t* free_list; /* capacity entries */
} orc_pool;

int orc_pool_init(orc_pool* p, int32_t capacity);
void orc_pool_release(orc_pool* p);
int32_t orc_pool_alloc(orc_pool* p);
void orc_pool_free(orc_pool* p, int32_t id);
void orc_pool_reset(orc_pool* p);

/* Per-layer page table state: num_cached and (k_id, v_id) per logical page. */
typedef struct orc_layer {
    int32_t num_cached;
    int32_t n_pages;
    int32_t table_cap;
    int32_t* k_ids;
    int32_t* v_ids;
    orc_pool k_pool;
    orc_pool v_pool;
} orc_layer;

int orc_layer_init(orc_layer* L, int32_t max_pages);
void orc_layer_release(orc_layer* L);
/* Reference semantics, including the quirk that a failed allocation stops
 * adding pages while num_cached still grows by count. Returns the number of
 * pages actually added. */
int32_t orc_layer_append_pages(orc_layer* L, int32_t count);
void orc_layer_reset(orc_layer* L);

/* Scatter S new tokens of K and V ([Hkv][S][D] contiguous, elem bytes each)
 * into the pools (page layout [slot 16][Hkv][D]), allocating pages first. */
void orc_layer_append_kv(orc_layer* L, uint8_t* k_pool_base, uint8_t* v_pool_base,
                         const uint8_t* K, const uint8_t* V, int32_t n_kv_heads,
                         int32_t seq_len, int32_t head_dim, int32_t elem_bytes);

/* Attention over the pages of one layer, loop order and arithmetic exactly
 * as the reference CPU op, stopping before the final store in Q's dtype.
 * q: [Hq][S][D] (batch 1) in dtype; out: [Hq][S][D] fp32. */
void orc_paged_attention_f32(const uint8_t* q, int32_t dtype, const uint8_t* k_pool_base,
                             const uint8_t* v_pool_base, const int32_t* k_ids,
                             const int32_t* v_ids, int32_t n_pages, int32_t total_cached,
                             int32_t n_q_heads, int32_t n_kv_heads, int32_t seq_len,
                             int32_t head_dim, int32_t n_kv_groups, float scale, int causal,
                             float* out);

/* Same, parallelised over (head, query) rows with pthreads (used only as the
 * timed CPU baseline when the reference build is absent). */
void orc_paged_attention_f32_mt(const uint8_t* q, int32_t dtype, const uint8_t* k_pool_base,
                                const uint8_t* v_pool_base, const int32_t* k_ids,
                                const int32_t* v_ids, int32_t n_pages, int32_t total_cached,
                                int32_t n_q_heads, int32_t n_kv_heads, int32_t seq_len,
                                int32_t head_dim, int32_t n_kv_groups, float scale, int causal,
                                float* out, int32_t n_threads);

/* Only the output rows listed (row r = head * S + query), out[i][D]. */
void orc_paged_attention_rows(const uint8_t* q, int32_t dtype, const uint8_t* k_pool_base,
                              const uint8_t* v_pool_base, const int32_t* k_ids,
                              const int32_t* v_ids, int32_t n_pages, int32_t total_cached,
                              int32_t n_q_heads, int32_t n_kv_heads, int32_t seq_len,
                              int32_t head_dim, int32_t n_kv_groups, float scale, int causal,
                              const int32_t* rows, int32_t n_rows, float* out, int32_t n_threads);

/* qk_rope_oracle.c: per-head RMSNorm (QK-norm) and RoPE, bf16 in and out. */
void orc_rms_norm_bf16(const uint16_t* x, const float* w, uint16_t* out, int64_t rows, int64_t dim, float eps);
void orc_apply_rope_bf16(const uint16_t* x, uint16_t* out, const float* cos_tab, const float* sin_tab,
                         int64_t n_heads, int64_t seq, int64_t head_dim, int64_t start_pos);
void orc_rope_cache(float theta, int32_t head_dim, int32_t max_seq, float* cos_out, float* sin_out);

/* flash_oracle.c: the non-paged attention op (self-attention over one chunk),
 * q [B][Hq][S][D], k/v [B][Hkv][S][D] bf16; out [B][Hq][S][D] fp32. */
void orc_flash_attention_f32(const uint16_t* q, const uint16_t* k, const uint16_t* v, int32_t batch, int32_t Hq,
                             int32_t Hkv, int32_t S, int32_t D, int32_t groups, float scale, int causal,
                             float* out);

/* kv_format_oracle.c: KV export / import between pages and dense head-major
 * [Hkv][tokens][D] (bf16, or OCP e4m3 with per (head, 16-token block) fp32
 * scales [Hkv][blocks]). */
uint8_t orc_e4m3_from_f32(float f);
float orc_e4m3_to_f32(uint8_t b);
void orc_export_kv(const uint16_t* k_pool_base, const uint16_t* v_pool_base, const int32_t* k_ids,
                   const int32_t* v_ids, int32_t n_tokens, int32_t n_kv_heads, int32_t head_dim, int fp8,
                   void* k_out, void* v_out, float* k_scales, float* v_scales);
void orc_import_fp8(uint16_t* k_pool_base, uint16_t* v_pool_base, const int32_t* k_ids, const int32_t* v_ids,
                    int32_t n_prior, const uint8_t* k_in, const uint8_t* v_in, const float* k_scales,
                    const float* v_scales, int32_t seq_len, int32_t n_kv_heads, int32_t head_dim);

/* Round an fp32 buffer to the reference's bf16 (RNE, subnormals to signed 0). */
void orc_round_bf16(const float* in, uint16_t* out, size_t n);

#ifdef __cplusplus
}
#endif
#endif
