/*
 * paged_oracle.c — CPU restatement of Genllm's paged KV-cache path.
 * TEST INFRASTRUCTURE ONLY (see paged_oracle.h). Reference line citations are
 * relative to the Genllm source tree.
 */
#include "paged_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---- number formats ---------------------------------------------------- */

/* include/utils/bfloat16.hpp:18-41: round to nearest even on the dropped 16
 * bits; exponent 0 (zero or subnormal) becomes signed zero; NaN keeps only a
 * single mantissa bit; rounding past the largest finite value gives inf. */
uint16_t orc_bf16_from_f32(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    uint32_t sign = u >> 31, e = (u >> 23) & 0xFFu, m = u & 0x7FFFFFu;
    if (e == 0xFFu) return (uint16_t)((sign << 15) | 0x7F80u | (m ? 1u : 0u));
    if (e == 0) return (uint16_t)(sign << 15);
    uint32_t low = u & 0xFFFFu;
    uint32_t up = (low > 0x8000u) || (low == 0x8000u && (m & 0x10000u));
    uint32_t hm = (m >> 16) + up;
    if (hm >= 0x80u) {
        hm = 0;
        e += 1;
        if (e >= 0xFFu) return (uint16_t)((sign << 15) | 0x7F80u);
    }
    return (uint16_t)((sign << 15) | (e << 7) | hm);
}

/* include/utils/bfloat16.hpp:42-45 */
float orc_bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* IEEE binary16 -> binary32 (include/utils/float16.hpp f16_bits_to_float). */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, u;
    if (e == 0) {
        if (m == 0) {
            u = sign << 31;
        } else {
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; ++sh; }
            u = (sign << 31) | ((uint32_t)(113 - sh) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        u = (sign << 31) | 0x7F800000u | (m ? 0x400000u : 0u);
    } else {
        u = (sign << 31) | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline float load_elem(const uint8_t* p, int32_t dtype) {
    if (dtype == ORC_BF16) { uint16_t b; memcpy(&b, p, 2); return orc_bf16_to_f32(b); }
    if (dtype == ORC_F16) { uint16_t b; memcpy(&b, p, 2); return orc_f16_to_f32(b); }
    float f; memcpy(&f, p, 4); return f;
}

static inline int32_t elem_bytes(int32_t dtype) { return dtype == ORC_F32 ? 4 : 2; }

void orc_round_bf16(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = orc_bf16_from_f32(in[i]);
}

/* ---- BlockPool: src/core/page_attention.cpp:25-64 ----------------------- */

int orc_pool_init(orc_pool* p, int32_t capacity) {
    p->capacity = capacity;
    p->num_blocks = 0;
    p->n_free = 0;
    p->free_list = (int32_t*)malloc(sizeof(int32_t) * (size_t)(capacity > 0 ? capacity : 1));
    return p->free_list ? 0 : -1;
}

void orc_pool_release(orc_pool* p) {
    free(p->free_list);
    p->free_list = NULL;
}

/* :38-47 — pop the most recently freed id; otherwise hand out the next never
 * used id; -1 once capacity is reached. */
int32_t orc_pool_alloc(orc_pool* p) {
    if (p->n_free > 0) return p->free_list[--p->n_free];
    if (p->capacity > 0 && p->num_blocks >= p->capacity) return -1;
    return p->num_blocks++;
}

/* :49-52 — ids never handed out are ignored. Like the reference, a double
 * free is not detected (the list is bounded here to stay memory safe). */
void orc_pool_free(orc_pool* p, int32_t id) {
    if (id >= 0 && id < p->num_blocks && p->n_free < p->capacity) p->free_list[p->n_free++] = id;
}

/* :54-58 — every id ever handed out goes back, ascending, so the next alloc
 * returns the highest id. */
void orc_pool_reset(orc_pool* p) {
    p->n_free = 0;
    for (int32_t i = 0; i < p->num_blocks; ++i) p->free_list[p->n_free++] = i;
}

/* ---- page table: src/core/page_attention.cpp:141-162, 209-216 ---------- */

int orc_layer_init(orc_layer* L, int32_t max_pages) {
    memset(L, 0, sizeof(*L));
    L->table_cap = max_pages + 1;
    L->k_ids = (int32_t*)calloc((size_t)L->table_cap, sizeof(int32_t));
    L->v_ids = (int32_t*)calloc((size_t)L->table_cap, sizeof(int32_t));
    if (!L->k_ids || !L->v_ids) return -1;
    if (orc_pool_init(&L->k_pool, max_pages) || orc_pool_init(&L->v_pool, max_pages)) return -1;
    return 0;
}

void orc_layer_release(orc_layer* L) {
    free(L->k_ids);
    free(L->v_ids);
    orc_pool_release(&L->k_pool);
    orc_pool_release(&L->v_pool);
}

int32_t orc_layer_append_pages(orc_layer* L, int32_t count) {
    int32_t added = 0;
    if (count <= 0) return 0;
    for (int32_t p = 0; p < count; ++p) {
        int32_t pos = L->num_cached + p;
        if (pos % ORC_PAGE_SLOTS != 0) continue;
        int32_t kid = orc_pool_alloc(&L->k_pool);
        int32_t vid = orc_pool_alloc(&L->v_pool);
        if (kid < 0 || vid < 0) break; /* :155 */
        if (pos / ORC_PAGE_SLOTS >= L->n_pages && L->n_pages < L->table_cap) {
            L->k_ids[L->n_pages] = kid;
            L->v_ids[L->n_pages] = vid;
            L->n_pages++;
            added++;
        }
    }
    L->num_cached += count; /* :161 — grows even when allocation failed */
    return added;
}

void orc_layer_reset(orc_layer* L) {
    L->num_cached = 0;
    L->n_pages = 0;
    orc_pool_reset(&L->k_pool);
    orc_pool_reset(&L->v_pool);
}

/* src/core/page_attention.cpp:104-139: token p of head h lands at
 * page(table[(prev+p)/16]) + ((prev+p)%16 * Hkv + h) * D elements. */
void orc_layer_append_kv(orc_layer* L, uint8_t* k_pool_base, uint8_t* v_pool_base,
                         const uint8_t* K, const uint8_t* V, int32_t n_kv_heads,
                         int32_t seq_len, int32_t head_dim, int32_t eb) {
    if (seq_len <= 0) return;
    int32_t prev = L->num_cached;
    size_t row = (size_t)head_dim * (size_t)eb;
    size_t page_bytes = (size_t)ORC_PAGE_SLOTS * (size_t)n_kv_heads * row;
    orc_layer_append_pages(L, seq_len);
    for (int32_t p = 0; p < seq_len; ++p) {
        int32_t pos = prev + p;
        int32_t lp = pos / ORC_PAGE_SLOTS, off = pos % ORC_PAGE_SLOTS;
        if (lp >= L->n_pages) break; /* the reference would index out of bounds here */
        uint8_t* kd = k_pool_base + (size_t)L->k_ids[lp] * page_bytes + (size_t)off * n_kv_heads * row;
        uint8_t* vd = v_pool_base + (size_t)L->v_ids[lp] * page_bytes + (size_t)off * n_kv_heads * row;
        for (int32_t h = 0; h < n_kv_heads; ++h) {
            memcpy(kd + (size_t)h * row, K + ((size_t)h * seq_len + p) * row, row);
            memcpy(vd + (size_t)h * row, V + ((size_t)h * seq_len + p) * row, row);
        }
    }
}

/* ---- attention: src/backend/cpu/attention.cpp:156-215 ------------------- */

/* One output row r = h * S + sq. The bf16 path converts Q once per row and
 * each K/V element as it is used; the float operations and their order are
 * exactly the reference loop's (the conversions are exact). */
static void attend_one(const uint8_t* q, int32_t dtype, const uint8_t* kb, const uint8_t* vb,
                       const int32_t* k_ids, const int32_t* v_ids, int32_t n_pages, int32_t total,
                       int32_t Hkv, int32_t S, int32_t D, int32_t groups, float scale, int causal,
                       int32_t r, float* orow, float* o, float* qf) {
    int32_t eb = elem_bytes(dtype);
    size_t page_elems = (size_t)ORC_PAGE_SLOTS * Hkv * D;
    int32_t h = r / S, sq = r % S;
    int32_t kvh = h / groups;
    float m = -INFINITY, l = 0.0f;
    for (int32_t d = 0; d < D; ++d) o[d] = 0.0f;
    int32_t q_abs = total - S + sq;
    int32_t limit = causal ? q_abs : total - 1;
    const uint8_t* qrow = q + (((size_t)h * S + sq) * D) * eb;
    for (int32_t d = 0; d < D; ++d) qf[d] = load_elem(qrow + (size_t)d * eb, dtype);
    for (int32_t blk = 0; blk < n_pages; ++blk) {
        int32_t start = blk * ORC_PAGE_SLOTS;
        int32_t end = start + ORC_PAGE_SLOTS < total ? start + ORC_PAGE_SLOTS : total;
        if (start > limit) break;
        const uint8_t* kp = kb + (size_t)k_ids[blk] * page_elems * eb;
        const uint8_t* vp = vb + (size_t)v_ids[blk] * page_elems * eb;
        for (int32_t s = 0; s < end - start; ++s) {
            if (causal && start + s > q_abs) break;
            size_t off = ((size_t)s * Hkv + kvh) * D;
            float score = 0.0f;
            if (dtype == ORC_BF16) {
                const uint16_t* kr = (const uint16_t*)(kp + off * 2);
                for (int32_t d = 0; d < D; ++d) score += qf[d] * orc_bf16_to_f32(kr[d]);
            } else {
                for (int32_t d = 0; d < D; ++d) score += qf[d] * load_elem(kp + (off + d) * eb, dtype);
            }
            score *= scale;
            float mp = m;
            m = fmaxf(m, score);
            float es = expf(score - m);
            float ep = expf(mp - m);
            if (dtype == ORC_BF16) {
                const uint16_t* vr = (const uint16_t*)(vp + off * 2);
                for (int32_t d = 0; d < D; ++d) o[d] = o[d] * ep + es * orc_bf16_to_f32(vr[d]);
            } else {
                for (int32_t d = 0; d < D; ++d) o[d] = o[d] * ep + es * load_elem(vp + (off + d) * eb, dtype);
            }
            l = l * ep + es;
        }
    }
    float inv = 1.0f / l;
    for (int32_t d = 0; d < D; ++d) orow[d] = o[d] * inv;
}

/* Rows rows[i0..i1) (or r = i0..i1 when rows is NULL) into out[i][D]. */
static void attend_rows(const uint8_t* q, int32_t dtype, const uint8_t* kb, const uint8_t* vb,
                        const int32_t* k_ids, const int32_t* v_ids, int32_t n_pages, int32_t total,
                        int32_t Hq, int32_t Hkv, int32_t S, int32_t D, int32_t groups, float scale,
                        int causal, float* out, int32_t i0, int32_t i1, const int32_t* rows) {
    (void)Hq;
    float* o = (float*)malloc(sizeof(float) * (size_t)D * 2);
    for (int32_t i = i0; i < i1; ++i) {
        int32_t r = rows ? rows[i] : i;
        attend_one(q, dtype, kb, vb, k_ids, v_ids, n_pages, total, Hkv, S, D, groups, scale, causal, r,
                   out + (size_t)i * D, o, o + D);
    }
    free(o);
}

void orc_paged_attention_f32(const uint8_t* q, int32_t dtype, const uint8_t* kb,
                             const uint8_t* vb, const int32_t* k_ids, const int32_t* v_ids,
                             int32_t n_pages, int32_t total, int32_t Hq, int32_t Hkv, int32_t S,
                             int32_t D, int32_t groups, float scale, int causal, float* out) {
    attend_rows(q, dtype, kb, vb, k_ids, v_ids, n_pages, total, Hq, Hkv, S, D, groups, scale,
                causal, out, 0, Hq * S, NULL);
}

typedef struct {
    const uint8_t *q, *kb, *vb;
    const int32_t *k_ids, *v_ids, *rows;
    int32_t dtype, n_pages, total, Hq, Hkv, S, D, groups, causal, row0, row1;
    float scale;
    float* out;
} orc_job;

static void* orc_job_run(void* a) {
    orc_job* j = (orc_job*)a;
    attend_rows(j->q, j->dtype, j->kb, j->vb, j->k_ids, j->v_ids, j->n_pages, j->total, j->Hq,
                j->Hkv, j->S, j->D, j->groups, j->scale, j->causal, j->out, j->row0, j->row1, j->rows);
    return NULL;
}

static void run_threads(const uint8_t* q, int32_t dtype, const uint8_t* kb, const uint8_t* vb,
                        const int32_t* k_ids, const int32_t* v_ids, int32_t n_pages, int32_t total,
                        int32_t Hq, int32_t Hkv, int32_t S, int32_t D, int32_t groups, float scale,
                        int causal, float* out, int32_t n_rows, const int32_t* rows,
                        int32_t n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > n_rows) n_threads = n_rows > 0 ? n_rows : 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)n_threads);
    orc_job* jobs = (orc_job*)malloc(sizeof(orc_job) * (size_t)n_threads);
    for (int32_t t = 0; t < n_threads; ++t) {
        orc_job j = {q, kb, vb, k_ids, v_ids, rows, dtype, n_pages, total, Hq, Hkv, S, D, groups,
                     causal, (int32_t)((int64_t)n_rows * t / n_threads),
                     (int32_t)((int64_t)n_rows * (t + 1) / n_threads), scale, out};
        jobs[t] = j;
        pthread_create(&th[t], NULL, orc_job_run, &jobs[t]);
    }
    for (int32_t t = 0; t < n_threads; ++t) pthread_join(th[t], NULL);
    free(th);
    free(jobs);
}

void orc_paged_attention_f32_mt(const uint8_t* q, int32_t dtype, const uint8_t* kb,
                                const uint8_t* vb, const int32_t* k_ids, const int32_t* v_ids,
                                int32_t n_pages, int32_t total, int32_t Hq, int32_t Hkv,
                                int32_t S, int32_t D, int32_t groups, float scale, int causal,
                                float* out, int32_t n_threads) {
    run_threads(q, dtype, kb, vb, k_ids, v_ids, n_pages, total, Hq, Hkv, S, D, groups, scale,
                causal, out, Hq * S, NULL, n_threads);
}

void orc_paged_attention_rows(const uint8_t* q, int32_t dtype, const uint8_t* kb,
                              const uint8_t* vb, const int32_t* k_ids, const int32_t* v_ids,
                              int32_t n_pages, int32_t total, int32_t Hq, int32_t Hkv, int32_t S,
                              int32_t D, int32_t groups, float scale, int causal,
                              const int32_t* rows, int32_t n_rows, float* out,
                              int32_t n_threads) {
    run_threads(q, dtype, kb, vb, k_ids, v_ids, n_pages, total, Hq, Hkv, S, D, groups, scale,
                causal, out, n_rows, rows, n_threads);
}
