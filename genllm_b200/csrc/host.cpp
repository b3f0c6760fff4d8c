// host.cpp — the C ABI (include/genllm_kv.h): page allocators, block tables,
// layer state and kernel dispatch for the B200 paged KV-cache path.
//
// Mirrors the reference's BlockPool / PagedAttentionManager
// (include/core/page_attention.h:11-89, src/core/page_attention.cpp:25-216)
// and replaces PagedAttentionImpl<Device::CUDA>::execute
// (src/backend/cuda/attention.cu:491-580). The differences are deliberate:
//   * the block table lives on the device and is updated incrementally by the
//     kernels themselves (new entries ride in the launch parameters), instead
//     of a cudaMalloc + H2D + cudaFree of the whole table per call;
//   * an exhausted pool is an error (GKV_ERR_NO_PAGES) that leaves the layer
//     unchanged, where the reference keeps counting tokens and later indexes
//     its table out of bounds (page_attention.cpp:155,161,127);
//   * all work is enqueued on the caller's stream; nothing synchronises.
#include <nvtx3/nvToolsExt.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/genllm_kv.h"
#include "kernels.h"

namespace {

thread_local std::string g_last_error;

// Set by gkv_paged_attention_gather around its call of the managed decode
// path: the fused head all-gather of that one launch.
thread_local const gkv::GatherLaunch* t_gather = nullptr;
// Set by the multi-layer entry points around every layer but the last of a
// step whose layers are distinct: the next launch is another layer's decode.
thread_local bool t_next_other_layer = false;
thread_local bool t_prev_other_layer = false;  // ... and around every layer but the first

int fail(int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(GKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Runs the body with `device` current and restores the caller's device.
class DeviceGuard {
   public:
    explicit DeviceGuard(int device) {
        ok_ = cudaGetDevice(&prev_) == cudaSuccess;
        if (ok_ && prev_ != device) ok_ = cudaSetDevice(device) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (cudaGetDevice(&cur) == cudaSuccess && cur != prev_) cudaSetDevice(prev_);
    }
    bool ok() const { return ok_; }

   private:
    int prev_ = 0;
    bool ok_ = false;
};

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library needs no link-time dependency on libcuda.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// GKV_PREFILL_KERNEL=simt selects the CUDA-core prefill kernel instead of the
// tensor-core one (a cross-check of two independent implementations).
bool prefill_on_cuda_cores() {
    static const bool simt = [] {
        const char* v = getenv("GKV_PREFILL_KERNEL");
        return v && std::strcmp(v, "simt") == 0;
    }();
    return simt;
}

bool is_out_dtype(int d) { return d == GKV_F32 || d == GKV_F16 || d == GKV_BF16; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace gkv {

void set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }

static bool encode(CUtensorMap* m, void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                   const cuuint32_t* box, CUtensorMapSwizzle swz, const char** why) {
    auto enc = tensor_map_encoder();
    if (!enc) {
        *why = "cuTensorMapEncodeTiled unavailable";
        return false;
    }
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        *why = "cuTensorMapEncodeTiled failed";
        return false;
    }
    return true;
}


bool encode_pool_maps_sw128(const PoolView& pool, CUtensorMap* k_map, CUtensorMap* v_map, const char** why) {
    cuuint64_t dims[3] = {(cuuint64_t)kHeadDim, (cuuint64_t)pool.n_kv_heads, (cuuint64_t)pool.pool_pages * 16};
    cuuint64_t strides[2] = {(cuuint64_t)kHeadDim * 2, (cuuint64_t)pool.n_kv_heads * kHeadDim * 2};
    cuuint32_t box[3] = {64, 1, 16};
    return encode(k_map, pool.k_base, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, why) &&
           encode(v_map, pool.v_base, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, why);
}

bool encode_decode_maps(const PoolView& pool, DecodeMaps* m, const char** why) {
    if (!encode_pool_maps_sw128(pool, &m->k_head, &m->v_head, why)) return false;
    // [slots][heads][128] viewed as (dims, slots, heads): a box {64, 16, Hkv}
    // lands in shared memory as [head][slot][64 dims].
    cuuint64_t dims[3] = {(cuuint64_t)kHeadDim, (cuuint64_t)pool.pool_pages * kPageSlots, (cuuint64_t)pool.n_kv_heads};
    cuuint64_t strides[2] = {(cuuint64_t)pool.n_kv_heads * kHeadDim * 2, (cuuint64_t)kHeadDim * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)kPageSlots, (cuuint32_t)pool.n_kv_heads};
    return encode(&m->k_page, pool.k_base, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, why) &&
           encode(&m->v_page, pool.v_base, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, why);
}

bool encode_pool_run_maps_sw128(const PoolView& pool, CUtensorMap* k_map, CUtensorMap* v_map, const char** why) {
    cuuint64_t dims[3] = {(cuuint64_t)kHeadDim, (cuuint64_t)pool.n_kv_heads, (cuuint64_t)pool.pool_pages * 16};
    cuuint64_t strides[2] = {(cuuint64_t)kHeadDim * 2, (cuuint64_t)pool.n_kv_heads * kHeadDim * 2};
    cuuint32_t box[3] = {64, 1, (cuuint32_t)kRunSlots};
    return encode(k_map, pool.k_base, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, why) &&
           encode(v_map, pool.v_base, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, why);
}

bool encode_contig_kv_maps_sw128(const uint16_t* k, const uint16_t* v, int32_t rows_per_head, int32_t heads,
                                 CUtensorMap* k_map, CUtensorMap* v_map, const char** why) {
    cuuint64_t dims[3] = {(cuuint64_t)kHeadDim, (cuuint64_t)rows_per_head, (cuuint64_t)heads};
    cuuint64_t strides[2] = {(cuuint64_t)kHeadDim * 2, (cuuint64_t)rows_per_head * kHeadDim * 2};
    cuuint32_t box[3] = {64, 128, 1};
    return encode(k_map, const_cast<uint16_t*>(k), 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, why) &&
           encode(v_map, const_cast<uint16_t*>(v), 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, why);
}

bool encode_q_map_sw128(const uint16_t* q, int32_t n_q_heads, int32_t seq_len, CUtensorMap* q_map,
                        const char** why) {
    cuuint64_t dims[3] = {(cuuint64_t)kHeadDim, (cuuint64_t)seq_len, (cuuint64_t)n_q_heads};
    cuuint64_t strides[2] = {(cuuint64_t)kHeadDim * 2, (cuuint64_t)seq_len * kHeadDim * 2};
    cuuint32_t box[3] = {64, 128, 1};
    return encode(q_map, const_cast<uint16_t*>(q), 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, why);
}

}  // namespace gkv

// ============================ raw tier ======================================

// NVTX range around a host entry point (the launches it enqueues): names
// the path's phases (append, decode, merge, gather, export) in a timeline
// profiler; a no-op unless a tool is attached.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

struct gkv_table {
    int device = 0;
    int32_t capacity = 0;
    int num_sms = 148;
    int2* d_table = nullptr;
    gkv::Scratch scratch{};
    // Tensor maps cached for the last pool seen.
    void* map_k_base = nullptr;
    void* map_v_base = nullptr;
    int32_t map_pages = -1;
    int32_t map_heads = -1;
    CUtensorMap k_map_sw;   // box {64 dims, 1 head, 16 slots}, 128-byte swizzle
    gkv::DecodeMaps dmaps;  // the decode kernel's maps of the same pool
    uint32_t posted = 0;    // decode steps numbered so far (completion word protocol, kernels.h)
    CUtensorMap v_map_sw;
    CUtensorMap k_map_run;  // box {64 dims, 1 head, 128 slots}: 8 pages with consecutive ids
    CUtensorMap v_map_run;
    bool runs = false;      // run maps valid (the pool holds at least 8 pages)
    void* qk_buf = nullptr;  // normalised / rotated / permuted Q, K, V of a chunk (gkv_paged_attention_raw_qknorm)
    size_t qk_bytes = 0;
    // Q tensor maps of recent chunk calls, keyed by (pointer, heads, rows):
    // an executor reuses its activation buffers, and encoding a map is a
    // driver call on every chunk otherwise.
    struct QMap {
        const void* q = nullptr;
        int32_t heads = 0, rows = 0;
        CUtensorMap map;
    };
    QMap qmaps[16];
    int qmap_next = 0;
    // The same for the chunk's K/V inputs (the prefill reads the chunk's own
    // tiles from them), keyed by (K, V, heads, rows).
    struct KvMap {
        const void* k = nullptr;
        const void* v = nullptr;
        int32_t heads = 0, rows = 0;
        CUtensorMap maps[2];
    };
    KvMap kvmaps[16];
    int kvmap_next = 0;
};

namespace {

void table_free(gkv_table* t) {
    cudaFree(t->d_table);
    cudaFree(t->scratch.part_acc);
    cudaFree(t->scratch.part_ml);
    cudaFree(t->scratch.err);
    cudaFree(t->qk_buf);
}

constexpr int kMaxKvHeads = 256;

int check_pool(const gkv_pool_desc* pool) {
    if (!pool) return fail(GKV_ERR_INVALID, "null pool descriptor");
    if (pool->head_dim != 128)
        return fail(GKV_ERR_UNSUPPORTED, "head_dim %d: only 128 is built", pool->head_dim);
    if (pool->dtype != GKV_BF16)
        return fail(GKV_ERR_UNSUPPORTED, "KV dtype %d: only bf16 (30) is built", pool->dtype);
    if (pool->n_kv_heads < 1 || pool->n_kv_heads > kMaxKvHeads)
        return fail(GKV_ERR_INVALID, "n_kv_heads %d out of range", pool->n_kv_heads);
    if (pool->pool_pages < 1) return fail(GKV_ERR_INVALID, "pool_pages %d", pool->pool_pages);
    if (!pool->k_base || !pool->v_base || !aligned16(pool->k_base) || !aligned16(pool->v_base))
        return fail(GKV_ERR_INVALID, "pool bases must be non-null and 16-byte aligned");
    return GKV_OK;
}

int table_maps(gkv_table* t, const gkv_pool_desc* pool) {
    if (t->map_k_base == pool->k_base && t->map_v_base == pool->v_base &&
        t->map_pages == pool->pool_pages && t->map_heads == pool->n_kv_heads)
        return GKV_OK;
    gkv::PoolView pv{static_cast<uint16_t*>(pool->k_base), static_cast<uint16_t*>(pool->v_base),
                     pool->pool_pages, pool->n_kv_heads};
    const char* why = nullptr;
    if (!gkv::encode_pool_maps_sw128(pv, &t->k_map_sw, &t->v_map_sw, &why) ||
        !gkv::encode_decode_maps(pv, &t->dmaps, &why))
        return fail(GKV_ERR_CUDA, "%s", why);
    t->runs = pool->pool_pages * 16 >= gkv::kRunSlots;
    if (t->runs && !gkv::encode_pool_run_maps_sw128(pv, &t->k_map_run, &t->v_map_run, &why))
        return fail(GKV_ERR_CUDA, "%s", why);
    t->map_k_base = pool->k_base;
    t->map_v_base = pool->v_base;
    t->map_pages = pool->pool_pages;
    t->map_heads = pool->n_kv_heads;
    return GKV_OK;
}

// Validate a table delta against a step that ends with n_pages logical pages.
int check_new_pages(const gkv_table* t, const gkv_new_pages* np, int32_t n_pages, int32_t pool_pages) {
    if (n_pages > t->capacity)
        return fail(GKV_ERR_NO_PAGES, "step needs %d table entries, table holds %d", n_pages, t->capacity);
    if (!np || np->n_new_pages == 0) return GKV_OK;
    if (np->n_new_pages < 0 || np->first_new_page < 0 || !np->k_ids || !np->v_ids ||
        np->first_new_page + np->n_new_pages > t->capacity)
        return fail(GKV_ERR_INVALID, "bad new-page list");
    for (int i = 0; i < np->n_new_pages; ++i)
        if (np->k_ids[i] < 0 || np->k_ids[i] >= pool_pages || np->v_ids[i] < 0 || np->v_ids[i] >= pool_pages)
            return fail(GKV_ERR_INVALID, "new page id out of the pool");
    return GKV_OK;
}

gkv::NewPages pack(const gkv_new_pages* np, int32_t from, int32_t n) {
    gkv::NewPages out;
    out.first = np ? np->first_new_page + from : 0;
    out.n = n;
    for (int i = 0; i < n; ++i) out.ids[i] = make_int2(np->k_ids[from + i], np->v_ids[from + i]);
    return out;
}

// Publish new-page entries [from, to) of np: table-only launches, or one
// upload when there are many.
int publish(const gkv_pool_desc* pool, gkv_table* t, const gkv_new_pages* np, int32_t from, int32_t to,
            cudaStream_t s) {
    gkv::PoolView pv{static_cast<uint16_t*>(pool->k_base), static_cast<uint16_t*>(pool->v_base),
                     pool->pool_pages, pool->n_kv_heads};
    if (to - from > gkv::kMaxNewPagesPerLaunch) {
        // Many entries (an import of a long sequence, a long host-only
        // growth): one stream-ordered upload instead of a launch per 64.
        // Pageable source: the copy is staged before this call returns.
        std::vector<int2> dev(to - from);
        for (int32_t i = from; i < to; ++i) dev[i - from] = make_int2(np->k_ids[i], np->v_ids[i]);
        cudaError_t e = cudaMemcpyAsync(t->d_table + np->first_new_page + from, dev.data(), sizeof(int2) * dev.size(),
                                        cudaMemcpyHostToDevice, s);
        return e == cudaSuccess ? GKV_OK : cuda_fail(e, "table upload");
    }
    while (from < to) {
        const int32_t n = std::min<int32_t>(to - from, gkv::kMaxNewPagesPerLaunch);
        gkv::NewPages p = pack(np, from, n);
        cudaError_t e = gkv::launch_append(pv, t->d_table, p, nullptr, nullptr, 0, 0, 0, 0, t->scratch.err, s);
        if (e != cudaSuccess) return cuda_fail(e, "table publish launch");
        from += n;
    }
    return GKV_OK;
}

// for_prefill: the chunked-prefill kernel follows (it waits for the
// appends): the appends are launched as programmatic dependents and the last
// one lets the prefill start its launch and setup early.
int append_chunks(const gkv_pool_desc* pool, gkv_table* t, int32_t n_prior, const gkv_new_pages* np,
                  const void* K, const void* V, int32_t seq_len, cudaStream_t s, bool for_prefill = false) {
    gkv::PoolView pv{static_cast<uint16_t*>(pool->k_base), static_cast<uint16_t*>(pool->v_base),
                     pool->pool_pages, pool->n_kv_heads};
    // Launch in chunks of at most 64 pages (1024 tokens) so that each launch's
    // new table entries fit in its parameters. Tokens of chunk c live in
    // logical pages [(n_prior + c0)/16, ...]; entries of the new-page list
    // that a chunk touches ride with it.
    const int32_t n_new = np ? np->n_new_pages : 0;
    const int32_t first_new = np ? np->first_new_page : 0;
    int32_t published = 0;  // entries of np already sent
    const int32_t chunk = gkv::kMaxNewPagesPerLaunch * 16 - 16;
    for (int32_t c0 = 0; c0 < seq_len; c0 += chunk) {
        const int32_t c1 = std::min(seq_len, c0 + chunk);
        const int32_t last_page = (n_prior + c1 - 1) / 16;  // inclusive
        const int32_t upto = std::min(n_new, std::max(published, last_page - first_new + 1));
        // Entries pending from earlier host-only growth go out first.
        if (upto - published > gkv::kMaxNewPagesPerLaunch) {
            const int32_t to = upto - gkv::kMaxNewPagesPerLaunch;
            const int st = publish(pool, t, np, published, to, s);
            if (st) return st;
            published = to;
        }
        gkv::NewPages p = pack(np, published, upto - published);
        const bool last = c1 >= seq_len && upto >= n_new;
        const int pdl = for_prefill ? gkv::kAppendDependent | (last ? gkv::kAppendTrigger : 0) : 0;
        cudaError_t e = gkv::launch_append(pv, t->d_table, p, static_cast<const uint16_t*>(K),
                                           static_cast<const uint16_t*>(V), n_prior, seq_len, c0, c1,
                                           t->scratch.err, s, pdl);
        if (e != cudaSuccess) return cuda_fail(e, "append launch");
        published = upto;
    }
    if (published < n_new) return publish(pool, t, np, published, n_new, s);
    return GKV_OK;
}

}  // namespace

extern "C" {

const char* gkv_status_string(int s) {
    switch (s) {
        case GKV_OK: return "ok";
        case GKV_ERR_INVALID: return "invalid argument";
        case GKV_ERR_NO_PAGES: return "page pool exhausted";
        case GKV_ERR_CUDA: return "CUDA error";
        case GKV_ERR_UNSUPPORTED: return "unsupported configuration";
        case GKV_ERR_STATE: return "layer not initialised or reserved";
        case GKV_ERR_DEVICE: return "device-side error flagged";
        default: return "unknown status";
    }
}

const char* gkv_last_error(void) { return g_last_error.c_str(); }

int gkv_table_create(int device, int32_t capacity, gkv_table** out) {
    if (!out || capacity < 1) return fail(GKV_ERR_INVALID, "gkv_table_create: bad arguments");
    DeviceGuard g(device);
    if (!g.ok()) return fail(GKV_ERR_CUDA, "cannot select device %d", device);
    auto* t = new gkv_table();
    t->device = device;
    t->capacity = capacity;
    cudaDeviceGetAttribute(&t->num_sms, cudaDevAttrMultiProcessorCount, device);
    cudaError_t e;
    t->scratch.err = nullptr;
    if ((e = cudaMalloc(&t->d_table, sizeof(int2) * (size_t)capacity)) != cudaSuccess ||
        (e = cudaMemset(t->d_table, 0xFF, sizeof(int2) * (size_t)capacity)) != cudaSuccess ||
        (e = cudaMalloc(&t->scratch.part_acc, sizeof(float) * gkv::kMaxPartialRows * 128)) != cudaSuccess ||
        (e = cudaMalloc(&t->scratch.part_ml, sizeof(float2) * gkv::kMaxPartialRows)) != cudaSuccess ||
        (e = cudaMalloc(&t->scratch.err, 256)) != cudaSuccess ||
        (e = cudaMemset(t->scratch.err, 0, 256)) != cudaSuccess) {
        table_free(t);
        delete t;
        return cuda_fail(e, "gkv_table_create");
    }
    t->scratch.done = t->scratch.err + 32;   // its own 128-byte line beside the error word
    t->scratch.merge = t->scratch.err + 48;  // fused split merge counters
    *out = t;
    return GKV_OK;
}

int gkv_table_destroy(gkv_table* t) {
    if (!t) return GKV_OK;
    DeviceGuard g(t->device);
    table_free(t);
    delete t;
    return GKV_OK;
}

const int32_t* gkv_table_device_ptr(const gkv_table* t) {
    return t ? reinterpret_cast<const int32_t*>(t->d_table) : nullptr;
}

int gkv_table_check_errors(gkv_table* t, uint32_t* flags) {
    if (!t) return fail(GKV_ERR_INVALID, "null table");
    DeviceGuard g(t->device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "synchronise");
    uint32_t v = 0;
    if ((e = cudaMemcpy(&v, t->scratch.err, 4, cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(e, "read error word");
    if ((e = cudaMemset(t->scratch.err, 0, 4)) != cudaSuccess) return cuda_fail(e, "clear error word");
    if (flags) *flags = v;
    return GKV_OK;
}

int gkv_append_kv_raw(const gkv_pool_desc* pool, gkv_table* t, int32_t n_prior, const gkv_new_pages* np,
                      const void* K, const void* V, int32_t seq_len, gkv_stream_t stream) {
    NvtxRange nvtx_range("gkv append");
    int st = check_pool(pool);
    if (st) return st;
    if (!t || n_prior < 0 || seq_len < 0) return fail(GKV_ERR_INVALID, "gkv_append_kv_raw: bad arguments");
    if (seq_len > 0 && (!K || !V || !aligned16(K) || !aligned16(V)))
        return fail(GKV_ERR_INVALID, "K/V must be non-null and 16-byte aligned");
    const int32_t n_pages = (n_prior + seq_len + 15) / 16;
    if ((st = check_new_pages(t, np, n_pages, pool->pool_pages))) return st;
    DeviceGuard g(t->device);
    if (!g.ok()) return fail(GKV_ERR_CUDA, "cannot select device %d", t->device);
    return append_chunks(pool, t, n_prior, np, K, V, seq_len, reinterpret_cast<cudaStream_t>(stream));
}

namespace {
int check_format_buffers(int32_t format, const void* K, const void* V, const void* ks, const void* vs) {
    if (format != GKV_KV_BF16 && format != GKV_KV_FP8_E4M3) return fail(GKV_ERR_INVALID, "unknown KV format %d", format);
    if (!K || !V || !aligned16(K) || !aligned16(V))
        return fail(GKV_ERR_INVALID, "K/V buffers must be non-null and 16-byte aligned");
    if (format == GKV_KV_FP8_E4M3 &&
        (!ks || !vs || reinterpret_cast<uintptr_t>(ks) % 4 || reinterpret_cast<uintptr_t>(vs) % 4))
        return fail(GKV_ERR_INVALID, "the fp8 format needs 4-byte aligned scale buffers");
    return GKV_OK;
}
}  // namespace

int gkv_export_kv_raw(const gkv_pool_desc* pool, gkv_table* t, int32_t n_tokens, int32_t format, void* K_out,
                      void* V_out, float* k_scales, float* v_scales, gkv_stream_t stream) {
    NvtxRange nvtx_range("gkv export");
    int st = check_pool(pool);
    if (st) return st;
    if (!t || n_tokens < 0) return fail(GKV_ERR_INVALID, "gkv_export_kv_raw: bad arguments");
    if (format != GKV_KV_BF16 && format != GKV_KV_FP8_E4M3) return fail(GKV_ERR_INVALID, "unknown KV format %d", format);
    if (n_tokens == 0) return GKV_OK;
    if ((st = check_format_buffers(format, K_out, V_out, k_scales, v_scales))) return st;
    const int32_t n_pages = (n_tokens + 15) / 16;
    if (n_pages > t->capacity)
        return fail(GKV_ERR_INVALID, "%d tokens need %d table entries, table holds %d", n_tokens, n_pages, t->capacity);
    DeviceGuard g(t->device);
    if (!g.ok()) return fail(GKV_ERR_CUDA, "cannot select device %d", t->device);
    gkv::PoolView pv{static_cast<uint16_t*>(pool->k_base), static_cast<uint16_t*>(pool->v_base),
                     pool->pool_pages, pool->n_kv_heads};
    cudaError_t e = gkv::launch_export(pv, t->d_table, n_tokens, format == GKV_KV_FP8_E4M3 ? 1 : 0, K_out, V_out,
                                       k_scales, v_scales, t->scratch.err, t->num_sms,
                                       reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? GKV_OK : cuda_fail(e, "export launch");
}

int gkv_import_kv_raw(const gkv_pool_desc* pool, gkv_table* t, int32_t n_prior, const gkv_new_pages* np,
                      int32_t format, const void* K_in, const void* V_in, const float* k_scales,
                      const float* v_scales, int32_t seq_len, gkv_stream_t stream) {
    NvtxRange nvtx_range("gkv import");
    if (format == GKV_KV_BF16) return gkv_append_kv_raw(pool, t, n_prior, np, K_in, V_in, seq_len, stream);
    int st = check_pool(pool);
    if (st) return st;
    if (format != GKV_KV_FP8_E4M3) return fail(GKV_ERR_INVALID, "unknown KV format %d", format);
    if (!t || n_prior < 0 || seq_len < 0) return fail(GKV_ERR_INVALID, "gkv_import_kv_raw: bad arguments");
    if (seq_len > 0 && (st = check_format_buffers(format, K_in, V_in, k_scales, v_scales))) return st;
    const int32_t n_pages = (n_prior + seq_len + 15) / 16;
    if ((st = check_new_pages(t, np, n_pages, pool->pool_pages))) return st;
    DeviceGuard g(t->device);
    if (!g.ok()) return fail(GKV_ERR_CUDA, "cannot select device %d", t->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // The table entries go out first (table-only launch), then the import
    // kernel reads them from the device table.
    if ((st = publish(pool, t, np, 0, np ? np->n_new_pages : 0, s))) return st;
    if (seq_len == 0) return GKV_OK;
    gkv::PoolView pv{static_cast<uint16_t*>(pool->k_base), static_cast<uint16_t*>(pool->v_base),
                     pool->pool_pages, pool->n_kv_heads};
    cudaError_t e = gkv::launch_import_fp8(pv, t->d_table, n_prior, seq_len, K_in, V_in, k_scales, v_scales,
                                           t->scratch.err, t->num_sms, s);
    return e == cudaSuccess ? GKV_OK : cuda_fail(e, "import launch");
}

namespace {
int attention_raw(const gkv_pool_desc* pool, gkv_table* t, int32_t n_prior, const gkv_new_pages* np, const void* Q,
                  const void* K, const void* V, void* out, int32_t n_q_heads, int32_t seq_len, float scale,
                  int32_t causal, int32_t out_dtype, const gkv::QkNorm* qk, gkv_stream_t stream);
}  // namespace

int gkv_paged_attention_raw(const gkv_pool_desc* pool, gkv_table* t, int32_t n_prior, const gkv_new_pages* np,
                            const void* Q, const void* K, const void* V, void* out, int32_t n_q_heads,
                            int32_t seq_len, float scale, int32_t causal, int32_t out_dtype,
                            gkv_stream_t stream) {
    return attention_raw(pool, t, n_prior, np, Q, K, V, out, n_q_heads, seq_len, scale, causal, out_dtype, nullptr,
                         stream);
}

namespace {
// Validate a gkv_qk_norm for positions [start, start + seq_len).
int check_qk(const gkv_qk_norm* qk, int32_t start, int32_t seq_len) {
    if (!qk || !qk->q_norm_w || !qk->k_norm_w || !qk->cos_tab || !qk->sin_tab)
        return fail(GKV_ERR_INVALID, "gkv_qk_norm: null weight or table");
    if (start < 0 || (int64_t)start + seq_len > qk->max_seq)
        return fail(GKV_ERR_INVALID, "positions [%d, %d) exceed the RoPE table (%d rows)", start, start + seq_len,
                    qk->max_seq);
    if (!(qk->eps >= 0.f)) return fail(GKV_ERR_INVALID, "eps %g", (double)qk->eps);
    return GKV_OK;
}

// GKV_DECODE_FUSED_MERGE=1: the decode merges its splits inside its own
// grid (the last CTAs to finish merge) instead of the combine kernel. Off by
// default: measured at 32k it is level with the combine on per-layer calls
// and slower inside a multi-layer step.
bool fused_merge_enabled() {
    static const bool on = [] {
        const char* v = getenv("GKV_DECODE_FUSED_MERGE");
        return v && v[0] == '1';
    }();
    return on;
}

int attention_raw(const gkv_pool_desc* pool, gkv_table* t, int32_t n_prior, const gkv_new_pages* np, const void* Q,
                  const void* K, const void* V, void* out, int32_t n_q_heads, int32_t seq_len, float scale,
                  int32_t causal, int32_t out_dtype, const gkv::QkNorm* qk, gkv_stream_t stream) {
    int st = check_pool(pool);
    if (st) return st;
    if (!t || n_prior < 0 || seq_len < 1 || !Q || !K || !V || !out)
        return fail(GKV_ERR_INVALID, "gkv_paged_attention_raw: bad arguments");
    if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(out))
        return fail(GKV_ERR_INVALID, "Q/K/V/out must be 16-byte aligned");
    if (n_q_heads < 1 || n_q_heads % pool->n_kv_heads != 0)
        return fail(GKV_ERR_INVALID, "n_q_heads %d is not a multiple of n_kv_heads %d", n_q_heads,
                    pool->n_kv_heads);
    const int G = n_q_heads / pool->n_kv_heads;
    if (G != 1 && G != 2 && G != 4 && G != 8)
        return fail(GKV_ERR_UNSUPPORTED, "group size %d: built for 1, 2, 4, 8", G);
    if (!is_out_dtype(out_dtype)) return fail(GKV_ERR_UNSUPPORTED, "out dtype %d", out_dtype);
    const int32_t total = n_prior + seq_len;
    const int32_t n_pages = (total + 15) / 16;
    if ((st = check_new_pages(t, np, n_pages, pool->pool_pages))) return st;
    DeviceGuard g(t->device);
    if (!g.ok()) return fail(GKV_ERR_CUDA, "cannot select device %d", t->device);
    if ((st = table_maps(t, pool))) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    gkv::PoolView pv{static_cast<uint16_t*>(pool->k_base), static_cast<uint16_t*>(pool->v_base),
                     pool->pool_pages, pool->n_kv_heads};

    if (seq_len == 1) {
        NvtxRange nvtx_range("gkv decode (append + attention + split merge)");
        if (pool->n_kv_heads > 8)
            return fail(GKV_ERR_UNSUPPORTED, "decode kernel built for at most 8 kv heads per GPU (got %d)",
                        pool->n_kv_heads);
        // Entries beyond the last 64 go first through table-only launches.
        const int32_t n_new = np ? np->n_new_pages : 0;
        const int32_t keep = std::min<int32_t>(n_new, gkv::kMaxNewPagesPerLaunch);
        if (n_new > keep && (st = publish(pool, t, np, 0, n_new - keep, s))) return st;
        gkv::NewPages p = pack(np, n_new - keep, keep);
        gkv::DecodeLaunch d{};
        d.q = static_cast<const uint16_t*>(Q);
        d.k_new = static_cast<const uint16_t*>(K);
        d.v_new = static_cast<const uint16_t*>(V);
        d.out = out;
        d.out_dtype = out_dtype;
        d.n_q_heads = n_q_heads;
        d.n_prior = n_prior;
        d.total = total;
        d.n_pages = n_pages;
        d.scale = scale;
        d.n_splits = 0;
        d.qk = qk;
        d.next_is_other_layer = t_next_other_layer;
        d.prev_is_other_layer = t_prev_other_layer;
        // A single step (not part of a multi-layer step) numbers itself on
        // the table's completion word, so that its combine can release the
        // next launch at entry.
        d.post_done = !t_next_other_layer && !t_prev_other_layer;
        d.done_seq = t->posted + 1u;
        d.fused_merge = fused_merge_enabled();
        cudaError_t e = gkv::launch_decode(pv, t->dmaps, t->d_table, p, t->scratch, d, t->num_sms, s, t_gather);
        if (e != cudaSuccess) return cuda_fail(e, "decode launch");
        if (d.post_done) t->posted = d.done_seq;
        return GKV_OK;
    }

    {
        NvtxRange nvtx_range("gkv chunk append");
        if ((st = append_chunks(pool, t, n_prior, np, K, V, seq_len, s, !prefill_on_cuda_cores()))) return st;
    }
    NvtxRange nvtx_range("gkv chunk attention");
    gkv::PrefillLaunch pl{};
    pl.q = static_cast<const uint16_t*>(Q);
    pl.out = out;
    pl.out_dtype = out_dtype;
    pl.n_q_heads = n_q_heads;
    pl.seq_len = seq_len;
    pl.total = total;
    pl.n_pages = n_pages;
    pl.scale = scale;
    pl.causal = causal ? 1 : 0;
    cudaError_t e;
    if (prefill_on_cuda_cores()) {
        e = gkv::launch_prefill_simt(pv, t->d_table, pl, t->scratch.err, s);
    } else {
        const CUtensorMap* q_map = nullptr;
        for (const auto& e : t->qmaps)
            if (e.q == pl.q && e.heads == n_q_heads && e.rows == seq_len) q_map = &e.map;
        if (!q_map) {
            auto& e = t->qmaps[t->qmap_next];
            t->qmap_next = (t->qmap_next + 1) % 16;
            const char* why = nullptr;
            e.q = nullptr;
            if (!gkv::encode_q_map_sw128(pl.q, n_q_heads, seq_len, &e.map, &why)) return fail(GKV_ERR_CUDA, "%s", why);
            e.q = pl.q;
            e.heads = n_q_heads;
            e.rows = seq_len;
            q_map = &e.map;
        }
        // The chunk's K/V inputs as tensor maps (16-byte aligned inputs only).
        const CUtensorMap* kv_new = nullptr;
        if ((reinterpret_cast<uintptr_t>(K) | reinterpret_cast<uintptr_t>(V)) % 16 == 0) {
            for (const auto& e : t->kvmaps)
                if (e.k == K && e.v == V && e.heads == pool->n_kv_heads && e.rows == seq_len) kv_new = e.maps;
            if (!kv_new) {
                auto& e = t->kvmaps[t->kvmap_next];
                t->kvmap_next = (t->kvmap_next + 1) % 16;
                const char* why = nullptr;
                e.k = e.v = nullptr;
                if (gkv::encode_contig_kv_maps_sw128(static_cast<const uint16_t*>(K), static_cast<const uint16_t*>(V),
                                                     seq_len, pool->n_kv_heads, &e.maps[0], &e.maps[1], &why)) {
                    e.k = K;
                    e.v = V;
                    e.heads = pool->n_kv_heads;
                    e.rows = seq_len;
                    kv_new = e.maps;
                }
            }
        }
        pl.kv_new = kv_new;
        const gkv::PoolMaps maps{t->k_map_sw, t->v_map_sw, t->runs ? t->k_map_run : t->k_map_sw,
                                 t->runs ? t->v_map_run : t->v_map_sw, t->runs};
        e = gkv::launch_prefill_tc(pv, *q_map, maps, t->d_table, pl, t->scratch.err, t->num_sms, s);
    }
    if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
    return GKV_OK;
}
}  // namespace

int gkv_rope_cache(float theta, int32_t head_dim, int32_t max_seq, float* cos_out, float* sin_out) {
    if (head_dim < 2 || head_dim % 2 || max_seq < 0 || !cos_out || !sin_out || !(theta > 0.f))
        return fail(GKV_ERR_INVALID, "gkv_rope_cache: bad arguments");
    // RopeCacheImpl<CPU> (src/backend/cpu/rope.cpp:112-140): angles in double,
    // inv_freq_i = theta^(-2i/d); cos/sin rounded to float, written to
    // columns i and i + d/2.
    const int32_t half = head_dim / 2;
    std::vector<double> inv(half);
    for (int32_t i = 0; i < half; ++i)
        inv[i] = 1.0 / std::pow(static_cast<double>(theta), (2.0 * i) / static_cast<double>(head_dim));
    for (int32_t p = 0; p < max_seq; ++p) {
        float* c = cos_out + static_cast<size_t>(p) * head_dim;
        float* sn = sin_out + static_cast<size_t>(p) * head_dim;
        for (int32_t i = 0; i < half; ++i) {
            const double a = static_cast<double>(p) * inv[i];
            c[i] = c[i + half] = static_cast<float>(std::cos(a));
            sn[i] = sn[i + half] = static_cast<float>(std::sin(a));
        }
    }
    return GKV_OK;
}

int gkv_qk_norm_rope(const void* q_flat, const void* k_flat, const void* v_flat, int32_t seq_len, int32_t n_q_heads,
                     int32_t n_kv_heads, const gkv_qk_norm* qk, int32_t start_pos, void* q_out, void* k_out,
                     void* v_out, gkv_stream_t stream) {
    NvtxRange nvtx_range("gkv qk-norm + rope");
    if (!q_flat || !k_flat || !v_flat || !q_out || !k_out || !v_out || seq_len < 0 || n_q_heads < 1 || n_kv_heads < 1)
        return fail(GKV_ERR_INVALID, "gkv_qk_norm_rope: bad arguments");
    if (!aligned16(q_flat) || !aligned16(k_flat) || !aligned16(v_flat) || !aligned16(q_out) || !aligned16(k_out) ||
        !aligned16(v_out))
        return fail(GKV_ERR_INVALID, "gkv_qk_norm_rope: every buffer must be 16-byte aligned");
    if (n_q_heads + n_kv_heads > 96)
        return fail(GKV_ERR_UNSUPPORTED, "gkv_qk_norm_rope: at most 96 query + kv heads per token");
    int st = check_qk(qk, start_pos, seq_len);
    if (st) return st;
    const gkv::QkNorm n{qk->q_norm_w, qk->k_norm_w, qk->cos_tab, qk->sin_tab, qk->eps};
    cudaError_t e = gkv::launch_qk_norm_rope(
        static_cast<const uint16_t*>(q_flat), static_cast<const uint16_t*>(k_flat), static_cast<const uint16_t*>(v_flat),
        seq_len, n_q_heads, n_kv_heads, n, start_pos, static_cast<uint16_t*>(q_out), static_cast<uint16_t*>(k_out),
        static_cast<uint16_t*>(v_out), reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "qk norm / rope launch");
    return GKV_OK;
}

int gkv_paged_attention_raw_qknorm(const gkv_pool_desc* pool, gkv_table* t, int32_t n_prior, const gkv_new_pages* np,
                                   const void* q_flat, const void* k_flat, const void* v_flat, void* out,
                                   int32_t n_q_heads, int32_t seq_len, float scale, int32_t causal, int32_t out_dtype,
                                   const gkv_qk_norm* qk, gkv_stream_t stream) {
    int st = check_pool(pool);
    if (st) return st;
    if (!t || seq_len < 1 || !q_flat || !k_flat || !v_flat) return fail(GKV_ERR_INVALID, "bad arguments");
    if ((st = check_qk(qk, n_prior, seq_len))) return st;
    const gkv::QkNorm n{qk->q_norm_w, qk->k_norm_w, qk->cos_tab, qk->sin_tab, qk->eps};
    if (seq_len == 1)  // [1][H*128] is already [H][1][128]: QK-norm + RoPE inside the decode kernel
        return attention_raw(pool, t, n_prior, np, q_flat, k_flat, v_flat, out, n_q_heads, 1, scale, causal,
                             out_dtype, &n, stream);
    // A chunk: normalise, rotate and permute into the table's buffer, then
    // the chunked-prefill path.
    const size_t elems_q = static_cast<size_t>(seq_len) * n_q_heads * 128;
    const size_t elems_kv = static_cast<size_t>(seq_len) * pool->n_kv_heads * 128;
    const size_t bytes = (elems_q + 2 * elems_kv) * sizeof(uint16_t);
    DeviceGuard g(t->device);
    if (!g.ok()) return fail(GKV_ERR_CUDA, "cannot select device %d", t->device);
    if (bytes > t->qk_bytes) {
        // The previous buffer may still be read by work queued on a stream.
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_fail(e, "qk buffer grow");
        cudaFree(t->qk_buf);
        t->qk_buf = nullptr;
        t->qk_bytes = 0;
        if ((e = cudaMalloc(&t->qk_buf, bytes)) != cudaSuccess) return cuda_fail(e, "qk buffer grow");
        t->qk_bytes = bytes;
    }
    uint16_t* qb = static_cast<uint16_t*>(t->qk_buf);
    uint16_t* kb = qb + elems_q;
    uint16_t* vb = kb + elems_kv;
    if ((st = gkv_qk_norm_rope(q_flat, k_flat, v_flat, seq_len, n_q_heads, pool->n_kv_heads, qk, n_prior, qb, kb, vb,
                               stream)))
        return st;
    return attention_raw(pool, t, n_prior, np, qb, kb, vb, out, n_q_heads, seq_len, scale, causal, out_dtype, nullptr,
                         stream);
}

}  // extern "C"

// ============================ managed tier ==================================

namespace {

// BlockPool (src/core/page_attention.cpp:25-64): ids [0, capacity); alloc
// takes the most recently freed id, else the next never-used one. Capacity 0
// means unbounded, as for the reference's default-constructed BlockPool (a
// layer that was never reserved, page_attention.cpp:44).
class PagePool {
   public:
    void init(int32_t capacity) {
        capacity_ = capacity;
        handed_out_ = 0;
        free_.clear();
        free_.reserve(capacity);
        is_free_.assign(capacity, 0);
    }
    int32_t capacity() const { return capacity_; }
    int32_t num_blocks() const { return handed_out_; }
    int32_t num_free() const { return static_cast<int32_t>(free_.size()); }
    int32_t available() const {
        return capacity_ > 0 ? num_free() + (capacity_ - handed_out_) : INT32_MAX;
    }
    int32_t alloc() {
        if (!free_.empty()) {
            const int32_t id = free_.back();
            free_.pop_back();
            is_free_[id] = 0;
            return id;
        }
        if (capacity_ > 0 && handed_out_ >= capacity_) return -1;
        if (handed_out_ >= static_cast<int32_t>(is_free_.size())) is_free_.push_back(0);
        return handed_out_++;
    }
    // 0 ok / ignored (never handed out), -1 double free.
    int free(int32_t id) {
        if (id < 0 || id >= handed_out_) return 0;
        if (is_free_[id]) return -1;
        is_free_[id] = 1;
        free_.push_back(id);
        return 0;
    }
    void reset() {
        free_.clear();
        for (int32_t i = 0; i < handed_out_; ++i) free_.push_back(i);
        std::fill(is_free_.begin(), is_free_.begin() + handed_out_, 1);
    }
    bool is_handed_out(int32_t id) const { return id >= 0 && id < handed_out_ && !is_free_[id]; }

   private:
    int32_t capacity_ = 0;
    int32_t handed_out_ = 0;
    std::vector<int32_t> free_;
    std::vector<uint8_t> is_free_;
};

struct Layer {
    bool active = false;
    bool reserved = false;
    int32_t num_cached = 0;
    int32_t n_kv_heads = 0;
    int32_t head_dim = 0;
    int32_t dtype = GKV_BF16;
    int32_t max_blocks = 0;
    PagePool k_pool, v_pool;
    std::vector<int32_t> k_ids, v_ids;  // host block table
    int32_t on_device = 0;              // table entries already published to the device
    void* k_base = nullptr;
    void* v_base = nullptr;
    bool owns_regions = false;
    gkv_table* table = nullptr;
};

}  // namespace

struct gkv_manager {
    int device = 0;
    std::map<int32_t, Layer> layers;
};

namespace {

Layer* find_layer(gkv_manager* m, int32_t id) {
    if (!m) return nullptr;
    auto it = m->layers.find(id);
    return it == m->layers.end() ? nullptr : &it->second;
}
const Layer* find_layer(const gkv_manager* m, int32_t id) {
    if (!m) return nullptr;
    auto it = m->layers.find(id);
    return it == m->layers.end() ? nullptr : &it->second;
}

void release_layer(Layer& L) {
    if (L.owns_regions) {
        cudaFree(L.k_base);
        cudaFree(L.v_base);
    }
    L.k_base = L.v_base = nullptr;
    L.owns_regions = false;
    gkv_table_destroy(L.table);
    L.table = nullptr;
    L.reserved = false;
}

gkv_pool_desc pool_of(const Layer& L) {
    return gkv_pool_desc{L.k_base, L.v_base, L.max_blocks, L.n_kv_heads, L.head_dim, L.dtype};
}

// Allocate the pages `count` more tokens need, all or nothing. Returns the
// first new logical page and how many were added.
int grow(Layer& L, int32_t count, int32_t* first_new, int32_t* n_new) {
    int32_t need = 0;
    for (int32_t p = 0; p < count; ++p)
        if ((L.num_cached + p) % 16 == 0) ++need;
    // A table can hold at most max_blocks logical pages.
    if (L.k_pool.available() < need || L.v_pool.available() < need ||
        (L.reserved && static_cast<int32_t>(L.k_ids.size()) + need > L.max_blocks))
        return fail(GKV_ERR_NO_PAGES, "layer needs %d more pages: K pool has %d, V pool has %d", need,
                    L.k_pool.available(), L.v_pool.available());
    *first_new = static_cast<int32_t>(L.k_ids.size());
    *n_new = need;
    for (int32_t i = 0; i < need; ++i) {
        L.k_ids.push_back(L.k_pool.alloc());
        L.v_ids.push_back(L.v_pool.alloc());
    }
    return GKV_OK;
}

void ungrow(Layer& L, int32_t first_new) {
    while (static_cast<int32_t>(L.k_ids.size()) > first_new) {
        L.k_pool.free(L.k_ids.back());
        L.v_pool.free(L.v_ids.back());
        L.k_ids.pop_back();
        L.v_ids.pop_back();
    }
    L.on_device = std::min<int32_t>(L.on_device, first_new);
}

// Everything from L.on_device to the end of the table goes to the device with
// the next launch.
gkv_new_pages pending(const Layer& L) {
    gkv_new_pages np;
    np.first_new_page = L.on_device;
    np.n_new_pages = static_cast<int32_t>(L.k_ids.size()) - L.on_device;
    np.k_ids = L.k_ids.data() + L.on_device;
    np.v_ids = L.v_ids.data() + L.on_device;
    return np;
}

// An active layer (page bookkeeping works on it even before reserve_layer,
// as in the reference's pool-less manager).
int active_layer(gkv_manager* m, int32_t layer_id, Layer** out) {
    Layer* L = find_layer(m, layer_id);
    if (!L || !L->active) return fail(GKV_ERR_STATE, "layer %d is not initialised", layer_id);
    *out = L;
    return GKV_OK;
}

// An active layer with device pools, ready for kernel launches.
int ready_layer(gkv_manager* m, int32_t layer_id, Layer** out) {
    int st = active_layer(m, layer_id, out);
    if (st) return st;
    if (!(*out)->reserved || !(*out)->table)
        return fail(GKV_ERR_STATE, "layer %d has no device pools (not reserved, or a host-only manager)",
                    layer_id);
    return GKV_OK;
}

}  // namespace

extern "C" {

int gkv_manager_create(int device, gkv_manager** out) {
    if (!out) return fail(GKV_ERR_INVALID, "null out");
    if (device != -1) {
        int n = 0;
        cudaError_t e = cudaGetDeviceCount(&n);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
        if (device < 0 || device >= n) return fail(GKV_ERR_INVALID, "device %d of %d", device, n);
    }
    auto* m = new gkv_manager();
    m->device = device;
    *out = m;
    return GKV_OK;
}

int gkv_manager_destroy(gkv_manager* m) {
    if (!m) return GKV_OK;
    if (m->device >= 0) {
        DeviceGuard g(m->device);
        for (auto& kv : m->layers) release_layer(kv.second);
    }
    delete m;
    return GKV_OK;
}

int gkv_init_layer(gkv_manager* m, int32_t layer_id, int32_t n_kv_heads, int32_t head_dim, int32_t dtype) {
    if (!m) return fail(GKV_ERR_INVALID, "null manager");
    if (n_kv_heads < 1 || n_kv_heads > kMaxKvHeads || head_dim < 1)
        return fail(GKV_ERR_INVALID, "bad layer geometry");
    Layer& L = m->layers[layer_id];
    L.n_kv_heads = n_kv_heads;
    L.head_dim = head_dim;
    L.dtype = dtype;
    L.active = true;
    L.num_cached = 0;
    return GKV_OK;
}

int gkv_reserve_layer(gkv_manager* m, int32_t layer_id, int32_t max_blocks, void* k_region, void* v_region) {
    Layer* L = find_layer(m, layer_id);
    if (!L || !L->active) return fail(GKV_ERR_STATE, "layer %d is not initialised", layer_id);
    if (max_blocks < 1) return fail(GKV_ERR_INVALID, "max_blocks %d", max_blocks);
    if ((k_region == nullptr) != (v_region == nullptr))
        return fail(GKV_ERR_INVALID, "give both regions or neither");
    if (k_region && (!aligned16(k_region) || !aligned16(v_region)))
        return fail(GKV_ERR_INVALID, "regions must be 16-byte aligned");
    if (m->device < 0) {
        // Host-only manager: page bookkeeping with the given capacity, no memory.
        L->max_blocks = max_blocks;
        L->k_pool.init(max_blocks);
        L->v_pool.init(max_blocks);
        L->k_ids.clear();
        L->v_ids.clear();
        L->on_device = 0;
        L->num_cached = 0;
        L->reserved = true;
        return GKV_OK;
    }
    const int eb = L->dtype == GKV_F32 ? 4 : 2;
    const size_t bytes = (size_t)max_blocks * 16 * L->n_kv_heads * L->head_dim * eb;
    DeviceGuard g(m->device);
    if (!g.ok()) return fail(GKV_ERR_CUDA, "cannot select device %d", m->device);
    release_layer(*L);
    if (k_region) {
        L->k_base = k_region;
        L->v_base = v_region;
    } else {
        cudaError_t e = cudaMalloc(&L->k_base, bytes);
        if (e == cudaSuccess) e = cudaMalloc(&L->v_base, bytes);
        if (e != cudaSuccess) {
            cudaFree(L->k_base);
            L->k_base = L->v_base = nullptr;
            return cuda_fail(e, "KV pool allocation");
        }
        L->owns_regions = true;
    }
    int st = gkv_table_create(m->device, max_blocks, &L->table);
    if (st) {
        release_layer(*L);
        return st;
    }
    L->max_blocks = max_blocks;
    L->k_pool.init(max_blocks);
    L->v_pool.init(max_blocks);
    L->k_ids.clear();
    L->v_ids.clear();
    L->on_device = 0;
    L->num_cached = 0;
    L->reserved = true;
    return GKV_OK;
}

int gkv_is_active(const gkv_manager* m, int32_t layer_id) {
    const Layer* L = find_layer(m, layer_id);
    return L && L->active ? 1 : 0;
}

int gkv_append_kv_pages(gkv_manager* m, int32_t layer_id, int32_t count) {
    Layer* L = nullptr;
    int st = active_layer(m, layer_id, &L);
    if (st) return st;
    if (count <= 0) return GKV_OK;  // the reference ignores count <= 0 (:143)
    int32_t first = 0, n = 0;
    if ((st = grow(*L, count, &first, &n))) return st;
    L->num_cached += count;
    return GKV_OK;
}

int gkv_append_kv(gkv_manager* m, int32_t layer_id, const void* K, const void* V, int32_t n_kv_heads,
                  int32_t seq_len, int32_t head_dim, int32_t dtype, gkv_stream_t stream) {
    Layer* L = nullptr;
    int st = ready_layer(m, layer_id, &L);
    if (st) return st;
    if (n_kv_heads != L->n_kv_heads || head_dim != L->head_dim || dtype != L->dtype)
        return fail(GKV_ERR_INVALID, "K/V geometry does not match layer %d", layer_id);
    if (seq_len <= 0) return GKV_OK;  // the reference returns early (:110)
    int32_t first = 0, n = 0;
    if ((st = grow(*L, seq_len, &first, &n))) return st;
    gkv_pool_desc pool = pool_of(*L);
    gkv_new_pages np = pending(*L);
    st = gkv_append_kv_raw(&pool, L->table, L->num_cached, &np, K, V, seq_len, stream);
    if (st) {
        ungrow(*L, first);
        return st;
    }
    L->on_device = static_cast<int32_t>(L->k_ids.size());
    L->num_cached += seq_len;
    return GKV_OK;
}

int gkv_paged_attention(gkv_manager* m, int32_t layer_id, const void* Q, const void* K, const void* V,
                        void* out, int32_t batch, int32_t n_q_heads, int32_t seq_len, int32_t head_dim,
                        int32_t n_kv_heads, float scale, int32_t causal, int32_t n_kv_groups,
                        int32_t dtype, int32_t out_dtype, gkv_stream_t stream) {
    Layer* L = nullptr;
    int st = ready_layer(m, layer_id, &L);
    if (st) return st;
    if (batch != 1) return fail(GKV_ERR_UNSUPPORTED, "batch %d: the paged cache holds one sequence", batch);
    if (n_kv_heads != L->n_kv_heads || head_dim != L->head_dim || dtype != L->dtype)
        return fail(GKV_ERR_INVALID, "Q/K/V geometry does not match layer %d", layer_id);
    if (n_kv_groups * n_kv_heads != n_q_heads)
        return fail(GKV_ERR_INVALID, "n_kv_groups %d * n_kv_heads %d != n_q_heads %d", n_kv_groups, n_kv_heads,
                    n_q_heads);
    if (seq_len < 1) return fail(GKV_ERR_INVALID, "seq_len %d", seq_len);
    int32_t first = 0, n = 0;
    if ((st = grow(*L, seq_len, &first, &n))) return st;
    gkv_pool_desc pool = pool_of(*L);
    gkv_new_pages np = pending(*L);
    st = gkv_paged_attention_raw(&pool, L->table, L->num_cached, &np, Q, K, V, out, n_q_heads, seq_len, scale,
                                 causal, out_dtype, stream);
    if (st) {
        ungrow(*L, first);
        return st;
    }
    L->on_device = static_cast<int32_t>(L->k_ids.size());
    L->num_cached += seq_len;
    return GKV_OK;
}

int gkv_paged_attention_qknorm(gkv_manager* m, int32_t layer_id, const void* q_flat, const void* k_flat,
                               const void* v_flat, void* out, int32_t n_q_heads, int32_t seq_len, float scale,
                               int32_t causal, int32_t out_dtype, const gkv_qk_norm* qk, gkv_stream_t stream) {
    Layer* L = nullptr;
    int st = ready_layer(m, layer_id, &L);
    if (st) return st;
    if (L->head_dim != 128 || L->dtype != GKV_BF16)
        return fail(GKV_ERR_UNSUPPORTED, "QK-norm + RoPE is built for head_dim 128, bf16");
    if (seq_len < 1) return fail(GKV_ERR_INVALID, "seq_len %d", seq_len);
    int32_t first = 0, n = 0;
    if ((st = grow(*L, seq_len, &first, &n))) return st;
    gkv_pool_desc pool = pool_of(*L);
    gkv_new_pages np = pending(*L);
    st = gkv_paged_attention_raw_qknorm(&pool, L->table, L->num_cached, &np, q_flat, k_flat, v_flat, out, n_q_heads,
                                        seq_len, scale, causal, out_dtype, qk, stream);
    if (st) {
        ungrow(*L, first);
        return st;
    }
    L->on_device = static_cast<int32_t>(L->k_ids.size());
    L->num_cached += seq_len;
    return GKV_OK;
}

int gkv_decode_layers(gkv_manager* m, int32_t n_layers, const int32_t* layer_ids, const void* const* Q,
                      const void* const* K, const void* const* V, void* const* out, int32_t n_q_heads, float scale,
                      int32_t out_dtype, gkv_stream_t stream) {
    NvtxRange nvtx_range("gkv decode step (multi-layer)");
    if (!m || n_layers < 0 || (n_layers && (!layer_ids || !Q || !K || !V || !out)))
        return fail(GKV_ERR_INVALID, "gkv_decode_layers: bad arguments");
    bool distinct = true;
    for (int32_t i = 0; i < n_layers && distinct; ++i)
        for (int32_t j = 0; j < i; ++j)
            if (layer_ids[j] == layer_ids[i]) distinct = false;
    for (int32_t i = 0; i < n_layers; ++i) {
        Layer* L = nullptr;
        int st = ready_layer(m, layer_ids[i], &L);
        if (st) return st;
        if (n_q_heads % L->n_kv_heads) return fail(GKV_ERR_INVALID, "n_q_heads %d, n_kv_heads %d", n_q_heads, L->n_kv_heads);
        // Layer 0's combine releases layer 1 only after layer 0's decode has
        // completed, i.e. after its wait on whatever produced the step's
        // inputs (a kernel before this call may itself release early); from
        // there on the inputs are complete and the layers distinct. A layer
        // whose new pages exceed one launch's list publishes them with extra
        // launches first: it keeps the wait.
        const int32_t pend = static_cast<int32_t>(L->k_ids.size()) - L->on_device + 1;
        t_next_other_layer = distinct && i >= 1 && i + 1 < n_layers;
        t_prev_other_layer = distinct && i > 0 && pend <= gkv::kMaxNewPagesPerLaunch;
        st = gkv_paged_attention(m, layer_ids[i], Q[i], K[i], V[i], out[i], 1, n_q_heads, 1, L->head_dim,
                                 L->n_kv_heads, scale, 1, n_q_heads / L->n_kv_heads, L->dtype, out_dtype, stream);
        t_next_other_layer = t_prev_other_layer = false;
        if (st) return st;
    }
    return GKV_OK;
}

// ============================ captured decode steps ===========================

struct gkv_decode_graph {
    gkv_manager* m = nullptr;
    int device = 0;
    int grid = 0;
    int32_t n_q_heads = 0;
    std::vector<int32_t> layers;
    std::vector<int32_t> max_seq;     // per layer: RoPE rows (0 without QK-norm)
    gkv::DeviceStep* host[2] = {nullptr, nullptr};  // pinned, one per graph
    gkv::DeviceStep* dev[2] = {nullptr, nullptr};
    cudaGraphExec_t exec[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    bool launched[2] = {false, false};
    uint64_t steps = 0;
};

namespace {

void decode_graph_free(gkv_decode_graph* g) {
    if (!g) return;
    DeviceGuard dg(g->device);
    for (int b = 0; b < 2; ++b) {
        if (g->done[b]) {
            cudaEventSynchronize(g->done[b]);
            cudaEventDestroy(g->done[b]);
        }
        if (g->exec[b]) cudaGraphExecDestroy(g->exec[b]);
        cudaFreeHost(g->host[b]);
        cudaFree(g->dev[b]);
    }
    delete g;
}

// Capture buffer b's step: the copy of the step block, then every layer's
// decode + combine launches reading it.
int capture_decode_graph(gkv_decode_graph* g, int b, const void* const* Q, const void* const* K,
                         const void* const* V, void* const* out, int32_t n_q_heads, float scale, int32_t out_dtype,
                         const gkv::QkNorm* qks) {
    cudaStream_t cs = nullptr;
    cudaError_t e = cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cuda_fail(e, "capture stream");
    const size_t n = g->layers.size();
    e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
    int st = GKV_OK;
    if (e == cudaSuccess) {
        e = cudaMemcpyAsync(g->dev[b], g->host[b], sizeof(gkv::DeviceStep) * n, cudaMemcpyHostToDevice, cs);
        for (size_t i = 0; i < n && e == cudaSuccess; ++i) {
            Layer* L = find_layer(g->m, g->layers[i]);
            gkv_table* t = L->table;
            gkv::PoolView pv{static_cast<uint16_t*>(L->k_base), static_cast<uint16_t*>(L->v_base), L->max_blocks,
                             L->n_kv_heads};
            gkv::DecodeLaunch d{};
            d.q = static_cast<const uint16_t*>(Q[i]);
            d.k_new = static_cast<const uint16_t*>(K[i]);
            d.v_new = static_cast<const uint16_t*>(V[i]);
            d.out = out[i];
            d.out_dtype = out_dtype;
            d.n_q_heads = n_q_heads;
            d.n_prior = 0;  // capture-time values; the kernels read the step block
            d.total = 1;
            d.n_pages = 1;
            d.scale = scale;
            d.qk = qks ? &qks[i] : nullptr;
            d.step = g->dev[b] + i;
            d.grid = g->grid;
            // The graph's layers are distinct, and its first node (the copy)
            // runs after all earlier work on the stream has completed, so the
            // inputs are complete when layer 0's decode starts.
            d.next_is_other_layer = i + 1 < n;
            d.prev_is_other_layer = i > 0;
            d.fused_merge = fused_merge_enabled();
            gkv::NewPages none{};
            e = gkv::launch_decode(pv, t->dmaps, t->d_table, none, t->scratch, d, t->num_sms, cs);
        }
        cudaGraph_t graph = nullptr;
        const cudaError_t e2 = cudaStreamEndCapture(cs, &graph);
        if (e == cudaSuccess) e = e2;
        if (e == cudaSuccess) e = cudaGraphInstantiate(&g->exec[b], graph, 0);
        if (graph) cudaGraphDestroy(graph);
    }
    if (e != cudaSuccess) st = cuda_fail(e, "decode step capture");
    cudaStreamDestroy(cs);
    return st;
}

}  // namespace

int gkv_decode_graph_create(gkv_manager* m, int32_t n_layers, const int32_t* layer_ids, const void* const* Q,
                            const void* const* K, const void* const* V, void* const* out, int32_t n_q_heads,
                            float scale, int32_t out_dtype, const gkv_qk_norm* const* qk, gkv_decode_graph** out_g) {
    if (!out_g) return fail(GKV_ERR_INVALID, "gkv_decode_graph_create: null output");
    *out_g = nullptr;
    if (!m || n_layers < 1 || !layer_ids || !Q || !K || !V || !out)
        return fail(GKV_ERR_INVALID, "gkv_decode_graph_create: bad arguments");
    if (!is_out_dtype(out_dtype)) return fail(GKV_ERR_UNSUPPORTED, "out dtype %d", out_dtype);
    std::vector<gkv::QkNorm> qks;
    auto* g = new gkv_decode_graph();
    g->m = m;
    g->device = m->device;
    g->n_q_heads = n_q_heads;
    for (int32_t i = 0; i < n_layers; ++i) {
        Layer* L = nullptr;
        int st = ready_layer(m, layer_ids[i], &L);
        if (!st && (L->n_kv_heads > 8 || L->head_dim != 128 || L->dtype != GKV_BF16))
            st = fail(GKV_ERR_UNSUPPORTED, "layer %d: the decode kernel is built for head_dim 128, bf16, <= 8 kv heads",
                      layer_ids[i]);
        const int G = L && L->n_kv_heads ? n_q_heads / L->n_kv_heads : 0;
        if (!st && (n_q_heads % L->n_kv_heads || (G != 1 && G != 2 && G != 4 && G != 8)))
            st = fail(GKV_ERR_UNSUPPORTED, "n_q_heads %d over %d kv heads", n_q_heads, L->n_kv_heads);
        for (int32_t j = 0; !st && j < i; ++j)
            if (layer_ids[j] == layer_ids[i]) st = fail(GKV_ERR_INVALID, "layer %d listed twice", layer_ids[i]);
        if (!st && (!Q[i] || !K[i] || !V[i] || !out[i] || !aligned16(Q[i]) || !aligned16(K[i]) || !aligned16(V[i]) ||
                    !aligned16(out[i])))
            st = fail(GKV_ERR_INVALID, "layer %d: Q/K/V/out must be non-null and 16-byte aligned", layer_ids[i]);
        if (!st && qk && qk[i]) {
            if ((st = check_qk(qk[i], 0, 1))) {
            } else {
                qks.push_back(gkv::QkNorm{qk[i]->q_norm_w, qk[i]->k_norm_w, qk[i]->cos_tab, qk[i]->sin_tab, qk[i]->eps});
            }
        } else if (!st && qk) {
            st = fail(GKV_ERR_INVALID, "qk given for some layers only");
        }
        if (st) {
            delete g;
            return st;
        }
        g->layers.push_back(layer_ids[i]);
        g->max_seq.push_back(qk ? qk[i]->max_seq : 0);
    }
    DeviceGuard dg(m->device);
    if (!dg.ok()) {
        delete g;
        return fail(GKV_ERR_CUDA, "cannot select device %d", m->device);
    }
    int num_sms = 148;
    cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, g->device);
    g->grid = std::min(num_sms, (int)(gkv::kMaxPartialRows / n_q_heads));
    for (int32_t i = 0; i < n_layers; ++i) {
        Layer* L = find_layer(m, layer_ids[i]);
        gkv_pool_desc pool = pool_of(*L);
        int st = table_maps(L->table, &pool);
        if (st) {
            decode_graph_free(g);
            return st;
        }
    }
    const size_t bytes = sizeof(gkv::DeviceStep) * n_layers;
    if (cudaError_t e = gkv::configure_decode_kernels(); e != cudaSuccess) {  // not during capture
        decode_graph_free(g);
        return cuda_fail(e, "decode kernel attributes");
    }
    for (int b = 0; b < 2; ++b) {
        cudaError_t e = cudaMallocHost(&g->host[b], bytes);
        if (e == cudaSuccess) e = cudaMalloc(&g->dev[b], bytes);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&g->done[b], cudaEventDisableTiming);
        if (e != cudaSuccess) {
            decode_graph_free(g);
            return cuda_fail(e, "decode graph buffers");
        }
        memset(g->host[b], 0, bytes);
        int st = capture_decode_graph(g, b, Q, K, V, out, n_q_heads, scale, out_dtype, qk ? qks.data() : nullptr);
        if (st) {
            decode_graph_free(g);
            return st;
        }
    }
    *out_g = g;
    return GKV_OK;
}

int gkv_decode_graph_step(gkv_decode_graph* g, gkv_stream_t stream) {
    NvtxRange nvtx_range("gkv decode step (captured)");
    if (!g) return fail(GKV_ERR_INVALID, "null decode graph");
    DeviceGuard dg(g->device);
    if (!dg.ok()) return fail(GKV_ERR_CUDA, "cannot select device %d", g->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int b = static_cast<int>(g->steps & 1);
    // The pinned block b was last read by the step launched two steps ago.
    if (g->launched[b]) {
        cudaError_t e = cudaEventSynchronize(g->done[b]);
        if (e != cudaSuccess) return cuda_fail(e, "decode graph: wait for the step block");
    }
    const size_t n = g->layers.size();
    std::vector<int32_t> first(n, -1);
    int st = GKV_OK;
    size_t i = 0;
    for (; i < n; ++i) {
        Layer* L = nullptr;
        if ((st = ready_layer(g->m, g->layers[i], &L))) break;
        if (g->max_seq[i] && L->num_cached + 1 > g->max_seq[i]) {
            st = fail(GKV_ERR_INVALID, "layer %d: position %d exceeds the RoPE table (%d rows)", g->layers[i],
                      L->num_cached, g->max_seq[i]);
            break;
        }
        int32_t f = 0, nn = 0;
        if ((st = grow(*L, 1, &f, &nn))) break;
        first[i] = f;
        gkv_pool_desc pool = pool_of(*L);
        gkv_new_pages np = pending(*L);
        const int32_t total = L->num_cached + 1;
        const int32_t n_pages = (total + 15) / 16;
        if ((st = check_new_pages(L->table, &np, n_pages, pool.pool_pages))) break;
        // Host-only growth beyond this step's page goes out first.
        if (np.n_new_pages > 1 && (st = publish(&pool, L->table, &np, 0, np.n_new_pages - 1, s))) break;
        gkv::DeviceStep& d = g->host[b][i];
        d.n_prior = L->num_cached;
        d.total = total;
        d.n_pages = n_pages;
        d.new_n = np.n_new_pages > 0 ? 1 : 0;
        d.new_first = np.first_new_page + np.n_new_pages - 1;
        d.new_id = d.new_n ? make_int2(np.k_ids[np.n_new_pages - 1], np.v_ids[np.n_new_pages - 1]) : make_int2(0, 0);
        d.pad = 0;
        if (!gkv::decode_split_geometry(n_pages, L->n_kv_heads, g->n_q_heads, 0, L->table->num_sms, &d.pages_per_split,
                                        &d.n_splits) ||
            d.n_splits > g->grid) {
            st = fail(GKV_ERR_UNSUPPORTED, "layer %d: %d tokens need more splits than the captured grid (%d)",
                      g->layers[i], total, g->grid);
            break;
        }
    }
    if (st) {
        for (size_t j = 0; j <= i && j < n; ++j)
            if (first[j] >= 0) ungrow(*find_layer(g->m, g->layers[j]), first[j]);
        return st;
    }
    cudaError_t e = cudaGraphLaunch(g->exec[b], s);
    if (e == cudaSuccess) e = cudaEventRecord(g->done[b], s);
    if (e != cudaSuccess) {
        for (size_t j = 0; j < n; ++j) ungrow(*find_layer(g->m, g->layers[j]), first[j]);
        return cuda_fail(e, "decode graph launch");
    }
    g->launched[b] = true;
    ++g->steps;
    for (size_t j = 0; j < n; ++j) {
        Layer* L = find_layer(g->m, g->layers[j]);
        L->on_device = static_cast<int32_t>(L->k_ids.size());
        L->num_cached += 1;
    }
    return GKV_OK;
}

int gkv_decode_graph_destroy(gkv_decode_graph* g) {
    decode_graph_free(g);
    return GKV_OK;
}

int gkv_export_kv(gkv_manager* m, int32_t layer_id, int32_t format, void* K_out, void* V_out, float* k_scales,
                  float* v_scales, int32_t* n_tokens, gkv_stream_t stream) {
    Layer* L = nullptr;
    int st = ready_layer(m, layer_id, &L);
    if (st) return st;
    gkv_pool_desc pool = pool_of(*L);
    // Pages grown on the host only (gkv_append_kv_pages) reach the device table first.
    gkv_new_pages np = pending(*L);
    if (np.n_new_pages > 0) {
        DeviceGuard g(L->table->device);
        if (!g.ok()) return fail(GKV_ERR_CUDA, "cannot select device %d", L->table->device);
        if ((st = check_new_pages(L->table, &np, static_cast<int32_t>(L->k_ids.size()), pool.pool_pages))) return st;
        if ((st = publish(&pool, L->table, &np, 0, np.n_new_pages, reinterpret_cast<cudaStream_t>(stream)))) return st;
        L->on_device = static_cast<int32_t>(L->k_ids.size());
    }
    if ((st = gkv_export_kv_raw(&pool, L->table, L->num_cached, format, K_out, V_out, k_scales, v_scales, stream)))
        return st;
    if (n_tokens) *n_tokens = L->num_cached;
    return GKV_OK;
}

int gkv_import_kv(gkv_manager* m, int32_t layer_id, int32_t format, const void* K_in, const void* V_in,
                  const float* k_scales, const float* v_scales, int32_t seq_len, gkv_stream_t stream) {
    Layer* L = nullptr;
    int st = ready_layer(m, layer_id, &L);
    if (st) return st;
    if (format != GKV_KV_BF16 && format != GKV_KV_FP8_E4M3) return fail(GKV_ERR_INVALID, "unknown KV format %d", format);
    if (seq_len < 0) return fail(GKV_ERR_INVALID, "seq_len %d", seq_len);
    if (seq_len == 0) return GKV_OK;
    int32_t first = 0, n = 0;
    if ((st = grow(*L, seq_len, &first, &n))) return st;
    gkv_pool_desc pool = pool_of(*L);
    gkv_new_pages np = pending(*L);
    st = gkv_import_kv_raw(&pool, L->table, L->num_cached, &np, format, K_in, V_in, k_scales, v_scales, seq_len,
                           stream);
    if (st) {
        ungrow(*L, first);
        return st;
    }
    L->on_device = static_cast<int32_t>(L->k_ids.size());
    L->num_cached += seq_len;
    return GKV_OK;
}

int gkv_reset_layer(gkv_manager* m, int32_t layer_id) {
    Layer* L = find_layer(m, layer_id);
    if (!L) return fail(GKV_ERR_STATE, "layer %d unknown", layer_id);
    L->num_cached = 0;
    L->k_ids.clear();
    L->v_ids.clear();
    L->on_device = 0;
    L->k_pool.reset();
    L->v_pool.reset();
    return GKV_OK;
}

int gkv_reset(gkv_manager* m) {
    if (!m) return fail(GKV_ERR_INVALID, "null manager");
    for (auto& kv : m->layers) gkv_reset_layer(m, kv.first);
    return GKV_OK;
}

int gkv_get_layer_info(const gkv_manager* m, int32_t layer_id, gkv_layer_info* info) {
    const Layer* L = find_layer(m, layer_id);
    if (!info) return fail(GKV_ERR_INVALID, "null info");
    std::memset(info, 0, sizeof *info);
    if (!L) return fail(GKV_ERR_STATE, "layer %d unknown", layer_id);
    info->active = L->active;
    info->num_cached = L->num_cached;
    info->n_pages = static_cast<int32_t>(L->k_ids.size());
    info->max_blocks = L->max_blocks;
    info->n_kv_heads = L->n_kv_heads;
    info->head_dim = L->head_dim;
    info->dtype = L->dtype;
    info->k_base = L->k_base;
    info->v_base = L->v_base;
    info->device_table = gkv_table_device_ptr(L->table);
    return GKV_OK;
}

int gkv_get_page_table(const gkv_manager* m, int32_t layer_id, int32_t* k_ids, int32_t* v_ids, int32_t cap,
                       int32_t* n_pages) {
    const Layer* L = find_layer(m, layer_id);
    if (!L) return fail(GKV_ERR_STATE, "layer %d unknown", layer_id);
    const int32_t n = static_cast<int32_t>(L->k_ids.size());
    if (n_pages) *n_pages = n;
    for (int32_t i = 0; i < n && i < cap; ++i) {
        if (k_ids) k_ids[i] = L->k_ids[i];
        if (v_ids) v_ids[i] = L->v_ids[i];
    }
    return GKV_OK;
}

int gkv_read_device_table(gkv_manager* m, int32_t layer_id, int32_t* k_ids, int32_t* v_ids, int32_t cap,
                          int32_t* n_published) {
    Layer* L = nullptr;
    int st = ready_layer(m, layer_id, &L);
    if (st) return st;
    const int32_t n = L->on_device;
    if (n_published) *n_published = n;
    const int32_t c = std::min(n, cap);
    if (c <= 0) return GKV_OK;
    DeviceGuard g(m->device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "synchronise");
    std::vector<int2> buf(c);
    if ((e = cudaMemcpy(buf.data(), L->table->d_table, sizeof(int2) * c, cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(e, "table download");
    for (int32_t i = 0; i < c; ++i) {
        if (k_ids) k_ids[i] = buf[i].x;
        if (v_ids) v_ids[i] = buf[i].y;
    }
    return GKV_OK;
}

int gkv_set_page_table(gkv_manager* m, int32_t layer_id, const int32_t* k_ids, const int32_t* v_ids,
                       int32_t n_pages, int32_t num_cached, gkv_stream_t stream) {
    Layer* L = nullptr;
    int st = active_layer(m, layer_id, &L);
    if (st) return st;
    if (!L->reserved) return fail(GKV_ERR_STATE, "layer %d has no pools", layer_id);
    if (n_pages < 0 || n_pages > L->max_blocks || (n_pages && (!k_ids || !v_ids)) || num_cached < 0 ||
        num_cached > n_pages * 16 || (num_cached + 15) / 16 != n_pages)
        return fail(GKV_ERR_INVALID, "table of %d pages cannot hold %d tokens", n_pages, num_cached);
    for (int32_t i = 0; i < n_pages; ++i)
        if (!L->k_pool.is_handed_out(k_ids[i]) || !L->v_pool.is_handed_out(v_ids[i]))
            return fail(GKV_ERR_INVALID, "entry %d names a page the pool has not handed out", i);
    std::vector<int2> dev(n_pages);
    for (int32_t i = 0; i < n_pages; ++i) dev[i] = make_int2(k_ids[i], v_ids[i]);
    DeviceGuard g(m->device >= 0 ? m->device : 0);
    if (n_pages && L->table) {
        // Pageable source: the copy is staged before this call returns.
        cudaError_t e = cudaMemcpyAsync(L->table->d_table, dev.data(), sizeof(int2) * n_pages,
                                        cudaMemcpyHostToDevice, reinterpret_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return cuda_fail(e, "table upload");
    }
    L->k_ids.assign(k_ids, k_ids + n_pages);
    L->v_ids.assign(v_ids, v_ids + n_pages);
    L->on_device = n_pages;
    L->num_cached = num_cached;
    return GKV_OK;
}

int gkv_page_alloc(gkv_manager* m, int32_t layer_id, int32_t which, int32_t* id) {
    Layer* L = nullptr;
    int st = active_layer(m, layer_id, &L);
    if (st) return st;
    if (!id || (which != 0 && which != 1)) return fail(GKV_ERR_INVALID, "bad arguments");
    *id = (which == 0 ? L->k_pool : L->v_pool).alloc();
    return *id < 0 ? fail(GKV_ERR_NO_PAGES, "pool exhausted") : GKV_OK;
}

int gkv_page_free(gkv_manager* m, int32_t layer_id, int32_t which, int32_t id) {
    Layer* L = nullptr;
    int st = active_layer(m, layer_id, &L);
    if (st) return st;
    if (which != 0 && which != 1) return fail(GKV_ERR_INVALID, "bad pool selector");
    if ((which == 0 ? L->k_pool : L->v_pool).free(id) != 0)
        return fail(GKV_ERR_INVALID, "page %d freed twice", id);
    return GKV_OK;
}

int gkv_pool_reset(gkv_manager* m, int32_t layer_id, int32_t which) {
    Layer* L = nullptr;
    int st = active_layer(m, layer_id, &L);
    if (st) return st;
    if (which != 0 && which != 1) return fail(GKV_ERR_INVALID, "bad pool selector");
    (which == 0 ? L->k_pool : L->v_pool).reset();
    return GKV_OK;
}

int gkv_pool_stats(const gkv_manager* m, int32_t layer_id, int32_t which, int32_t* num_blocks, int32_t* num_free,
                   int32_t* capacity) {
    const Layer* L = find_layer(m, layer_id);
    if (!L || !L->active) return fail(GKV_ERR_STATE, "layer %d is not initialised", layer_id);
    if (which != 0 && which != 1) return fail(GKV_ERR_INVALID, "bad pool selector");
    const PagePool& p = which == 0 ? L->k_pool : L->v_pool;
    if (num_blocks) *num_blocks = p.num_blocks();
    if (num_free) *num_free = p.num_free();
    if (capacity) *capacity = p.capacity();
    return GKV_OK;
}

int gkv_check_device_errors(gkv_manager* m, int32_t layer_id, uint32_t* flags) {
    Layer* L = nullptr;
    int st = ready_layer(m, layer_id, &L);
    if (st) return st;
    return gkv_table_check_errors(L->table, flags);
}

}  // extern "C"

// ============================ multi-GPU head gather ==========================

struct gkv_gather {
    int device = 0;
    int world = 0;
    int rank = 0;
    int max_layers = 0;
    void* bases[gkv::kMaxGatherRanks] = {};
    uint32_t* flags[gkv::kMaxGatherRanks] = {};
    uint32_t* tickets = nullptr;  // [max_layers], zero between launches
    std::vector<uint32_t> epochs;  // calls so far per layer
    uint64_t wait_ns = 1000ull * 1000ull * 1000ull;  // limit of the wait for the peers' flags (1 s)
};

namespace {
bool gather_flags_pulled() {
    static const bool on = [] {
        const char* v = getenv("GKV_GATHER_FLAGS");
        return v && v[0] == 'p';
    }();
    return on;
}
}  // namespace

extern "C" {

int gkv_device_alloc(int device, size_t bytes, void** ptr) {
    if (!ptr || bytes == 0) return fail(GKV_ERR_INVALID, "bad arguments");
    DeviceGuard g(device);
    if (!g.ok()) return fail(GKV_ERR_CUDA, "cannot select device %d", device);
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
    return e == cudaSuccess ? GKV_OK : cuda_fail(e, "gkv_device_alloc");
}

int gkv_device_free(int device, void* ptr) {
    DeviceGuard g(device);
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? GKV_OK : cuda_fail(e, "gkv_device_free");
}

int gkv_ipc_export(int device, const void* dev_ptr, void* handle) {
    if (!dev_ptr || !handle) return fail(GKV_ERR_INVALID, "bad arguments");
    DeviceGuard g(device);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    std::memcpy(handle, &h, sizeof h);
    return GKV_OK;
}

int gkv_ipc_open(int device, const void* handle, void** dev_ptr) {
    if (!dev_ptr || !handle) return fail(GKV_ERR_INVALID, "bad arguments");
    DeviceGuard g(device);
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof h);
    cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? GKV_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int gkv_ipc_close(int device, void* dev_ptr) {
    DeviceGuard g(device);
    cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
    return e == cudaSuccess ? GKV_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int gkv_gather_create(int device, int world, int rank, int max_layers, void* const* out_bases,
                      uint32_t* const* flag_bases, gkv_gather** out) {
    if (!out || world < 2 || world > gkv::kMaxGatherRanks || rank < 0 || rank >= world || max_layers < 1 ||
        !out_bases || !flag_bases)
        return fail(GKV_ERR_INVALID, "gkv_gather_create: bad arguments");
    for (int r = 0; r < world; ++r)
        if (!out_bases[r] || !flag_bases[r]) return fail(GKV_ERR_INVALID, "null base for rank %d", r);
    DeviceGuard g(device);
    if (!g.ok()) return fail(GKV_ERR_CUDA, "cannot select device %d", device);
    auto* gg = new gkv_gather();
    gg->device = device;
    gg->world = world;
    gg->rank = rank;
    gg->max_layers = max_layers;
    for (int r = 0; r < world; ++r) {
        gg->bases[r] = out_bases[r];
        gg->flags[r] = flag_bases[r];
    }
    gg->epochs.assign(max_layers, 0);
    cudaError_t e = cudaMalloc(&gg->tickets, sizeof(uint32_t) * (size_t)max_layers);
    if (e == cudaSuccess) e = cudaMemset(gg->tickets, 0, sizeof(uint32_t) * (size_t)max_layers);
    if (e != cudaSuccess) {
        cudaFree(gg->tickets);
        delete gg;
        return cuda_fail(e, "gkv_gather_create");
    }
    *out = gg;
    return GKV_OK;
}

int gkv_gather_set_wait_limit(gkv_gather* gg, uint64_t limit_ns) {
    if (!gg || limit_ns < 1000ull || limit_ns > 10ull * 1000 * 1000 * 1000)
        return fail(GKV_ERR_INVALID, "gkv_gather_set_wait_limit: limit must be 1 us to 10 s");
    gg->wait_ns = limit_ns;
    return GKV_OK;
}

int gkv_gather_destroy(gkv_gather* gg) {
    if (!gg) return GKV_OK;
    DeviceGuard g(gg->device);
    cudaFree(gg->tickets);
    delete gg;
    return GKV_OK;
}

int gkv_paged_attention_gather(gkv_manager* m, int32_t layer_id, const void* Q, const void* K, const void* V,
                               gkv_gather* gg, size_t out_offset, int32_t n_q_heads, float scale, int32_t out_dtype,
                               gkv_stream_t stream) {
    NvtxRange nvtx_range("gkv decode + head all-gather");
    if (!gg) return fail(GKV_ERR_INVALID, "null gather");
    if (layer_id < 0 || layer_id >= gg->max_layers) return fail(GKV_ERR_INVALID, "layer %d beyond the gather's %d",
                                                             layer_id, gg->max_layers);
    if (m->device != gg->device) return fail(GKV_ERR_INVALID, "manager and gather on different devices");
    const Layer* L = find_layer(m, layer_id);
    if (!L || !L->reserved) return fail(GKV_ERR_STATE, "layer %d not reserved", layer_id);
    const size_t esize = out_dtype == GKV_F32 ? 4 : 2;
    const size_t block = (size_t)n_q_heads * 128 * esize;
    if (out_offset % 16 != 0) return fail(GKV_ERR_INVALID, "out_offset must be 16-byte aligned");
    gkv::GatherLaunch gl{};
    gl.world = gg->world;
    gl.rank = gg->rank;
    // Flags pushed (default): this rank stores its flag into every rank's
    // array and polls its own. Pulled (GKV_GATHER_FLAGS=pull): it stores only
    // into its own array and polls the peers' over NVLink, so that the
    // combine issues no remote store after its fence.
    const bool pull = gather_flags_pulled();
    gl.n_flag_dst = pull ? 1 : gg->world;
    for (int r = 0; r < gg->world; ++r) {
        gl.dst[r] = static_cast<char*>(gg->bases[r]) + out_offset + (size_t)gg->rank * block;
        if (!pull) gl.flag_dst[r] = gg->flags[r] + (size_t)layer_id * gg->world + gg->rank;
        gl.flag_wait[r] = pull ? gg->flags[r] + (size_t)layer_id * gg->world + r
                               : gg->flags[gg->rank] + (size_t)layer_id * gg->world + r;
    }
    if (pull) gl.flag_dst[0] = gg->flags[gg->rank] + (size_t)layer_id * gg->world + gg->rank;
    gl.epoch = gg->epochs[layer_id] + 1;
    gl.ticket = gg->tickets + layer_id;
    gl.wait_ns = gg->wait_ns;
    // The managed decode path, with this gather attached to its combine launch.
    t_gather = &gl;
    const int st = gkv_paged_attention(m, layer_id, Q, K, V, gl.dst[gg->rank], 1, n_q_heads, 1, 128, L->n_kv_heads,
                                       scale, 1, n_q_heads / L->n_kv_heads, L->dtype, out_dtype, stream);
    t_gather = nullptr;
    if (st == GKV_OK) gg->epochs[layer_id] = gl.epoch;
    return st;
}

}  // extern "C"
