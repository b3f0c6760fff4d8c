// noalloc.cu — a decode entry point that allocates no device memory.
//
// Some callers cannot call cudaMalloc: code running inside a host
// framework that owns every device allocation through its own arena (and
// forbids side allocations), plugins loaded into a process whose allocator
// is locked down, or real-time loops where an allocation's latency and
// possible implicit synchronisation are not acceptable. They still need the
// split-K decode, whose partial results live in scratch memory. This file
// gives that scratch a fixed home: a file-scope __device__ array that every
// GPU loading the library holds until the process exits.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/genllm_kv.h"
#include "kernels.h"

namespace gkv {
namespace {

// Capacity: kStaticRows (split x query-head) partial rows.
constexpr int kStaticRows = 4096;
constexpr size_t kAccBytes = (size_t)kStaticRows * kHeadDim * sizeof(float);  // 2 MiB
constexpr size_t kMlBytes = (size_t)kStaticRows * sizeof(float2);             // 32 KiB
constexpr size_t kScratchBytes = kAccBytes + kMlBytes + 256;                   // + error word

// The shared scratch. Host code must not pass this name to a kernel: on the
// host it only stands for the symbol; its device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_static_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_addr[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};

int fail(int status, const char* what) {
    set_last_error(what);  // reported by gkv_last_error()
    return status;
}

}  // namespace
}  // namespace gkv

extern "C" int gkv_paged_decode_static_scratch(const gkv_pool_desc* pool, const int32_t* device_table,
                                               int32_t n_prior, const void* Q, const void* K, const void* V,
                                               void* out, int32_t n_q_heads, float scale, int32_t out_dtype,
                                               gkv_stream_t stream) {
    using namespace gkv;
    if (!pool || !device_table || n_prior < 0 || !Q || !K || !V || !out)
        return fail(GKV_ERR_INVALID, "null argument or negative n_prior");
    if (pool->head_dim != kHeadDim || pool->dtype != GKV_BF16)
        return fail(GKV_ERR_UNSUPPORTED, "only head_dim 128 and bf16 pages are built");
    if (pool->n_kv_heads < 1 || pool->n_kv_heads > 8 || pool->pool_pages < 1)
        return fail(GKV_ERR_UNSUPPORTED, "1 to 8 kv heads per GPU");
    if (n_q_heads < 1 || n_q_heads % pool->n_kv_heads) return fail(GKV_ERR_INVALID, "n_q_heads not a multiple of n_kv_heads");
    const int G = n_q_heads / pool->n_kv_heads;
    if (G != 1 && G != 2 && G != 4 && G != 8) return fail(GKV_ERR_UNSUPPORTED, "group size must be 1, 2, 4 or 8");
    if (out_dtype != GKV_F32 && out_dtype != GKV_F16 && out_dtype != GKV_BF16)
        return fail(GKV_ERR_UNSUPPORTED, "output dtype");
    const int32_t total = n_prior + 1;
    const int32_t n_pages = (total + kPageSlots - 1) / kPageSlots;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return fail(GKV_ERR_CUDA, "cannot query the current device");
    unsigned char* base = nullptr;
    int sms = 0;
    {
        // Once per device: the scratch's device address (no allocation).
        std::lock_guard<std::mutex> lock(g_mu);
        if (!g_addr[dev]) {
            void* p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
            if (e != cudaSuccess) return fail(GKV_ERR_CUDA, cudaGetErrorString(e));
            if (cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
                return fail(GKV_ERR_CUDA, "cannot query the SM count");
            g_addr[dev] = static_cast<unsigned char*>(p);
        }
        base = g_addr[dev];
        sms = g_sms[dev];
    }
    // Splits are capped so that the partial rows (splits x query heads) fit
    // the static rows; the geometry the launch will use (which may add
    // splits for very long contexts) is checked against the same bound.
    int n_splits = sms;
    if (n_splits * n_q_heads > kStaticRows) n_splits = kStaticRows / n_q_heads;
    if (n_splits < 1) return fail(GKV_ERR_UNSUPPORTED, "too many query heads for the static scratch");
    int32_t pages_per_split = 0, used_splits = 0;
    if (!decode_split_geometry(n_pages, pool->n_kv_heads, n_q_heads, n_splits, sms, &pages_per_split, &used_splits) ||
        (long long)used_splits * n_q_heads > kStaticRows)
        return fail(GKV_ERR_INVALID, "context longer than the static scratch supports");

    PoolView pv{static_cast<uint16_t*>(pool->k_base), static_cast<uint16_t*>(pool->v_base), pool->pool_pages,
                pool->n_kv_heads};
    DecodeMaps maps;
    const char* why = nullptr;
    if (!encode_decode_maps(pv, &maps, &why)) return fail(GKV_ERR_CUDA, why);

    Scratch sc;
    sc.part_acc = reinterpret_cast<float*>(base);
    sc.part_ml = reinterpret_cast<float2*>(base + kAccBytes);
    sc.err = reinterpret_cast<uint32_t*>(base + kAccBytes + kMlBytes);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // The error word is the only part that must start at zero.
    cudaError_t e = cudaMemsetAsync(sc.err, 0, sizeof(uint32_t), s);
    if (e != cudaSuccess) return fail(GKV_ERR_CUDA, cudaGetErrorString(e));

    NewPages np;
    np.first = 0;
    np.n = 0;  // every entry, the new token's page included, is already in device_table
    DecodeLaunch d{};
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
    d.n_splits = n_splits;
    e = launch_decode(pv, maps, reinterpret_cast<int2*>(const_cast<int32_t*>(device_table)), np, sc, d, sms, s);
    if (e != cudaSuccess) return fail(GKV_ERR_CUDA, cudaGetErrorString(e));
    return GKV_OK;
}

extern "C" int gkv_paged_decode_static_scratch_errors(uint32_t* flags, gkv_stream_t stream) {
    using namespace gkv;
    if (!flags) return fail(GKV_ERR_INVALID, "null flags");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return fail(GKV_ERR_CUDA, "cannot query the current device");
    unsigned char* base = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        base = g_addr[dev];
    }
    if (!base) {  // no decode call on this device yet
        *flags = 0;
        return GKV_OK;
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint32_t v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, base + kAccBytes + kMlBytes, sizeof(v), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(GKV_ERR_CUDA, cudaGetErrorString(e));
    *flags = v;
    return GKV_OK;
}
