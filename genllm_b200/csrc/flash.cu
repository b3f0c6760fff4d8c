// flash.cu — the reference's non-paged attention op (FlashAttentionImpl<CUDA>,
// src/backend/cuda/attention.cu:317-399; CPU semantics in
// src/backend/cpu/attention.cpp:39-120): self-attention of B sequences of
// seq_len tokens with contiguous Q/K/V, on the tcgen05 chunked-prefill kernel
// (prefill_tc.cu) with its K/V tiles copied straight from the tensors.
// Allocates nothing: its device error word is a file-scope __device__ word.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/genllm_kv.h"
#include "kernels.h"

namespace gkv {
namespace {

constexpr int kMaxDevices = 64;
static __device__ uint32_t g_flash_err;

std::mutex g_mu;
uint32_t* g_err_addr[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};

int fail(int status, const char* what) {
    set_last_error(what);
    return status;
}

// The current device's error word address and SM count (looked up once).
int device_state(uint32_t** err, int* sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return fail(GKV_ERR_CUDA, "cannot query the current device");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_err_addr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_flash_err);
        if (e != cudaSuccess) return fail(GKV_ERR_CUDA, cudaGetErrorString(e));
        if (cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return fail(GKV_ERR_CUDA, "cannot query the SM count");
        g_err_addr[dev] = static_cast<uint32_t*>(p);
    }
    *err = g_err_addr[dev];
    *sms = g_sms[dev];
    return GKV_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace gkv

extern "C" int gkv_flash_attention(const void* Q, const void* K, const void* V, void* out, int32_t batch,
                                   int32_t n_q_heads, int32_t n_kv_heads, int32_t seq_len, int32_t head_dim,
                                   float scale, int32_t causal, int32_t dtype, int32_t out_dtype,
                                   gkv_stream_t stream) {
    using namespace gkv;
    if (!Q || !K || !V || !out || batch < 1 || seq_len < 1 || n_q_heads < 1 || n_kv_heads < 1)
        return fail(GKV_ERR_INVALID, "gkv_flash_attention: bad arguments");
    if (head_dim != kHeadDim || dtype != GKV_BF16)
        return fail(GKV_ERR_UNSUPPORTED, "only head_dim 128 and bf16 Q/K/V are built");
    if (out_dtype != GKV_F32 && out_dtype != GKV_F16 && out_dtype != GKV_BF16)
        return fail(GKV_ERR_UNSUPPORTED, "output dtype");
    if (n_q_heads % n_kv_heads) return fail(GKV_ERR_INVALID, "n_q_heads not a multiple of n_kv_heads");
    const int G = n_q_heads / n_kv_heads;
    if (G != 1 && G != 2 && G != 4 && G != 8) return fail(GKV_ERR_UNSUPPORTED, "group size must be 1, 2, 4 or 8");
    if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(out))
        return fail(GKV_ERR_INVALID, "Q/K/V/out must be 16-byte aligned");
    if ((long long)batch * n_q_heads > 65535) return fail(GKV_ERR_UNSUPPORTED, "batch x heads above 65535");
    uint32_t* err = nullptr;
    int sms = 0;
    int st = device_state(&err, &sms);
    if (st) return st;
    CUtensorMap q_map, k_map, v_map;
    const char* why = nullptr;
    if (!encode_q_map_sw128(static_cast<const uint16_t*>(Q), batch * n_q_heads, seq_len, &q_map, &why) ||
        !encode_contig_kv_maps_sw128(static_cast<const uint16_t*>(K), static_cast<const uint16_t*>(V), seq_len,
                                     batch * n_kv_heads, &k_map, &v_map, &why))
        return fail(GKV_ERR_CUDA, why);
    FlashLaunch f{out, out_dtype, batch, n_q_heads, n_kv_heads, seq_len, scale, causal ? 1 : 0};
    cudaError_t e = launch_flash_tc(q_map, k_map, v_map, f, err, sms, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(GKV_ERR_CUDA, cudaGetErrorString(e));
    return GKV_OK;
}

extern "C" int gkv_flash_check_errors(uint32_t* flags) {
    using namespace gkv;
    uint32_t* err = nullptr;
    int sms = 0;
    int st = device_state(&err, &sms);
    if (st) return st;
    uint32_t v = 0;
    cudaError_t e = cudaMemcpy(&v, err, sizeof v, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(err, 0, sizeof v);
    if (e != cudaSuccess) return fail(GKV_ERR_CUDA, cudaGetErrorString(e));
    if (flags) *flags = v;
    return v ? GKV_ERR_DEVICE : GKV_OK;
}
