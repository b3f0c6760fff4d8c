// append.cu — scatter a chunk of K/V tokens into their pages (one launch).
//
// Replaces the reference's per-(token, head) synchronous cudaMemcpy loop
// (src/core/page_attention.cpp:122-139): token p of head h, a 256-byte row
// of K[h][p][:], lands at page(table[(n_prior+p)/16]) + ((n_prior+p)%16 * Hkv
// + h) * 128 elements, in K's pool; the same for V. Each thread moves 16-byte
// units ordered so that consecutive threads write consecutive bytes of a
// page slot ([Hkv][128] contiguous). Pure byte copy: bit-exact by design.
#include "device.cuh"
#include "kernels.h"

namespace gkv {
namespace {

struct AppendParams {
    const uint4* k;
    const uint4* v;
    uint4* k_base;
    uint4* v_base;
    int2* table;
    uint32_t* err;
    int32_t n_prior;
    int32_t src_len;  // token stride of the K/V inputs
    int32_t p_begin;  // first source token of this launch
    int32_t count;    // tokens moved by this launch
    int32_t n_kv_heads;
    int32_t pool_pages;
    int32_t new_first;
    int32_t new_n;
    int2 new_ids[kMaxNewPagesPerLaunch];
};

__global__ void __launch_bounds__(256) kv_append_kernel(const AppendParams a) {
    if (blockIdx.x == 0 && (int)threadIdx.x < a.new_n)
        a.table[a.new_first + threadIdx.x] = a.new_ids[threadIdx.x];

    constexpr int kUnitsPerRow = kHeadDim * 2 / 16;  // 16-byte units in a 256-byte row
    const int Hkv = a.n_kv_heads;
    const long long units = 2ll * a.count * Hkv * kUnitsPerRow;
    for (long long u = blockIdx.x * (long long)blockDim.x + threadIdx.x; u < units;
         u += (long long)gridDim.x * blockDim.x) {
        const int d16 = (int)(u % kUnitsPerRow);
        long long r = u / kUnitsPerRow;
        const int h = (int)(r % Hkv);
        r /= Hkv;
        const int p = a.p_begin + (int)(r % a.count);
        const int which = (int)(r / a.count);  // 0 = K, 1 = V
        const int pos = a.n_prior + p;
        const int lp = pos / kPageSlots;
        const int slot = pos % kPageSlots;
        const int rr = lp - a.new_first;
        const int2 e = (rr >= 0 && rr < a.new_n) ? a.new_ids[rr] : a.table[lp];
        const int page = which ? e.y : e.x;
        if (page < 0 || page >= a.pool_pages) {
            atomicOr(a.err, kErrBadPage);
            continue;
        }
        const uint4* src = which ? a.v : a.k;
        uint4* dst = which ? a.v_base : a.k_base;
        const size_t s_idx = ((size_t)h * a.src_len + p) * kUnitsPerRow + d16;
        const size_t d_idx = (((size_t)page * kPageSlots + slot) * Hkv + h) * kUnitsPerRow + d16;
        dst[d_idx] = __ldg(src + s_idx);
    }
}

}  // namespace

cudaError_t launch_append(const PoolView& pool, int2* table, const NewPages& np,
                          const uint16_t* k, const uint16_t* v, int32_t n_prior,
                          int32_t src_len, int32_t p_begin, int32_t p_end, uint32_t* err,
                          cudaStream_t stream) {
    AppendParams a;
    a.k = reinterpret_cast<const uint4*>(k);
    a.v = reinterpret_cast<const uint4*>(v);
    a.k_base = reinterpret_cast<uint4*>(pool.k_base);
    a.v_base = reinterpret_cast<uint4*>(pool.v_base);
    a.table = table;
    a.err = err;
    a.n_prior = n_prior;
    a.src_len = src_len;
    a.p_begin = p_begin;
    a.count = p_end - p_begin;
    a.n_kv_heads = pool.n_kv_heads;
    a.pool_pages = pool.pool_pages;
    a.new_first = np.first;
    a.new_n = np.n;
    for (int i = 0; i < np.n; ++i) a.new_ids[i] = np.ids[i];
    const long long units = 2ll * a.count * pool.n_kv_heads * (kHeadDim * 2 / 16);
    long long blocks = (units + 255) / 256;
    if (blocks < 1) blocks = 1;
    if (blocks > 148 * 16) blocks = 148 * 16;
    kv_append_kernel<<<(unsigned)blocks, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace gkv
