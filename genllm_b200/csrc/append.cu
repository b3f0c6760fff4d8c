// append.cu — scatter a chunk of K/V tokens into their pages (one launch).
//
// Replaces the reference's per-(token, head) synchronous cudaMemcpy loop
// (src/core/page_attention.cpp:122-139): token p of head h, a 256-byte row
// of K[h][p][:], lands at page(table[(n_prior+p)/16]) + ((n_prior+p)%16 * Hkv
// + h) * 128 elements, in K's pool; the same for V. A warp fills one page
// slot ([Hkv][128] contiguous) with 16-byte units, consecutive lanes on
// consecutive bytes. Pure byte copy: bit-exact by design.
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
    int32_t pdl;  // kAppendDependent | kAppendTrigger
    int2 new_ids[kMaxNewPagesPerLaunch];
};

constexpr int kAppendWarps = 4;

// One warp per (token, K|V): the token's Hkv rows (one per head, src_len
// rows apart in the input) land in one contiguous page slot [Hkv][128]. Each
// lane loads its 16-byte units of the slot before the table entry is known
// (the source does not depend on it), so the two latencies overlap; then it
// stores them in slot order (consecutive lanes, consecutive bytes).
__global__ void __launch_bounds__(kAppendWarps * 32) kv_append_kernel(const AppendParams a) {
    // The chunked-prefill kernel that follows may start at once: it waits for
    // this kernel before it reads anything this kernel writes (or, reading
    // the chunk's own tiles from the inputs, before its output stores).
    if (a.pdl & kAppendTrigger) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // As a programmatic dependent: nothing of the previous kernel's output
    // (pages, table, the K/V source) is touched before it has completed.
    if (a.pdl & kAppendDependent) asm volatile("griddepcontrol.wait;" ::: "memory");
    if (blockIdx.x == 0 && (int)threadIdx.x < a.new_n)
        a.table[a.new_first + threadIdx.x] = a.new_ids[threadIdx.x];

    constexpr int kUnitsPerRow = kHeadDim * 2 / 16;  // 16-byte units in a 256-byte row
    constexpr int kBatch = 4;                        // units per lane in flight
    const int lane = threadIdx.x & 31;
    const int Hkv = a.n_kv_heads;
    const int units = Hkv * kUnitsPerRow;            // units of one page slot
    const int n_items = 2 * a.count;
    for (int w = blockIdx.x * kAppendWarps + (int)(threadIdx.x >> 5); w < n_items; w += gridDim.x * kAppendWarps) {
        const int which = w & 1;  // 0 = K, 1 = V
        const int p = a.p_begin + (w >> 1);
        const int pos = a.n_prior + p;
        const int lp = pos / kPageSlots;
        const int slot = pos % kPageSlots;
        int page = 0;
        if (lane == 0) {
            const int rr = lp - a.new_first;
            const int2 e = (rr >= 0 && rr < a.new_n) ? a.new_ids[rr] : a.table[lp];
            page = which ? e.y : e.x;
        }
        const uint4* src = which ? a.v : a.k;
        uint4* dst = which ? a.v_base : a.k_base;
        for (int u0 = 0; u0 < units; u0 += 32 * kBatch) {
            uint4 buf[kBatch];
#pragma unroll
            for (int b = 0; b < kBatch; ++b) {
                const int j = u0 + b * 32 + lane;
                if (j < units) {
                    const int h = j / kUnitsPerRow, d16 = j % kUnitsPerRow;
                    buf[b] = __ldg(src + ((size_t)h * a.src_len + p) * kUnitsPerRow + d16);
                }
            }
            const int pg = __shfl_sync(0xFFFFFFFFu, page, 0);
            if (pg < 0 || pg >= a.pool_pages) {
                if (lane == 0 && u0 == 0) atomicOr(a.err, kErrBadPage);
                continue;
            }
            uint4* slot_base = dst + ((size_t)pg * kPageSlots + slot) * units;
#pragma unroll
            for (int b = 0; b < kBatch; ++b) {
                const int j = u0 + b * 32 + lane;
                if (j < units) slot_base[j] = buf[b];
            }
        }
    }
}

}  // namespace

cudaError_t launch_append(const PoolView& pool, int2* table, const NewPages& np,
                          const uint16_t* k, const uint16_t* v, int32_t n_prior,
                          int32_t src_len, int32_t p_begin, int32_t p_end, uint32_t* err,
                          cudaStream_t stream, int pdl) {
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
    a.pdl = pdl;
    for (int i = 0; i < np.n; ++i) a.new_ids[i] = np.ids[i];
    long long blocks = (2ll * a.count + kAppendWarps - 1) / kAppendWarps;
    if (blocks < 1) blocks = 1;
    if (blocks > 148 * 16) blocks = 148 * 16;
    // Ahead of a prefill launch (which starts while this one waits for its
    // predecessor): one CTA per SM, so that a waiting append CTA never keeps
    // a prefill CTA (168 x 352 registers) off an SM.
    if ((pdl & kAppendTrigger) && blocks > 148) blocks = 148;
    if (!(pdl & kAppendDependent)) {
        kv_append_kernel<<<(unsigned)blocks, kAppendWarps * 32, 0, stream>>>(a);
        return cudaGetLastError();
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(kAppendWarps * 32);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kv_append_kernel, a);
}

}  // namespace gkv
