// export.cu — KV page format export and import.
//
// The reference keeps a layer's cache only in its page layout
// (src/core/page_attention.cpp:128: page(id) + (slot * Hkv + h) * D) and has
// no way to read it back out. These kernels move a layer's first n_tokens
// tokens between the pages and a dense head-major copy [Hkv][n_tokens][128]
// (the layout append_kv_from_tensor takes, src/core/page_attention.cpp:104-139),
// either in the pool's bf16 (a byte copy, so export followed by append is the
// identity) or as fp8 e4m3 with one fp32 scale per (head, 16-token block):
//
//   amax  = max |x| over the block's finite elements (0 when there are none)
//   scale = amax / 448, inv = 448 / amax      (IEEE divisions; both 1 when
//                                               448 / amax is not finite)
//   q     = e4m3(x * inv)                      (round to nearest even, finite
//                                               values saturate at +-448, NaN -> 0x7F)
//   x'    = bf16(e4m3_value(q) * scale)        (import: the reference's bf16 rounding)
//
// One warp per (K|V, page, head) unit for the export: it copies the unit's
// 16 rows of 256 bytes into its shared-memory ring with cp.async (two slots
// per instruction), kRing - 1 units ahead of the one it converts; reduces the
// block's amax with shuffles, and writes the 16 rows of the head-major
// output, which are contiguous. The import is the same with one warp per
// (K|V, 16-token block, head). Both directions are a single pass over HBM:
// read 2 B and write 1 B (fp8) or 2 B (bf16) per element. The hardware
// conversions are used only where they give the rounding defined above
// bit for bit (see each kernel); elsewhere the element-wise path runs.
#include <atomic>

#include "device.cuh"
#include "kernels.h"

namespace gkv {
namespace {

struct ExportParams {
    const uint4* k_base;
    const uint4* v_base;
    const int2* table;
    uint32_t* err;
    void* k_out;
    void* v_out;
    float* k_scales;  // [Hkv][n_pages] (fp8 only)
    float* v_scales;
    int32_t n_tokens;
    int32_t n_pages;
    int32_t n_kv_heads;
    int32_t pool_pages;
    int32_t fp8;
};

// Eight bf16 values (one 16-byte unit) to fp32.
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = bf16_lo(w[i]);
        f[2 * i + 1] = bf16_hi(w[i]);
    }
}

// Two fp32 values to e4m3 (RNE, satfinite); lo lands in the low byte.
__device__ __forceinline__ uint32_t e4m3x2_raw(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

// Four fp32 values to four e4m3 bytes of one word (a0 in the low byte).
__device__ __forceinline__ uint32_t e4m3x4_raw(float a0, float a1, float a2, float a3) {
    uint32_t d;
    asm("{\n\t.reg .b16 l, h;\n\t"
        "cvt.rn.satfinite.e4m3x2.f32 l, %2, %1;\n\t"
        "cvt.rn.satfinite.e4m3x2.f32 h, %4, %3;\n\t"
        "mov.b32 %0, {l, h};\n\t}"
        : "=r"(d)
        : "f"(a0), "f"(a1), "f"(a2), "f"(a3));
    return d;
}

// The same for blocks that may hold NaN: NaN inputs encode as 0x7F whatever
// the hardware conversion gives for them.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
    uint32_t v = e4m3x2_raw(lo, hi);
    if (lo != lo) v = (v & 0xFF00u) | 0x7Fu;
    if (hi != hi) v = (v & 0x00FFu) | 0x7F00u;
    return v;
}

// Per-thread asynchronous global -> shared copies (cp.async): src_size 0
// writes zeros and reads nothing. Each thread later reads back only what it
// copied itself, so waiting on its own groups is all the ordering needed.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(valid ? 8 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Units in flight per warp: the one being converted and kRing - 1 prefetched.
constexpr int kRing = 3;

// One (K|V, page, head) unit of the export: where its rows are and how many.
struct ExportUnit {
    const uint4* src;  // this lane's first 16-byte unit, null for a bad page id
    size_t row0;       // first output row (h * n_tokens + lp * 16)
    int h, lp, which, valid;
};

__device__ __forceinline__ ExportUnit export_unit(const ExportParams& a, long long u, int half, int col) {
    constexpr int kUnitsPerRow = kHeadDim * 2 / 16;
    ExportUnit x;
    // Consecutive warps take the heads of one page: a CTA reads a page's
    // contiguous [16][Hkv][128] region together.
    x.h = (int)(u % a.n_kv_heads);
    const long long r = u / a.n_kv_heads;
    x.lp = (int)(r % a.n_pages);
    x.which = (int)(r / a.n_pages);
    const int2 e = a.table[x.lp];
    const int page = x.which ? e.y : e.x;
    x.valid = min(kPageSlots, a.n_tokens - x.lp * kPageSlots);
    x.row0 = (size_t)x.h * a.n_tokens + (size_t)x.lp * kPageSlots;
    x.src = (page < 0 || page >= a.pool_pages)
                ? nullptr
                : (x.which ? a.v_base : a.k_base) + ((size_t)page * kPageSlots * a.n_kv_heads + x.h) * kUnitsPerRow + col;
    return x;
}

// Start the copies of a unit's 16 rows (this lane's 16-byte column of each)
// into ring slot `buf` ([16 slots][16 columns] of uint4); rows past the
// valid tokens and the rows of a bad page id land as zeros.
__device__ __forceinline__ void export_issue(const ExportParams& a, const ExportUnit& x, bool live, int half,
                                             int col, uint32_t buf) {
    constexpr int kUnitsPerRow = kHeadDim * 2 / 16;
    if (live) {
#pragma unroll
        for (int i = 0; i < kPageSlots / 2; ++i) {
            const int slot = 2 * i + half;
            const bool ok = x.src && slot < x.valid;
            cp_async16(buf + (slot * kUnitsPerRow + col) * 16,
                       ok ? (const void*)(x.src + (size_t)slot * a.n_kv_heads * kUnitsPerRow) : (const void*)a.k_base,
                       ok);
        }
    }
    cp_async_commit();
}

// Grid-stride over units, one warp per unit, persistent grid. Each warp keeps
// kRing - 1 units' copies in flight (a per-warp ring in shared memory) while
// it reduces, converts and stores the current one.
__global__ void __launch_bounds__(256, 2) kv_export_kernel(const ExportParams a) {
    constexpr int kUnitsPerRow = kHeadDim * 2 / 16;  // 16 x 16-byte units per 256-byte row
    constexpr uint32_t kBufBytes = kPageSlots * kHeadDim * 2;  // 4 KiB: one unit
    extern __shared__ __align__(16) uint8_t export_smem[];
    const int lane = threadIdx.x & 31;
    const int half = lane >> 4;   // slot parity this lane reads
    const int col = lane & 15;    // 16-byte unit within the row
    const long long units = 2ll * a.n_pages * a.n_kv_heads;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    long long u = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5);
    if (u >= units) return;
    const uint32_t ring = smem_addr(export_smem) + (threadIdx.x >> 5) * kRing * kBufBytes;
    const uint4* ring_p = reinterpret_cast<const uint4*>(export_smem + (threadIdx.x >> 5) * kRing * kBufBytes);

    // prologue: units u, u + W, ... in ring slots 0 .. kRing - 2
    ExportUnit info[kRing - 1];
#pragma unroll
    for (int k = 0; k < kRing - 1; ++k) {
        const long long uu = u + k * warps;
        info[k] = uu < units ? export_unit(a, uu, half, col) : ExportUnit{};
        export_issue(a, info[k], uu < units, half, col, ring + k * kBufBytes);
    }
    for (int it = 0; u < units; u += warps, ++it) {
        const ExportUnit cur = info[0];
        // refill: the slot read in the previous iteration takes unit u + (kRing-1) W
        {
            const long long uu = u + (kRing - 1) * warps;
            const ExportUnit nx = uu < units ? export_unit(a, uu, half, col) : ExportUnit{};
            export_issue(a, nx, uu < units, half, col, ring + ((it + kRing - 1) % kRing) * kBufBytes);
#pragma unroll
            for (int k = 0; k < kRing - 2; ++k) info[k] = info[k + 1];
            info[kRing - 2] = nx;
        }
        cp_async_wait<kRing - 1>();  // this unit's group is complete
        const uint4* bp = ring_p + (it % kRing) * (kBufBytes / 16) + col;
        uint4 x[kPageSlots / 2];
#pragma unroll
        for (int i = 0; i < kPageSlots / 2; ++i) x[i] = bp[(2 * i + half) * kUnitsPerRow];
        if (!cur.src) {
            if (lane == 0) atomicOr(a.err, kErrBadPage);
        } else if (!a.fp8) {
            uint4* dst = static_cast<uint4*>(cur.which ? a.v_out : a.k_out) + cur.row0 * kUnitsPerRow + col;
#pragma unroll
            for (int i = 0; i < kPageSlots / 2; ++i) {
                const int slot = 2 * i + half;
                if (slot < cur.valid) __stcs(dst + (size_t)slot * kUnitsPerRow, x[i]);
            }
        } else {
            // |x| of a bf16 orders like its bit pattern with the sign cleared;
            // patterns from 0x7F80 up are infinities and NaNs. Fast path: a
            // packed max over both halves of each word, reduced over the warp;
            // a block whose max is non-finite redoes it without those values.
            uint32_t m2 = 0;
#pragma unroll
            for (int i = 0; i < kPageSlots / 2; ++i) {
                m2 = __vmaxu2(m2, x[i].x & 0x7FFF7FFFu);
                m2 = __vmaxu2(m2, x[i].y & 0x7FFF7FFFu);
                m2 = __vmaxu2(m2, x[i].z & 0x7FFF7FFFu);
                m2 = __vmaxu2(m2, x[i].w & 0x7FFF7FFFu);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m2 = __vmaxu2(m2, __shfl_xor_sync(0xffffffffu, m2, o));
            uint32_t mbits = max(m2 & 0xFFFFu, m2 >> 16);
            const bool any_nonfinite = mbits >= 0x7F80u;  // warp-uniform
            if (any_nonfinite) {
                mbits = 0;
#pragma unroll
                for (int i = 0; i < kPageSlots / 2; ++i) {
                    const uint32_t w[4] = {x[i].x, x[i].y, x[i].z, x[i].w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t lo = w[j] & 0x7FFFu, hi = (w[j] >> 16) & 0x7FFFu;
                        if (lo < 0x7F80u) mbits = max(mbits, lo);
                        if (hi < 0x7F80u) mbits = max(mbits, hi);
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) mbits = max(mbits, __shfl_xor_sync(0xffffffffu, mbits, o));
            }
            const float amax = __uint_as_float(mbits << 16);
            // A block whose 448 / amax is not finite (amax 0, or below ~2^-119)
            // keeps scale 1: its values round to signed zeros.
            float inv = __fdiv_rn(448.f, amax);
            const bool unit = !(inv < __int_as_float(0x7f800000));
            const float scale = unit ? 1.f : __fdiv_rn(amax, 448.f);
            if (unit) inv = 1.f;
            uint2* dst = static_cast<uint2*>(cur.which ? a.v_out : a.k_out) + cur.row0 * kUnitsPerRow + col;
#pragma unroll
            for (int i = 0; i < kPageSlots / 2; ++i) {
                const int slot = 2 * i + half;
                if (slot >= cur.valid) continue;
                float f[8];
                unpack8(x[i], f);
                uint2 q;
                if (!any_nonfinite) {
                    q.x = e4m3x4_raw(__fmul_rn(f[0], inv), __fmul_rn(f[1], inv), __fmul_rn(f[2], inv),
                                     __fmul_rn(f[3], inv));
                    q.y = e4m3x4_raw(__fmul_rn(f[4], inv), __fmul_rn(f[5], inv), __fmul_rn(f[6], inv),
                                     __fmul_rn(f[7], inv));
                } else {
                    q.x = e4m3x2(__fmul_rn(f[0], inv), __fmul_rn(f[1], inv)) |
                          (e4m3x2(__fmul_rn(f[2], inv), __fmul_rn(f[3], inv)) << 16);
                    q.y = e4m3x2(__fmul_rn(f[4], inv), __fmul_rn(f[5], inv)) |
                          (e4m3x2(__fmul_rn(f[6], inv), __fmul_rn(f[7], inv)) << 16);
                }
                __stcs(dst + (size_t)slot * kUnitsPerRow, q);
            }
            if (lane == 0) (cur.which ? a.v_scales : a.k_scales)[(size_t)cur.h * a.n_pages + cur.lp] = scale;
        }
    }
    cp_async_wait<0>();
}

// The bf16 export is a byte copy: no ring, few registers, many warps. One
// warp per (K|V, page, head) unit, 8 x 16 bytes in flight per lane.
__global__ void __launch_bounds__(256, 4) kv_export_bf16_kernel(const ExportParams a) {
    constexpr int kUnitsPerRow = kHeadDim * 2 / 16;
    const int lane = threadIdx.x & 31;
    const int half = lane >> 4;
    const int col = lane & 15;
    const long long units = 2ll * a.n_pages * a.n_kv_heads;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    for (long long u = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); u < units; u += warps) {
        const ExportUnit x = export_unit(a, u, half, col);
        if (!x.src) {
            if (lane == 0) atomicOr(a.err, kErrBadPage);
            continue;
        }
        uint4 v[kPageSlots / 2];
#pragma unroll
        for (int i = 0; i < kPageSlots / 2; ++i) {
            const int slot = 2 * i + half;
            if (slot < x.valid) v[i] = __ldcs(x.src + (size_t)slot * a.n_kv_heads * kUnitsPerRow);
        }
        uint4* dst = static_cast<uint4*>(x.which ? a.v_out : a.k_out) + x.row0 * kUnitsPerRow + col;
#pragma unroll
        for (int i = 0; i < kPageSlots / 2; ++i) {
            const int slot = 2 * i + half;
            if (slot < x.valid) __stcs(dst + (size_t)slot * kUnitsPerRow, v[i]);
        }
    }
}

struct ImportParams {
    const uint2* k_in;  // [Hkv][seq_len][128] e4m3
    const uint2* v_in;
    const float* k_scales;  // [Hkv][ceil(seq_len / 16)]
    const float* v_scales;
    uint4* k_base;
    uint4* v_base;
    const int2* table;
    uint32_t* err;
    int32_t n_prior;
    int32_t seq_len;
    int32_t n_blocks;
    int32_t n_kv_heads;
    int32_t pool_pages;
};

// e4m3 byte pair (lo byte first) to two fp32 values; exact.
__device__ __forceinline__ float2 e4m3x2_to_f32(uint32_t b) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"((uint16_t)b));
    const __half2 h = *reinterpret_cast<const __half2*>(&h2);
    return __half22float2(h);
}

// One warp per (K|V, 16-token input block, head) unit: each half-warp reads a
// token's 128-byte e4m3 row (8 bytes a lane) and writes its 256-byte page row
// (16 bytes a lane); 8 rows per lane, kRing - 1 units' copies in flight in
// the warp's shared-memory ring while the current unit is converted.
struct ImportUnit {
    const uint2* src;  // this lane's first 8-byte unit
    float scale;
    int h, p0, which, valid;
    bool fast;         // 2^-117 <= scale < inf: hardware bf16 rounding is exact
};

__device__ __forceinline__ ImportUnit import_unit(const ImportParams& a, long long u, int col) {
    constexpr int kUnitsPerRow = kHeadDim / 8;
    ImportUnit x;
    x.h = (int)(u % a.n_kv_heads);
    const long long r = u / a.n_kv_heads;
    const int b = (int)(r % a.n_blocks);
    x.which = (int)(r / a.n_blocks);
    x.p0 = b * kPageSlots;
    x.valid = min(kPageSlots, a.seq_len - x.p0);
    x.scale = (x.which ? a.v_scales : a.k_scales)[(size_t)x.h * a.n_blocks + b];
    x.fast = x.scale >= 0x1p-117f && x.scale < __int_as_float(0x7f800000);
    x.src = (x.which ? a.v_in : a.k_in) + ((size_t)x.h * a.seq_len + x.p0) * kUnitsPerRow + col;
    return x;
}

// Start the copies of a unit's 16 e4m3 rows (this lane's 8-byte column of
// each) into ring slot `buf` ([16 rows][16 columns] of 8 bytes).
__device__ __forceinline__ void import_issue(const ImportUnit& x, bool live, int half, int col, uint32_t buf) {
    constexpr int kUnitsPerRow = kHeadDim / 8;
    if (live) {
#pragma unroll
        for (int i = 0; i < kPageSlots / 2; ++i) {
            const int t = 2 * i + half;
            const bool ok = t < x.valid;
            cp_async8(buf + (t * kUnitsPerRow + col) * 8, ok ? (const void*)(x.src + (size_t)t * kUnitsPerRow)
                                                             : (const void*)x.src, ok);
        }
    }
    cp_async_commit();
}

__global__ void __launch_bounds__(256, 3) kv_import_fp8_kernel(const ImportParams a) {
    constexpr int kUnitsPerRow = kHeadDim / 8;  // 16-byte output units per 256-byte page row
    constexpr uint32_t kBufBytes = kPageSlots * kHeadDim;  // 2 KiB: one unit of e4m3 rows
    extern __shared__ __align__(16) uint8_t import_smem[];
    const int lane = threadIdx.x & 31;
    const int half = lane >> 4;
    const int col = lane & 15;
    const long long units = 2ll * a.n_blocks * a.n_kv_heads;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    long long u = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5);
    if (u >= units) return;
    const uint32_t ring = smem_addr(import_smem) + (threadIdx.x >> 5) * kRing * kBufBytes;
    const uint2* ring_p = reinterpret_cast<const uint2*>(import_smem + (threadIdx.x >> 5) * kRing * kBufBytes);

    ImportUnit info[kRing - 1];
#pragma unroll
    for (int k = 0; k < kRing - 1; ++k) {
        const long long uu = u + k * warps;
        info[k] = uu < units ? import_unit(a, uu, col) : ImportUnit{};
        import_issue(info[k], uu < units, half, col, ring + k * kBufBytes);
    }
    for (int it = 0; u < units; u += warps, ++it) {
        const ImportUnit cur = info[0];
        {
            const long long uu = u + (kRing - 1) * warps;
            const ImportUnit nx = uu < units ? import_unit(a, uu, col) : ImportUnit{};
            import_issue(nx, uu < units, half, col, ring + ((it + kRing - 1) % kRing) * kBufBytes);
#pragma unroll
            for (int k = 0; k < kRing - 2; ++k) info[k] = info[k + 1];
            info[kRing - 2] = nx;
        }
        cp_async_wait<kRing - 1>();
        const uint2* bp = ring_p + (it % kRing) * (kBufBytes / 8) + col;
        uint4* base = cur.which ? a.v_base : a.k_base;
#pragma unroll
        for (int i = 0; i < kPageSlots / 2; ++i) {
            const int t = 2 * i + half;
            if (t >= cur.valid) continue;
            const uint2 q = bp[t * kUnitsPerRow];
            const int pos = a.n_prior + cur.p0 + t;
            const int2 e = a.table[pos / kPageSlots];
            const int page = cur.which ? e.y : e.x;
            if (page < 0 || page >= a.pool_pages) {
                atomicOr(a.err, kErrBadPage);
                continue;
            }
            const uint32_t w[4] = {q.x & 0xFFFFu, q.x >> 16, q.y & 0xFFFFu, q.y >> 16};
            uint32_t o[4];
            // Fast path: with the scale at least 2^-117 (and finite) every
            // nonzero product is a normal fp32 and the hardware RNE pack equals
            // the reference's bf16 rounding; NaN codes (x111 1111) and other
            // scales take the reference rounding element by element.
            const bool nan_code = (__vcmpeq4(q.x & 0x7F7F7F7Fu, 0x7F7F7F7Fu) | __vcmpeq4(q.y & 0x7F7F7F7Fu, 0x7F7F7F7Fu)) != 0;
            if (cur.fast && !nan_code) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = e4m3x2_to_f32(w[j]);
                    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(o[j]) : "f"(__fmul_rn(f.y, cur.scale)),
                        "f"(__fmul_rn(f.x, cur.scale)));
                }
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = e4m3x2_to_f32(w[j]);
                    o[j] = (uint32_t)bf16_bits_ref(__fmul_rn(f.x, cur.scale)) |
                           ((uint32_t)bf16_bits_ref(__fmul_rn(f.y, cur.scale)) << 16);
                }
            }
            base[(((size_t)page * kPageSlots + pos % kPageSlots) * a.n_kv_heads + cur.h) * kUnitsPerRow + col] =
                make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
    cp_async_wait<0>();
}

// Persistent grid: at most the CTAs that are resident at once (resident
// CTAs per SM x SMs), so that every warp strides over several units and its
// prefetch of the next one overlaps the current one's work.
long long grid_for(long long work_items, int per_block, int num_sms, int per_sm) {
    long long b = (work_items + per_block - 1) / per_block;
    const long long cap = (long long)num_sms * per_sm;
    return b < 1 ? 1 : (b > cap ? cap : b);
}

}  // namespace

cudaError_t launch_export(const PoolView& pool, const int2* table, int32_t n_tokens, int32_t fp8, void* k_out,
                          void* v_out, float* k_scales, float* v_scales, uint32_t* err, int num_sms,
                          cudaStream_t stream) {
    ExportParams a;
    a.k_base = reinterpret_cast<const uint4*>(pool.k_base);
    a.v_base = reinterpret_cast<const uint4*>(pool.v_base);
    a.table = table;
    a.err = err;
    a.k_out = k_out;
    a.v_out = v_out;
    a.k_scales = k_scales;
    a.v_scales = v_scales;
    a.n_tokens = n_tokens;
    a.n_pages = (n_tokens + kPageSlots - 1) / kPageSlots;
    a.n_kv_heads = pool.n_kv_heads;
    a.pool_pages = pool.pool_pages;
    a.fp8 = fp8;
    const long long units = 2ll * a.n_pages * pool.n_kv_heads;
    if (!fp8) {
        kv_export_bf16_kernel<<<(unsigned)grid_for(units, 8, num_sms, 4), 256, 0, stream>>>(a);
        return cudaGetLastError();
    }
    constexpr int smem = 8 * kRing * kPageSlots * kHeadDim * 2;  // 8 warps x kRing x 4 KiB
    static std::atomic<uint64_t> configured{0};  // devices whose attribute is set
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 64 || !(configured.load() & (1ull << dev))) {
        e = cudaFuncSetAttribute(kv_export_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured.fetch_or(1ull << dev);
    }
    kv_export_kernel<<<(unsigned)grid_for(units, 8, num_sms, 2), 256, smem, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_import_fp8(const PoolView& pool, const int2* table, int32_t n_prior, int32_t seq_len,
                              const void* k_in, const void* v_in, const float* k_scales, const float* v_scales,
                              uint32_t* err, int num_sms, cudaStream_t stream) {
    ImportParams a;
    a.k_in = static_cast<const uint2*>(k_in);
    a.v_in = static_cast<const uint2*>(v_in);
    a.k_scales = k_scales;
    a.v_scales = v_scales;
    a.k_base = reinterpret_cast<uint4*>(pool.k_base);
    a.v_base = reinterpret_cast<uint4*>(pool.v_base);
    a.table = table;
    a.err = err;
    a.n_prior = n_prior;
    a.seq_len = seq_len;
    a.n_blocks = (seq_len + kPageSlots - 1) / kPageSlots;
    a.n_kv_heads = pool.n_kv_heads;
    a.pool_pages = pool.pool_pages;
    const long long units = 2ll * a.n_blocks * pool.n_kv_heads;
    constexpr int smem = 8 * kRing * kPageSlots * kHeadDim;  // 8 warps x kRing x 2 KiB
    kv_import_fp8_kernel<<<(unsigned)grid_for(units, 8, num_sms, 3), 256, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace gkv
