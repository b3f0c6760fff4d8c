// kernels.h — internal launch interface between the host runtime (host.cpp)
// and the CUDA kernels. Not part of the C ABI.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gkv {

constexpr int kPageSlots = 16;  // PAGE_BLOCK_SIZE (include/core/page_attention.h:9)
constexpr int kHeadDim = 128;   // the reference CUDA op's only head size (attention.cu:511)

// Table entries a launch publishes to the device block table. The kernels
// read entries [first, first + n) from here (not from the table, which they
// are writing) and one thread stores them into the table.
constexpr int kMaxNewPagesPerLaunch = 64;
struct NewPages {
    int32_t first;
    int32_t n;
    int2 ids[kMaxNewPagesPerLaunch];  // {k_id, v_id}
};

// Split-K partials capacity (q-head rows x splits) of one scratch area.
constexpr int kMaxPartialRows = 10240;

struct Scratch {
    float* part_acc;     // [kMaxPartialRows][128] un-normalised split outputs
    float2* part_ml;     // [kMaxPartialRows] (running max in log2 units, sum)
    uint32_t* err;       // device error word
    uint32_t* done = nullptr;  // completion word of the table's decode steps (see DecodeLaunch::post_done)
    uint32_t* merge = nullptr; // two zeroed counters of the fused split merge (see DecodeLaunch::fused_merge)
};

struct PoolView {
    uint16_t* k_base;
    uint16_t* v_base;
    int32_t pool_pages;
    int32_t n_kv_heads;
};


// QK-norm + RoPE parameters (qk_rope.cuh): device pointers and eps.
struct QkNorm {
    const float* q_w;  // [128] fp32 RMSNorm weights of Q heads
    const float* k_w;  // [128] of K heads
    const float* cos;  // [max_seq][128] fp32 RoPE table (both halves equal)
    const float* sin;
    float eps;
};

// Per-step state of one layer's decode launch, in device memory: a captured
// (CUDA-graph) decode step reads it instead of its launch parameters, which
// are frozen at capture. The step's first node copies the host's values in;
// the kernels only read it.
struct DeviceStep {
    int32_t n_prior;
    int32_t total;
    int32_t n_pages;
    int32_t pages_per_split;
    int32_t n_splits;
    int32_t new_first;
    int32_t new_n;       // 0 or 1
    int32_t pad;
    int2 new_id;
};

struct DecodeLaunch {
    const uint16_t* q;      // [Hq][128]
    const uint16_t* k_new;  // [Hkv][128] token appended by this step (or null)
    const uint16_t* v_new;
    void* out;              // [Hq][128]
    int32_t out_dtype;
    int32_t n_q_heads;
    int32_t n_prior;        // tokens cached before this step
    int32_t total;          // tokens attended (n_prior + 1 with an append)
    int32_t n_pages;        // logical pages covering `total`
    float scale;
    int32_t n_splits;       // 0 = choose
    const QkNorm* qk;       // non-null: q / k_new are pre-norm; QK-norm + RoPE fused (position n_prior)
    const DeviceStep* step = nullptr;  // non-null: n_prior / total / n_pages / split size / new page from here
    int32_t grid = 0;                  // with step: the fixed decode grid (>= every step's n_splits)
    bool next_is_other_layer = false;  // the next launch on the stream is a decode of a layer distinct
                                       // from this one and from every layer launched since the last
                                       // launch without this flag: the combine releases it at entry
    bool prev_is_other_layer = false;  // the previous launch is the combine of an earlier layer of the
                                       // same multi-layer step (launched with next_is_other_layer), and
                                       // Q / K / V were complete before the step's first launch
    // Completion word protocol (scratch.done must be set): the decode grid
    // waits until the word reaches done_seq - 1 (the table's previous decode
    // step completed) before it reads the table or any page, and the combine
    // stores done_seq once this step's decode grid has completed. The combine
    // then releases the next launch at entry. The caller numbers the steps of
    // a table 1, 2, 3, ... and only launches that post the word may be
    // numbered.
    bool post_done = false;
    uint32_t done_seq = 0;
    // Merge the splits inside the decode grid (the last CTAs to finish
    // merge; scratch.merge must be set) instead of a combine launch. Not
    // with a captured step or a multi-GPU gather.
    bool fused_merge = false;
};

// Split geometry of a decode step: pages per split and the number of splits
// (grid size), as launch_decode chooses them. Returns false when the context
// needs more partial rows than the scratch holds.
// Shared-memory size / carveout attributes of the decode kernels on the
// current device (once per device; launch_decode calls it too).
cudaError_t configure_decode_kernels();

bool decode_split_geometry(int32_t n_pages, int32_t n_kv_heads, int32_t n_q_heads, int32_t n_splits_hint,
                           int num_sms, int32_t* pages_per_split, int32_t* n_splits);

// Head all-gather fused into the split combine (multi-GPU KV-head sharding):
// every rank's combine stores its query-head block into every rank's full
// output buffer over NVLink peer memory (plain stores), then publishes the
// step's call count in each peer's flag slot and waits (bounded) until all
// peers' slots for this layer reach it.
constexpr int kMaxGatherRanks = 8;
struct GatherLaunch {
    int32_t world;                        // 0 = no gather
    int32_t rank;
    void* dst[kMaxGatherRanks];           // this rank's head block in rank r's full buffer
    int32_t n_flag_dst;                   // flag slots this rank publishes to (world, or 1)
    uint32_t* flag_dst[kMaxGatherRanks];  // this rank's flag slot (this layer): on every rank, or its own
    const uint32_t* flag_wait[kMaxGatherRanks];  // where rank r's flag for this layer is read
    uint32_t epoch;                       // call count of this layer, 1-based
    uint32_t* ticket;                     // CTA completion counter (zero between launches)
    uint64_t wait_ns;                     // limit of the wait for the peers' flags
};

// Fused decode step: append one token's K/V, GQA-grouped split-K
// flash-decoding over the block table (k_map/v_map: the pool's 128-byte
// swizzled maps), then the split combine. Returns the CUDA error.
// The decode kernel's tensor maps of a pool: per (page, head) boxes
// {64, 1, 16} and per page boxes {64, 16 slots, Hkv heads}, 128-byte swizzle.
struct DecodeMaps {
    CUtensorMap k_head, v_head;
    CUtensorMap k_page, v_page;
};
bool encode_decode_maps(const PoolView& pool, DecodeMaps* m, const char** why);

cudaError_t launch_decode(const PoolView& pool, const DecodeMaps& maps,
                          int2* table, const NewPages& np, const Scratch& scratch,
                          const DecodeLaunch& d, int num_sms, cudaStream_t stream,
                          const GatherLaunch* gather = nullptr);

// export.cu: pages <-> dense head-major [Hkv][tokens][128] (bf16, or e4m3
// with per (head, 16-token block) fp32 scales).
cudaError_t launch_export(const PoolView& pool, const int2* table, int32_t n_tokens, int32_t fp8, void* k_out,
                          void* v_out, float* k_scales, float* v_scales, uint32_t* err, int num_sms,
                          cudaStream_t stream);
cudaError_t launch_import_fp8(const PoolView& pool, const int2* table, int32_t n_prior, int32_t seq_len,
                              const void* k_in, const void* v_in, const float* k_scales, const float* v_scales,
                              uint32_t* err, int num_sms, cudaStream_t stream);

// Scatter tokens [p_begin, p_end) of K/V ([Hkv][src_len][128]) to positions
// n_prior + p, and publish np's entries to the table. With p_begin == p_end
// only the table entries are written. pdl: kAppendDependent launches it as a
// programmatic dependent of the previous kernel (it waits for that kernel
// before touching memory); kAppendTrigger lets the next kernel, which must be
// one that waits for it likewise (the chunked-prefill kernel), start its
// launch and setup while this one runs.
constexpr int kAppendDependent = 1, kAppendTrigger = 2;
cudaError_t launch_append(const PoolView& pool, int2* table, const NewPages& np,
                          const uint16_t* k, const uint16_t* v, int32_t n_prior,
                          int32_t src_len, int32_t p_begin, int32_t p_end, uint32_t* err,
                          cudaStream_t stream, int pdl = 0);

struct PrefillLaunch {
    const uint16_t* q;  // [Hq][S][128]
    void* out;          // [Hq][S][128]
    int32_t out_dtype;
    int32_t n_q_heads;
    int32_t seq_len;
    int32_t total;      // tokens cached including this chunk
    int32_t n_pages;
    float scale;
    int32_t causal;
    // Tensor-core prefill only: tensor maps {K, V} over the chunk's inputs
    // ([Hkv][S][128], box {64, 128, 1}). When given and the chunk starts on a
    // 128-token tile boundary, the chunk's own KV tiles are read from them
    // rather than from the pages, and the launch waits for the preceding
    // append only before it completes, so the two run side by side.
    const CUtensorMap* kv_new = nullptr;
};

// Per-head QK-norm + RoPE of Q and K and the head-major permute of Q, K and
// V, in one launch (qk_rope.cu): [S][H*128] in, [H][S][128] out.
cudaError_t launch_qk_norm_rope(const uint16_t* q, const uint16_t* k, const uint16_t* v, int32_t seq_len,
                                int32_t n_q_heads, int32_t n_kv_heads, const QkNorm& n, int32_t start_pos,
                                uint16_t* q_out, uint16_t* k_out, uint16_t* v_out, cudaStream_t stream);

// Record the message gkv_last_error() returns on this host thread.
void set_last_error(const char* msg);

// Tensor maps of the tensor-core prefill: the pool's K/V with 128-byte
// swizzle, box {64, 1, 16}; the chunk's Q [Hq][S][128], box {64, 128, 1}.
bool encode_pool_maps_sw128(const PoolView& pool, CUtensorMap* k_map, CUtensorMap* v_map,
                            const char** why);
// The same with box {64, 1, 128}: one copy covers a run of 8 pages whose ids
// are consecutive (the common case for a sequence appended in one go).
constexpr int kRunSlots = 128;
bool encode_pool_run_maps_sw128(const PoolView& pool, CUtensorMap* k_map, CUtensorMap* v_map,
                                const char** why);
struct PoolMaps {
    CUtensorMap k, v;          // one page per copy
    CUtensorMap k_run, v_run;  // 8 consecutive pages per copy
    bool runs;                 // k_run / v_run usable
};
bool encode_q_map_sw128(const uint16_t* q, int32_t n_q_heads, int32_t seq_len, CUtensorMap* q_map,
                        const char** why);

// Attention of a chunk of seq_len queries over the cached pages (the chunk's
// own K/V already appended), on the tensor cores.
cudaError_t launch_prefill_tc(const PoolView& pool, const CUtensorMap& q_map, const PoolMaps& maps,
                              const int2* table, const PrefillLaunch& p, uint32_t* err,
                              int num_sms, cudaStream_t stream);

// Non-paged attention (the reference's FlashAttentionImpl): B sequences of
// seq_len tokens, Q [B][Hq][S][128], K/V [B][Hkv][S][128] contiguous,
// self-attention (query s at position s), on the same tcgen05 kernel with the
// K/V tiles copied straight from the tensors.
struct FlashLaunch {
    void* out;          // [B][Hq][S][128]
    int32_t out_dtype;
    int32_t batch;
    int32_t n_q_heads;
    int32_t n_kv_heads;
    int32_t seq_len;
    float scale;
    int32_t causal;
};
// K/V tensor maps over [B*Hkv][S][128], box {64, 128, 1}, 128-byte swizzle.
bool encode_contig_kv_maps_sw128(const uint16_t* k, const uint16_t* v, int32_t rows_per_head, int32_t heads,
                                 CUtensorMap* k_map, CUtensorMap* v_map, const char** why);
cudaError_t launch_flash_tc(const CUtensorMap& q_map, const CUtensorMap& k_map, const CUtensorMap& v_map,
                            const FlashLaunch& f, uint32_t* err, int num_sms, cudaStream_t stream);

// The same on CUDA cores (one warp per query row); kept as an independent
// second implementation for cross-checking.
cudaError_t launch_prefill_simt(const PoolView& pool, const int2* table, const PrefillLaunch& p,
                                uint32_t* err, cudaStream_t stream);

}  // namespace gkv
