/*
 * genllm_kv.h — C ABI of the B200-native paged KV-cache path.
 *
 * Replaces the CUDA side of Genllm's paged-attention path (paths relative to
 * the Genllm source tree):
 *   - BlockPool / PagedAttentionManager   include/core/page_attention.h:11-89,
 *                                         src/core/page_attention.cpp:25-216
 *   - PagedAttentionImpl<Device::CUDA>    include/backend/cuda/attention.h:16-18,
 *                                         src/backend/cuda/attention.cu:491-580
 *   - kernel::paged_attention             include/core/kernels.h:32
 *
 * Two tiers:
 *   1. the managed tier (gkv_manager_*, gkv_*_layer, gkv_paged_attention ...)
 *      mirrors PagedAttentionManager: it owns the per-layer LIFO page
 *      allocators, the host copy of each block table and a device-resident
 *      copy of it, and launches the kernels;
 *   2. the raw tier (gkv_table_*, gkv_*_raw) runs the kernels over pools and
 *      page allocation that the CALLER manages (e.g. the reference's own
 *      BlockPool, when this library is dropped in under the unchanged
 *      scheduler). The managed tier is built on the raw tier.
 *
 * Conventions: every function returns a gkv_status (0 = success); work is
 * enqueued on the given cudaStream_t (0 = legacy default stream) and nothing
 * synchronises unless documented. No function takes or returns torch types.
 * Calls on one manager (or one gkv_table) must be ordered on one stream:
 * they share split-K scratch and the device block table.
 *
 * Shapes follow the reference operator (include/model/op_factory.hpp:413-476):
 * Q [1][Hq][S][D], K and V [1][Hkv][S][D], out [1][Hq][S][D], all contiguous;
 * D = 128 (the reference CUDA op's requirement, attention.cu:511); page layout
 * [16 slots][Hkv][D] (src/core/page_attention.cpp:128-129).
 */
#ifndef GENLLM_KV_H
#define GENLLM_KV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without including the CUDA headers. */
typedef struct CUstream_st* gkv_stream_t;

#define GKV_PAGE_SLOTS 16 /* PAGE_BLOCK_SIZE, include/core/page_attention.h:9 */

typedef enum gkv_status {
    GKV_OK = 0,
    GKV_ERR_INVALID = 1,     /* bad argument, unknown layer, shape mismatch */
    GKV_ERR_NO_PAGES = 2,    /* a page pool is exhausted (the reference silently
                                corrupts its table here, page_attention.cpp:155,161) */
    GKV_ERR_CUDA = 3,        /* a CUDA runtime call failed; see gkv_last_error() */
    GKV_ERR_UNSUPPORTED = 4, /* dtype / head_dim / batch / group size not built */
    GKV_ERR_STATE = 5,       /* layer not initialised or not reserved */
    GKV_ERR_DEVICE = 6       /* a kernel flagged an error (bad page id, wait timeout) */
} gkv_status;

/* Element types use the reference's DataType codes (include/utils/utils.hpp). */
typedef enum gkv_dtype { GKV_F32 = 0, GKV_F16 = 1, GKV_BF16 = 30 } gkv_dtype;

/* Status text, and the message of the last failure on this host thread. */
const char* gkv_status_string(int status);
const char* gkv_last_error(void);

/* ======================= managed tier ==================================== */

typedef struct gkv_manager gkv_manager;

/* PagedAttentionManager(MemoryPool*) (page_attention.cpp:66-70) for CUDA
 * device `device`. device = -1 makes a host-only manager: page bookkeeping
 * (init/reserve/append_kv_pages/alloc/free/reset/tables) with no device memory
 * and no CUDA calls, like the reference's pool-less manager used by its
 * allocator tests (tests/test_page_attention.cpp:49-85); launches on it
 * return GKV_ERR_STATE. Before reserve_layer a layer's pools are unbounded,
 * as the reference's default BlockPool. */
int gkv_manager_create(int device, gkv_manager** out);
int gkv_manager_destroy(gkv_manager* m);

/* init_layer (page_attention.cpp:72-79): mark the layer active with its KV
 * geometry; resets its cached-token count. */
int gkv_init_layer(gkv_manager* m, int32_t layer_id, int32_t n_kv_heads, int32_t head_dim,
                   int32_t dtype);

/* reserve_layer (page_attention.cpp:81-101): give the layer a K and a V region
 * of max_blocks pages each. With k_region/v_region NULL the library allocates
 * them (cudaMalloc, freed by gkv_manager_destroy); otherwise they are caller
 * memory (e.g. carved from the reference's kv_cache MemoryPool), at least
 * 16-byte aligned and max_blocks * 16 * Hkv * D * elem bytes long. Also
 * allocates the layer's device block table. */
int gkv_reserve_layer(gkv_manager* m, int32_t layer_id, int32_t max_blocks, void* k_region,
                      void* v_region);

/* is_active (page_attention.h:82-85): 1 active, 0 not. */
int gkv_is_active(const gkv_manager* m, int32_t layer_id);

/* append_kv_pages (page_attention.cpp:141-162): grow the table for `count`
 * more tokens and advance num_cached, host bookkeeping only. Unlike the
 * reference, when a pool cannot supply every page this returns
 * GKV_ERR_NO_PAGES and changes nothing. The new table entries reach the
 * device with the next append/attention launch on this layer. */
int gkv_append_kv_pages(gkv_manager* m, int32_t layer_id, int32_t count);

/* append_kv_from_tensor (page_attention.cpp:104-139): allocate pages, then
 * scatter K and V ([Hkv][seq_len][D] device pointers) into them with one
 * kernel. Bit-exact byte copy. */
int gkv_append_kv(gkv_manager* m, int32_t layer_id, const void* K, const void* V,
                  int32_t n_kv_heads, int32_t seq_len, int32_t head_dim, int32_t dtype,
                  gkv_stream_t stream);

/* PagedAttentionImpl<CUDA>::execute (attention.cu:491-580) / the CPU op
 * (src/backend/cpu/attention.cpp:123-216): append this step's K/V, then attend
 * Q over every cached token, causally when `causal` (query sq sits at absolute
 * position num_cached - seq_len + sq). seq_len == 1 runs the fused split-K
 * decode kernel (append + attention + split combine); seq_len > 1 runs the
 * append kernel and the chunked-prefill kernel. Device pointers. `out_dtype`
 * may differ from the K/V dtype (F32 output gives the pre-rounding values).
 * n_kv_groups = Hq / Hkv (op_params[3]). batch must be 1 (the reference
 * shares one cache across the batch; README.md:150 states batch 1). */
int gkv_paged_attention(gkv_manager* m, int32_t layer_id, const void* Q, const void* K,
                        const void* V, void* out, int32_t batch, int32_t n_q_heads,
                        int32_t seq_len, int32_t head_dim, int32_t n_kv_heads, float scale,
                        int32_t causal, int32_t n_kv_groups, int32_t dtype, int32_t out_dtype,
                        gkv_stream_t stream);

/* One decode token through n_layers layers in one call: gkv_paged_attention
 * (seq_len 1, causal, batch 1) on layer_ids[i] with Q[i], K[i], V[i], out[i]
 * (device pointers, arrays of n_layers), in order on one stream. The layers
 * are independent here (the host drives the layer-to-layer data flow), so
 * this is a launch loop in the library: one host call per step instead of one
 * per layer, the executor's per-op host cost gone (the reference executor
 * synchronises the device after every op, src/core/executor.cpp:169-172).
 * Every layer's Q, K and V must be complete when the call's first launch
 * runs (produced by earlier work on the stream), and no layer's out may be
 * another listed layer's Q, K or V: with distinct layers the kernels of
 * layer i + 1 start while layer i finishes and read their inputs without
 * waiting for it. Stops at the first failing layer (layers before it have
 * advanced). */
int gkv_decode_layers(gkv_manager* m, int32_t n_layers, const int32_t* layer_ids, const void* const* Q,
                      const void* const* K, const void* const* V, void* const* out, int32_t n_q_heads,
                      float scale, int32_t out_dtype, gkv_stream_t stream);

/* reset (page_attention.cpp:209-216) for every layer, or one layer. Host
 * bookkeeping only: num_cached = 0, empty table, every page handed out so far
 * back on the free list in ascending order. */
int gkv_reset(gkv_manager* m);
int gkv_reset_layer(gkv_manager* m, int32_t layer_id);

typedef struct gkv_layer_info {
    int32_t active;
    int32_t num_cached;
    int32_t n_pages;     /* logical pages in the table */
    int32_t max_blocks;  /* pages per pool */
    int32_t n_kv_heads;
    int32_t head_dim;
    int32_t dtype;
    int32_t reserved;
    void* k_base;        /* device address of page 0 of the K pool */
    void* v_base;
    const int32_t* device_table; /* [max_blocks][2] {k_id, v_id}, valid for n_pages
                                    entries once the launches that wrote them ran */
} gkv_layer_info;

/* get_layer (page_attention.cpp:205-207), as a snapshot. */
int gkv_get_layer_info(const gkv_manager* m, int32_t layer_id, gkv_layer_info* info);

/* Copy the host block table (PageEntry list) into k_ids/v_ids (cap entries);
 * *n_pages receives the full length. */
int gkv_get_page_table(const gkv_manager* m, int32_t layer_id, int32_t* k_ids, int32_t* v_ids,
                       int32_t cap, int32_t* n_pages);

/* Synchronise the device and copy the DEVICE block table's first n_pages
 * entries (those the launches so far have published) into k_ids/v_ids. A
 * debugging and test aid: it must equal gkv_get_page_table after any
 * append/attention launch. */
int gkv_read_device_table(gkv_manager* m, int32_t layer_id, int32_t* k_ids, int32_t* v_ids,
                          int32_t cap, int32_t* n_published);

/* Replace the layer's table and num_cached (e.g. to restore a saved cache or
 * to build a fragmented one in tests). Every id must already be handed out by
 * the pool (gkv_page_alloc). Uploads the table on `stream`. */
int gkv_set_page_table(gkv_manager* m, int32_t layer_id, const int32_t* k_ids,
                       const int32_t* v_ids, int32_t n_pages, int32_t num_cached,
                       gkv_stream_t stream);

/* BlockPool::alloc / free / reset / num_blocks / num_free
 * (page_attention.cpp:25-64) on the layer's K (which = 0) or V (which = 1)
 * pool. alloc: most recently freed id first (LIFO), else the next never-used
 * id; GKV_ERR_NO_PAGES at capacity (the reference returns -1, which *id also
 * receives). free: ids never handed out are ignored, like the reference;
 * freeing an id twice is rejected (GKV_ERR_INVALID), which the reference does
 * not check. */
int gkv_page_alloc(gkv_manager* m, int32_t layer_id, int32_t which, int32_t* id);
int gkv_page_free(gkv_manager* m, int32_t layer_id, int32_t which, int32_t id);
int gkv_pool_reset(gkv_manager* m, int32_t layer_id, int32_t which);
int gkv_pool_stats(const gkv_manager* m, int32_t layer_id, int32_t which, int32_t* num_blocks,
                   int32_t* num_free, int32_t* capacity);

/* Read and clear the device error word of a layer (synchronises the layer's
 * last stream): bit 0 = a page id outside the pool was skipped, bit 1 = a
 * wait on an asynchronous copy timed out. *flags = 0 when clean. */
int gkv_check_device_errors(gkv_manager* m, int32_t layer_id, uint32_t* flags);

/* ======================= raw tier ======================================== */

/* Device-resident block table of one layer plus its kernel scratch (split-K
 * partials, per-head completion counters, error word). */
typedef struct gkv_table gkv_table;

int gkv_table_create(int device, int32_t capacity, gkv_table** out);
int gkv_table_destroy(gkv_table* t);
const int32_t* gkv_table_device_ptr(const gkv_table* t);
/* Synchronise the table's device, read and clear its device error word (the
 * bits of gkv_check_device_errors). */
int gkv_table_check_errors(gkv_table* t, uint32_t* flags);

/* A KV pool pair in the reference's page layout, managed by the caller. */
typedef struct gkv_pool_desc {
    void* k_base;
    void* v_base;
    int32_t pool_pages; /* pages addressable from each base (bounds for ids) */
    int32_t n_kv_heads;
    int32_t head_dim;
    int32_t dtype;
} gkv_pool_desc;

/* The table delta of one step: logical pages [first_new_page, first_new_page +
 * n_new_pages) were just allocated by the caller with these ids. The kernels
 * write them into the device table; older entries must already be there. */
typedef struct gkv_new_pages {
    int32_t first_new_page;
    int32_t n_new_pages;
    const int32_t* k_ids; /* host arrays, n_new_pages entries */
    const int32_t* v_ids;
} gkv_new_pages;

/* Scatter seq_len tokens of K/V (device [Hkv][seq_len][D]) into positions
 * [n_prior, n_prior + seq_len) of the table. */
int gkv_append_kv_raw(const gkv_pool_desc* pool, gkv_table* t, int32_t n_prior,
                      const gkv_new_pages* np, const void* K, const void* V, int32_t seq_len,
                      gkv_stream_t stream);

/* Append, then attend; n_prior tokens were cached before the call. */
int gkv_paged_attention_raw(const gkv_pool_desc* pool, gkv_table* t, int32_t n_prior,
                            const gkv_new_pages* np, const void* Q, const void* K, const void* V,
                            void* out, int32_t n_q_heads, int32_t seq_len, float scale,
                            int32_t causal, int32_t out_dtype, gkv_stream_t stream);

/* ======================= multi-GPU head all-gather ======================== */

/* KV-head sharding across the GPUs of one node (the reference has no
 * multi-GPU attention; its layers move between devices through host copies,
 * src/backend/cuda/memcpy.cu:29-44). Each rank's manager holds Hkv / N heads;
 * after a decode step every rank needs all N head blocks of the output. This
 * tier writes them there from inside the split-combine kernel over NVLink
 * (plain peer stores into memory opened with CUDA IPC), instead of a
 * separate all-gather launch.
 *
 * Device buffers to share between processes come from gkv_device_alloc
 * (zero-filled cudaMalloc); gkv_ipc_export / gkv_ipc_open / gkv_ipc_close
 * move them across processes (64-byte handles, exchanged by the caller). */
int gkv_device_alloc(int device, size_t bytes, void** ptr);
int gkv_device_free(int device, void* ptr);
int gkv_ipc_export(int device, const void* dev_ptr, void* handle /* 64 bytes */);
int gkv_ipc_open(int device, const void* handle, void** dev_ptr);
int gkv_ipc_close(int device, void* dev_ptr);

typedef struct gkv_gather gkv_gather;

/* out_bases[r]: rank r's full-output region as mapped in this process (its
 * own region for r == rank); flag_bases[r]: rank r's flag array of
 * max_layers * world uint32, zero-filled, mapped likewise. */
int gkv_gather_create(int device, int world, int rank, int max_layers, void* const* out_bases,
                      uint32_t* const* flag_bases, gkv_gather** out);
int gkv_gather_destroy(gkv_gather* g);

/* The same all-gather over NCCL, for hosts that shard without the IPC tier
 * (the reference has no multi-GPU attention; its devices exchange layer
 * outputs through host copies, src/backend/cuda/memcpy.cu:29-44). After each
 * rank's decode step of its Hkv / N heads (gkv_paged_attention with
 * n_q_heads = Hq / N), gkv_allgather_heads gathers the ranks' output blocks
 * [Hq / N][128] (bytes_per_rank each) into full, rank-major, on `stream`.
 * NCCL is loaded at run time (libnccl.so.2, or $GKV_NCCL_LIB); a
 * communicator passed in must come from that same library (or from
 * gkv_nccl_comm_create). Without NCCL these return GKV_ERR_UNSUPPORTED. */
int gkv_nccl_unique_id(void* id /* 128 bytes, rank 0 creates it and sends it to the others */);
int gkv_nccl_comm_create(int device, int world, int rank, const void* id, void** comm);
int gkv_nccl_comm_destroy(void* comm);
int gkv_allgather_heads(void* comm, const void* local, void* full, size_t bytes_per_rank, gkv_stream_t stream);

/* The limit of the wait for the peers' blocks (default 1 s; 1 us to 10 s).
 * When it runs out the combine stops waiting, sets bit 1 of the device
 * error word (gkv_check_device_errors) and finishes, so the stream stays
 * usable; the output then lacks the missing peers' blocks. */
int gkv_gather_set_wait_limit(gkv_gather* g, uint64_t limit_ns);

/* One decode step of this rank's heads (as gkv_paged_attention with
 * seq_len 1, causal), whose [n_q_heads][128] output block lands in EVERY
 * rank's region at out_offset + rank * n_q_heads * 128 * elem bytes. The
 * launch completes only once all ranks' blocks for this layer and step have
 * arrived in this rank's region (a bounded wait, gkv_gather_set_wait_limit;
 * on timeout the device error word gets bit 1). Every rank must make the same
 * sequence of calls. A layer's blocks stay in place until that layer's next
 * call on any rank: a peer's next call for the layer stores over them as
 * soon as that peer gets there, so read the region (stream-ordered) before
 * this rank's next call for the same layer. With two or more layers called
 * in turn every rank waits for the others at each layer, which keeps peers
 * from running a whole step ahead; with a single layer, copy the output out
 * before the next call. */
int gkv_paged_attention_gather(gkv_manager* m, int32_t layer_id, const void* Q, const void* K,
                               const void* V, gkv_gather* g, size_t out_offset, int32_t n_q_heads,
                               float scale, int32_t out_dtype, gkv_stream_t stream);

/* ======================= no-allocation decode ============================ */

/* No counterpart in the reference. One fused decode step (append the token
 * at position n_prior into its page, then attend Q over all n_prior + 1
 * tokens) for callers that may not allocate device memory — for example code
 * running under a host framework that owns every device allocation through
 * its own arena, or a latency-critical loop that cannot afford cudaMalloc's
 * cost or implicit synchronisation. Nothing is allocated: the split-K scratch
 * is a fixed 2 MiB + 32 KiB array inside the library that every GPU loading
 * it keeps until the process exits.
 *   device_table: [n_pages][2] {k_id, v_id} int32 in device memory, holding
 *   every page up to and including the one that receives the new token.
 *   Q [Hq][128], K and V [Hkv][128] (this step's token), out [Hq][128].
 * Limits: head_dim 128, bf16 pages, 1-8 kv heads, group size 1/2/4/8; the
 * fixed scratch holds 4096 partial rows (splits x Hq), so larger
 * Hq gets fewer splits; context <= 1000 pages per split; larger requests return GKV_ERR_INVALID / GKV_ERR_UNSUPPORTED.
 * The first call on a device looks up the scratch address on the current
 * device; make that first call before any stream capture. All calls share
 * the one scratch array (it keeps the previous call's contents), so calls
 * that overlap on the GPU — other streams, other threads — race; order them.
 * The device error word is cleared at the start of each call; read it with
 * gkv_paged_decode_static_scratch_errors. */
int gkv_paged_decode_static_scratch(const gkv_pool_desc* pool, const int32_t* device_table,
                                    int32_t n_prior, const void* Q, const void* K, const void* V,
                                    void* out, int32_t n_q_heads, float scale, int32_t out_dtype,
                                    gkv_stream_t stream);

/* No counterpart in the reference. The device error word of the last
 * gkv_paged_decode_static_scratch call on the current device, after the
 * stream's work has finished (this call synchronises `stream`): bit 0 = a
 * page id in device_table outside [0, pool_pages) (that page was skipped, so
 * the output is wrong), bit 1 = a bounded wait ran out. Allocates nothing;
 * the word stays as it is until the next decode call clears it. */
int gkv_paged_decode_static_scratch_errors(uint32_t* flags, gkv_stream_t stream);

/* ---------------- QK-norm + RoPE (the step feeding the append) -------------
 * Qwen3's attention block turns the Q/K/V projections [S][H*128] into the
 * post-QK-norm, post-RoPE Q and K the paged-attention op appends and attends
 * (src/model/Qwen3.cpp:136-154: reshape_permute x3, rms_norm x2 with the
 * per-head weights attn_q_norm / attn_k_norm, apply_rope x2). These entry
 * points fuse that step: standalone (one launch instead of seven), or inside
 * the attention call itself (decode: no launch of its own). Results are
 * bit-exact with the reference CPU ops (RmsNormImpl / ApplyRopeImpl<CPU>,
 * src/backend/cpu/normalization.cpp, src/backend/cpu/rope.cpp). head_dim 128. */
typedef struct gkv_qk_norm {
    const float* q_norm_w; /* device, [128] fp32 (blk.N.attn_q_norm.weight) */
    const float* k_norm_w; /* device, [128] fp32 (blk.N.attn_k_norm.weight) */
    const float* cos_tab;  /* device, [max_seq][128] fp32, from gkv_rope_cache */
    const float* sin_tab;
    int32_t max_seq;       /* rows of the tables; positions must stay below */
    float eps;             /* rms_norm_eps */
} gkv_qk_norm;

/* Host: the RoPE cos/sin tables [max_seq][head_dim] fp32 into host arrays, as
 * RopeCacheImpl<CPU>::execute (src/backend/cpu/rope.cpp:112-140) fills them
 * (double-precision angles; both halves of a row equal). */
int gkv_rope_cache(float theta, int32_t head_dim, int32_t max_seq, float* cos_out, float* sin_out);

/* Device: q_flat [S][Hq*128], k_flat / v_flat [S][Hkv*128] bf16 ->
 * q_out [Hq][S][128] (norm + RoPE), k_out [Hkv][S][128] (norm + RoPE),
 * v_out [Hkv][S][128] (permute only); token s sits at position start_pos + s.
 * Replaces ApplyRopeImpl<CUDA>::execute (src/backend/cuda/rope.cu:52-111),
 * RmsNormImpl<CUDA>::execute (src/backend/cuda/normalization.cu:49-90) on
 * the heads and PermuteImpl<CUDA>::execute (src/backend/cuda/shape.cu:45) x3.
 * All six buffers 16-byte aligned; Hq + Hkv <= 96. Allocates nothing. */
int gkv_qk_norm_rope(const void* q_flat, const void* k_flat, const void* v_flat, int32_t seq_len,
                     int32_t n_q_heads, int32_t n_kv_heads, const gkv_qk_norm* qk, int32_t start_pos,
                     void* q_out, void* k_out, void* v_out, gkv_stream_t stream);

/* gkv_paged_attention_raw on the projections: Q, K, V as q_flat / k_flat /
 * v_flat above, QK-norm + RoPE applied at positions n_prior + s. seq_len 1
 * fuses it into the decode kernel; longer chunks run gkv_qk_norm_rope into a
 * buffer the table owns (grown on demand), then the chunked-prefill path. */
int gkv_paged_attention_raw_qknorm(const gkv_pool_desc* pool, gkv_table* t, int32_t n_prior,
                                   const gkv_new_pages* np, const void* q_flat, const void* k_flat,
                                   const void* v_flat, void* out, int32_t n_q_heads, int32_t seq_len,
                                   float scale, int32_t causal, int32_t out_dtype, const gkv_qk_norm* qk,
                                   gkv_stream_t stream);

/* The managed tier's gkv_paged_attention on the projections (positions =
 * the layer's cached token count), batch 1, head_dim 128. */
int gkv_paged_attention_qknorm(gkv_manager* m, int32_t layer_id, const void* q_flat, const void* k_flat,
                               const void* v_flat, void* out, int32_t n_q_heads, int32_t seq_len, float scale,
                               int32_t causal, int32_t out_dtype, const gkv_qk_norm* qk, gkv_stream_t stream);

/* gkv_decode_layers' decode step captured once as a CUDA graph and replayed per
 * token: one graph launch per step instead of two kernel launches per layer.
 * The layers' Q/K/V/out pointers (and, if qk is non-NULL, each layer's
 * QK-norm + RoPE parameters: Q/K are then the projections, as
 * gkv_paged_attention_qknorm takes them) are bound at creation. Each
 * gkv_decode_graph_step allocates the step's pages on the host as
 * gkv_decode_layers does, writes every layer's step state (cached length,
 * page count, split geometry, new page id) into a pinned block, and launches
 * the graph, whose first node copies that block to the device; the kernels
 * read it there instead of their frozen launch parameters. Results are
 * identical to gkv_decode_layers (same kernels, same split geometry), with
 * the same requirement on the inputs (complete before the step, no layer's
 * out feeding another layer of the step). The
 * decode grid is fixed at one CTA per SM, which bounds the context a step
 * can serve (GKV_ERR_UNSUPPORTED beyond it; 147 splits of up to 1000 pages).
 * A step waits on the host only for the step launched two steps earlier to
 * finish (the pinned blocks alternate). Not for the multi-GPU gather tier.
 * The step's layers must not be driven by other calls while the graph is in
 * use, except between steps on the same stream. */
typedef struct gkv_decode_graph gkv_decode_graph;
int gkv_decode_graph_create(gkv_manager* m, int32_t n_layers, const int32_t* layer_ids, const void* const* Q,
                            const void* const* K, const void* const* V, void* const* out, int32_t n_q_heads,
                            float scale, int32_t out_dtype, const gkv_qk_norm* const* qk,
                            gkv_decode_graph** graph);
int gkv_decode_graph_step(gkv_decode_graph* graph, gkv_stream_t stream);
int gkv_decode_graph_destroy(gkv_decode_graph* graph);

/* ---------------- non-paged attention ------------------------------------
 * FlashAttentionImpl<CUDA>::execute (src/backend/cuda/attention.cu:317-399;
 * semantics of the CPU op, src/backend/cpu/attention.cpp:39-120):
 * self-attention of `batch` sequences of seq_len tokens each, Q
 * [B][Hq][S][D], K/V [B][Hkv][S][D] contiguous device tensors, query s at
 * position s (causal: keys 0..s), GQA group Hq / Hkv, out [B][Hq][S][D] in
 * out_dtype. Runs on the tcgen05 chunked-prefill kernel with its K/V tiles
 * copied straight from the tensors. head_dim 128, bf16. Allocates nothing;
 * timeouts set the current device's error word, read (and cleared) by
 * gkv_flash_check_errors (GKV_ERR_DEVICE when set). */
int gkv_flash_attention(const void* Q, const void* K, const void* V, void* out, int32_t batch, int32_t n_q_heads,
                        int32_t n_kv_heads, int32_t seq_len, int32_t head_dim, float scale, int32_t causal,
                        int32_t dtype, int32_t out_dtype, gkv_stream_t stream);
int gkv_flash_check_errors(uint32_t* flags);

/* ---------------- KV format export / import -------------------------------
 * The reference keeps a layer's cache only in its page layout
 * (src/core/page_attention.cpp:128) and cannot read it back. These entry
 * points move a layer's first n_tokens tokens between the pages and a dense
 * head-major copy [Hkv][n_tokens][128] (the layout append_kv_from_tensor
 * takes, src/core/page_attention.cpp:104-139), in one of two formats:
 *   GKV_KV_BF16: the pool's own bf16 bytes; export then append is the identity.
 *   GKV_KV_FP8_E4M3: one byte per element plus one fp32 scale per (head,
 *     16-token block), scales [Hkv][ceil(n_tokens / 16)]:
 *       amax  = max |x| over the block's finite elements
 *       scale = amax / 448, inv = 448 / amax (both 1 when 448 / amax is
 *               not finite: amax 0, or below ~2^-119)
 *       byte  = e4m3(x * inv): round to nearest even, finite overflow and
 *               infinities saturate at +-448, NaN -> 0x7F
 *     import: x' = bf16(e4m3_value(byte) * scale), bf16 rounded as the
 *     reference rounds (include/utils/bfloat16.hpp:18-45).
 * Device buffers, 16-byte aligned; stream-ordered, nothing synchronises. */
typedef enum gkv_kv_format { GKV_KV_BF16 = 0, GKV_KV_FP8_E4M3 = 1 } gkv_kv_format;

/* Raw tier: tokens [0, n_tokens) of the table's pages. k_scales / v_scales
 * are used (and required) for GKV_KV_FP8_E4M3 only. */
int gkv_export_kv_raw(const gkv_pool_desc* pool, gkv_table* t, int32_t n_tokens, int32_t format, void* K_out,
                      void* V_out, float* k_scales, float* v_scales, gkv_stream_t stream);
/* Raw tier: the inverse, seq_len tokens into positions [n_prior, n_prior +
 * seq_len), table delta as gkv_append_kv_raw. Scales are indexed by 16-token
 * blocks of the INPUT ([Hkv][ceil(seq_len / 16)]). GKV_KV_BF16 is
 * gkv_append_kv_raw. */
int gkv_import_kv_raw(const gkv_pool_desc* pool, gkv_table* t, int32_t n_prior, const gkv_new_pages* np,
                      int32_t format, const void* K_in, const void* V_in, const float* k_scales,
                      const float* v_scales, int32_t seq_len, gkv_stream_t stream);
/* Managed tier: export the layer's cached tokens (*n_tokens receives the
 * count; the buffers must hold it, see gkv_get_layer_info), or append
 * seq_len imported tokens to the layer (pages allocated as gkv_append_kv). */
int gkv_export_kv(gkv_manager* m, int32_t layer_id, int32_t format, void* K_out, void* V_out, float* k_scales,
                  float* v_scales, int32_t* n_tokens, gkv_stream_t stream);
int gkv_import_kv(gkv_manager* m, int32_t layer_id, int32_t format, const void* K_in, const void* V_in,
                  const float* k_scales, const float* v_scales, int32_t seq_len, gkv_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif
