// paged_attention_cuda.cpp — drop-in ops::PagedAttentionImpl<Device::CUDA>
// for the Genllm engine, on libgenllm_kv.so (include/genllm_kv.h).
//
// Replaces the definition in src/backend/cuda/attention.cu:491-580; the
// declaration (include/backend/cuda/attention.h:16-18), kernel::paged_attention
// (include/core/kernels.h:32), the executor (src/core/executor.cpp:502) and
// the scheduler's KV set-up (src/core/scheduler.cpp:404-430) stay unchanged.
//
// Host bookkeeping stays the reference's: pages are allocated by its own
// BlockPool (LIFO) through PagedAttentionManager::append_kv_pages, and the
// pools are the regions reserve_layer carved from the kv_cache MemoryPool.
// What changes is the device side, through the raw tier of the C ABI:
//   * the block table is mirrored on the device per (manager, layer) and
//     only the entries added since the last call travel (in the kernel
//     launch parameters) — no cudaMalloc / H2D / cudaFree per call;
//   * append + attention run as one fused decode launch (+ the split
//     combine) for seq_len == 1, or append + tensor-core prefill otherwise,
//     instead of 2*Hkv*S synchronous cudaMemcpy calls and a serial kernel.
// An exhausted pool throws before any page is taken, instead of leaving
// num_cached ahead of the table and popped ids unreachable
// (src/core/page_attention.cpp:152-161).
#include <algorithm>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "backend/cuda/attention.h"
#include "core/manager.h"
#include "core/page_attention.h"
#include "genllm_kv.h"

namespace {

struct DeviceMirror {
    gkv_table* table = nullptr;
    int32_t capacity = 0;
    int32_t published = 0;    // entries of the reference page_table already on the device
    int32_t last_cached = 0;  // num_cached after the previous call (a drop means reset)
};

std::mutex g_mu;
std::map<std::pair<const PagedAttentionManager*, int32_t>, DeviceMirror> g_mirrors;

// BlockPool keeps its capacity (the max_blocks reserve_layer carved) private
// (include/core/page_attention.h:15). Explicit instantiation of a template
// on a member pointer is exempt from access checking, which lets this file
// read it without touching the reference's header; a public
// `int32_t capacity() const` on BlockPool would replace these lines.
struct CapacityTag {
    using type = int32_t BlockPool::*;
    friend type member(CapacityTag);
};
template <typename Tag, typename Tag::type M>
struct Expose {
    friend typename Tag::type member(Tag) { return M; }
};
template struct Expose<CapacityTag, &BlockPool::block_capacity_>;

int32_t capacity(const BlockPool& p) { return p.*member(CapacityTag{}); }

// Pages BlockPool::alloc can still hand out: its free list, then fresh ids
// up to the capacity (src/core/page_attention.cpp:38-47).
int32_t available(const BlockPool& p) { return p.num_free() + (capacity(p) - p.num_blocks()); }

// New pages append_kv_pages takes for `count` tokens after `cached`: one per
// position that starts a page (src/core/page_attention.cpp:146-157).
int32_t pages_needed(int32_t cached, int32_t count) {
    const int32_t first = (cached + PAGE_BLOCK_SIZE - 1) / PAGE_BLOCK_SIZE;
    const int32_t last = (cached + count + PAGE_BLOCK_SIZE - 1) / PAGE_BLOCK_SIZE;
    return last - first;
}

int32_t to_gkv_dtype(DataType d) {
    switch (d) {
        case DataType::GGML_TYPE_F32: return GKV_F32;
        case DataType::GGML_TYPE_F16: return GKV_F16;
        case DataType::GGML_TYPE_BF16: return GKV_BF16;
        default: throw std::runtime_error("paged_attention: unsupported dtype");
    }
}

[[noreturn]] void raise(const char* what) {
    throw std::runtime_error(std::string("paged_attention: ") + what + ": " + gkv_last_error());
}

}  // namespace

namespace ops {

void PagedAttentionImpl<Device::CUDA>::execute(Tensor* out, int32_t dev_id) {
    auto* mgr = g_mem_manager->get_attention_manager(out->device, dev_id);
    const int32_t layer_id = out->layer_id;
    if (!mgr || !mgr->is_active(layer_id)) return;  // as the reference (attention.cu:494)

    Tensor* Q = out->src[0];
    Tensor* K = out->src[1];
    Tensor* V = out->src[2];
    const int32_t batch = static_cast<int32_t>(Q->dims[0]);
    const int32_t n_q_heads = static_cast<int32_t>(Q->dims[1]);
    const int32_t seq_len = static_cast<int32_t>(Q->dims[2]);
    const int32_t head_dim = static_cast<int32_t>(Q->dims[3]);
    const int32_t n_kv_heads = static_cast<int32_t>(K->dims[1]);
    const float scale = out->op_params[1];
    const bool causal = static_cast<int32_t>(out->op_params[2]) != 0;
    if (head_dim != 128) throw std::runtime_error("paged_attention requires head_dim == 128");
    if (batch != 1) throw std::runtime_error("paged_attention: the paged cache holds one sequence (batch 1)");
    if (seq_len <= 0) return;

    auto& layer = mgr->get_layer(layer_id);
    const int32_t prev_cached = layer.num_cached;

    // Host allocation by the reference's own allocator, checked first: if
    // either pool cannot supply every page the chunk opens, nothing is
    // allocated and the cache is left as it was.
    const int32_t need = pages_needed(prev_cached, seq_len);
    if (available(layer.k_pool) < need || available(layer.v_pool) < need)
        throw std::runtime_error("paged_attention: KV page pool exhausted");
    const size_t prev_pages = layer.page_table.size();
    mgr->append_kv_pages(layer_id, seq_len);
    const int32_t n_pages = static_cast<int32_t>(layer.page_table.size());
    // On a failed launch the step is undone: num_cached restored, the pages
    // it opened returned to the free lists, newest first, so the LIFO order
    // of the next allocations is what it would have been.
    auto undo = [&] {
        layer.num_cached = prev_cached;
        while (layer.page_table.size() > prev_pages) {
            layer.k_pool.free(layer.page_table.back().k_block_id);
            layer.v_pool.free(layer.page_table.back().v_block_id);
            layer.page_table.pop_back();
        }
    };

    std::lock_guard<std::mutex> lock(g_mu);
    DeviceMirror& dm = g_mirrors[{mgr, layer_id}];
    if (prev_cached < dm.last_cached) dm.published = 0;  // reset_kv_cache happened: ids were reissued
    if (!dm.table || dm.capacity < n_pages) {
        const int32_t cap = std::max<int32_t>(256, 2 * n_pages);
        gkv_table* t = nullptr;
        if (gkv_table_create(dev_id, cap, &t) != GKV_OK) {
            undo();
            raise("device table");
        }
        if (dm.table) gkv_table_destroy(dm.table);
        dm.table = t;
        dm.capacity = cap;
        dm.published = 0;
    }
    std::vector<int32_t> k_ids, v_ids;
    for (int32_t i = dm.published; i < n_pages; ++i) {
        k_ids.push_back(layer.page_table[i].k_block_id);
        v_ids.push_back(layer.page_table[i].v_block_id);
    }
    gkv_new_pages np{dm.published, static_cast<int32_t>(k_ids.size()), k_ids.data(), v_ids.data()};
    // The pools' full reserved extent (fixed per layer, so the library's
    // tensor maps are encoded once), not the allocation high-water mark.
    gkv_pool_desc pool{layer.k_pool.block_data(0), layer.v_pool.block_data(0),
                       std::min(capacity(layer.k_pool), capacity(layer.v_pool)), n_kv_heads, head_dim,
                       to_gkv_dtype(K->dtype)};
    if (gkv_paged_attention_raw(&pool, dm.table, prev_cached, &np, Q->data, K->data, V->data, out->data,
                                n_q_heads, seq_len, scale, causal ? 1 : 0, to_gkv_dtype(out->dtype),
                                nullptr) != GKV_OK) {
        undo();
        raise("launch");
    }
    dm.published = n_pages;
    dm.last_cached = layer.num_cached;
}

template struct PagedAttentionImpl<Device::CUDA>;

}  // namespace ops
