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
// An exhausted pool throws instead of leaving num_cached ahead of the table
// (src/core/page_attention.cpp:155,161).
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

    // Host allocation by the reference's own allocator.
    mgr->append_kv_pages(layer_id, seq_len);
    const int32_t n_pages = static_cast<int32_t>(layer.page_table.size());
    if (n_pages < (layer.num_cached + PAGE_BLOCK_SIZE - 1) / PAGE_BLOCK_SIZE) {
        layer.num_cached = prev_cached;
        throw std::runtime_error("paged_attention: KV page pool exhausted");
    }

    std::lock_guard<std::mutex> lock(g_mu);
    DeviceMirror& dm = g_mirrors[{mgr, layer_id}];
    if (prev_cached < dm.last_cached) dm.published = 0;  // reset_kv_cache happened: ids were reissued
    if (!dm.table || dm.capacity < n_pages) {
        const int32_t cap = std::max<int32_t>(256, 2 * n_pages);
        gkv_table* t = nullptr;
        if (gkv_table_create(dev_id, cap, &t) != GKV_OK) raise("device table");
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
    gkv_pool_desc pool{layer.k_pool.block_data(0), layer.v_pool.block_data(0),
                       std::max(layer.k_pool.num_blocks(), layer.v_pool.num_blocks()), n_kv_heads, head_dim,
                       to_gkv_dtype(K->dtype)};
    if (gkv_paged_attention_raw(&pool, dm.table, prev_cached, &np, Q->data, K->data, V->data, out->data,
                                n_q_heads, seq_len, scale, causal ? 1 : 0, to_gkv_dtype(out->dtype),
                                nullptr) != GKV_OK) {
        layer.num_cached = prev_cached;
        raise("launch");
    }
    dm.published = n_pages;
    dm.last_cached = layer.num_cached;
}

template struct PagedAttentionImpl<Device::CUDA>;

}  // namespace ops
