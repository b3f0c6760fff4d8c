// ref_harness.cpp — C entry points that drive the UNMODIFIED reference CPU
// paged-attention op and its page allocator.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles this file together with
// the reference's own translation units (src/core/{page_attention,pools,
// resource_cpu,manager,gguf_parser}.cpp and src/backend/cpu/attention.cpp,
// read in place from the reference tree) into oracle/_ref/libgenllm_ref.so.
// It is used to pin the C restatement (paged_oracle.c), to make the golden
// fixtures, and as the timed CPU baseline. The product never links it.
//
// The set-up mirrors what the reference's scheduler does for one device
// (src/core/scheduler.cpp:364-373, 404-430): a kv_cache MemoryPool, one
// PagedAttentionManager, then init_layer + reserve_layer per layer.
#include <cstring>
#include <memory>
#include <thread>
#include <vector>

#include "backend/cpu/attention.h"
#include "core/manager.h"
#include "core/page_attention.h"
#include "core/tensor.hpp"

namespace {
struct RefSession {
    std::unique_ptr<MemoryManager> mm;
    PagedAttentionManager* mgr = nullptr;
    int32_t n_kv_heads = 0, head_dim = 0, max_blocks = 0;
    std::byte* kv_base = nullptr;  // start of the kv_cache MemoryPool buffer
    DataType dtype = DataType::GGML_TYPE_BF16;
};

DataType to_dt(int32_t code) { return static_cast<DataType>(code); }
}  // namespace

extern "C" {

// One MemoryManager (it installs itself as g_mem_manager, which the op uses)
// with n_layers paged layers of max_blocks pages each.
void* ref_session_create(int32_t n_layers, int32_t n_kv_heads, int32_t head_dim,
                         int32_t max_blocks, int32_t dtype) {
    auto* s = new RefSession();
    s->mm = std::make_unique<MemoryManager>();
    s->n_kv_heads = n_kv_heads;
    s->head_dim = head_dim;
    s->max_blocks = max_blocks;
    s->dtype = to_dt(dtype);
    size_t block_bytes = static_cast<size_t>(PAGE_BLOCK_SIZE) * n_kv_heads * head_dim *
                         data_type_size(s->dtype);
    size_t kv_bytes = (2 * static_cast<size_t>(max_blocks) * block_bytes + 64) * n_layers;
    s->mm->get_or_create(Device::CPU, 0, 0, 0, kv_bytes);
    s->mgr = &s->mm->create_attention_manager(Device::CPU, 0);
    for (int32_t l = 0; l < n_layers; ++l) {
        s->mgr->init_layer(l, n_kv_heads, head_dim, s->dtype);
        s->mgr->reserve_layer(l, max_blocks);
    }
    // MemoryPool exposes no base pointer; a 1-byte block at the cursor gives
    // base + offset, from which base follows. The layers' pools record their
    // offsets (BlockPool::device_offset), which locates each K and V region.
    MemoryBlock probe = s->mm->get(Device::CPU, 0)->kv_cache->allocate(1, 1);
    s->kv_base = static_cast<std::byte*>(probe.ptr) - probe.offset;
    return s;
}

void ref_session_destroy(void* h) { delete static_cast<RefSession*>(h); }

void* ref_layer_k_base(void* h, int32_t layer) {
    auto* s = static_cast<RefSession*>(h);
    return s->kv_base + s->mgr->get_layer(layer).k_pool.device_offset();
}
void* ref_layer_v_base(void* h, int32_t layer) {
    auto* s = static_cast<RefSession*>(h);
    return s->kv_base + s->mgr->get_layer(layer).v_pool.device_offset();
}

int32_t ref_page_alloc(void* h, int32_t layer, int32_t which) {
    auto& L = static_cast<RefSession*>(h)->mgr->get_layer(layer);
    return which == 0 ? L.k_pool.alloc() : L.v_pool.alloc();
}
void ref_page_free(void* h, int32_t layer, int32_t which, int32_t id) {
    auto& L = static_cast<RefSession*>(h)->mgr->get_layer(layer);
    if (which == 0) L.k_pool.free(id); else L.v_pool.free(id);
}
void ref_pool_stats(void* h, int32_t layer, int32_t which, int32_t* num_blocks, int32_t* num_free) {
    auto& L = static_cast<RefSession*>(h)->mgr->get_layer(layer);
    BlockPool& p = which == 0 ? L.k_pool : L.v_pool;
    *num_blocks = p.num_blocks();
    *num_free = p.num_free();
}

// Overwrite the layer's page table and cached-token count (the harness's way
// to build a fragmented cache, as the reference has no API for it).
void ref_set_table(void* h, int32_t layer, const int32_t* k_ids, const int32_t* v_ids,
                   int32_t n_pages, int32_t num_cached) {
    auto& L = static_cast<RefSession*>(h)->mgr->get_layer(layer);
    L.page_table.clear();
    for (int32_t i = 0; i < n_pages; ++i) L.page_table.push_back({k_ids[i], v_ids[i]});
    L.num_cached = num_cached;
}

int32_t ref_get_table(void* h, int32_t layer, int32_t* k_ids, int32_t* v_ids, int32_t cap,
                      int32_t* num_cached) {
    auto& L = static_cast<RefSession*>(h)->mgr->get_layer(layer);
    int32_t n = static_cast<int32_t>(L.page_table.size());
    for (int32_t i = 0; i < n && i < cap; ++i) {
        k_ids[i] = L.page_table[i].k_block_id;
        v_ids[i] = L.page_table[i].v_block_id;
    }
    *num_cached = L.num_cached;
    return n;
}

void ref_append_pages(void* h, int32_t layer, int32_t count) {
    static_cast<RefSession*>(h)->mgr->append_kv_pages(layer, count);
}

void ref_append_kv(void* h, int32_t layer, const void* K, const void* V, int32_t seq_len) {
    auto* s = static_cast<RefSession*>(h);
    s->mgr->append_kv_from_tensor(layer, K, V, s->n_kv_heads, seq_len, s->head_dim, s->dtype);
}

void ref_reset(void* h) { static_cast<RefSession*>(h)->mm->reset_kv_cache(); }

// One call of ops::PagedAttentionImpl<Device::CPU>::execute: append K/V
// ([1][Hkv][S][D]) into the layer's pages, then attend Q ([1][Hq][S][D]).
// out is [1][Hq][S][D] in Q's dtype, as the reference writes it.
void ref_paged_attention(void* h, int32_t layer, void* Q, void* K, void* V, void* out,
                         int32_t n_q_heads, int32_t seq_len, float scale, int32_t causal) {
    auto* s = static_cast<RefSession*>(h);
    Tensor q, k, v, o;
    q.data = Q; k.data = K; v.data = V; o.data = out;
    for (Tensor* t : {&q, &k, &v, &o}) { t->device = Device::CPU; t->dtype = s->dtype; }
    q.dims = {1, n_q_heads, seq_len, s->head_dim};
    k.dims = {1, s->n_kv_heads, seq_len, s->head_dim};
    v.dims = k.dims;
    o.dims = q.dims;
    o.src[0] = &q; o.src[1] = &k; o.src[2] = &v;
    o.layer_id = layer;
    o.op_type = OperationType::OP_TYPE_PAGED_ATTN;
    o.op_params = {static_cast<float>(s->head_dim), scale, static_cast<float>(causal),
                   static_cast<float>(n_q_heads / s->n_kv_heads)};
    ops::PagedAttentionImpl<Device::CPU>::execute(&o, 0);
}

// The same op on several layers at once, one host thread per layer (the op is
// single-threaded; distinct layers touch disjoint state). Used to time the
// reference with every host core it can use.
void ref_paged_attention_layers(void* h, int32_t n_layers, void** Q, void** K, void** V,
                                void** out, int32_t n_q_heads, int32_t seq_len, float scale,
                                int32_t causal) {
    std::vector<std::thread> th;
    for (int32_t l = 0; l < n_layers; ++l)
        th.emplace_back([=] { ref_paged_attention(h, l, Q[l], K[l], V[l], out[l], n_q_heads,
                                                  seq_len, scale, causal); });
    for (auto& t : th) t.join();
}

// One call of ops::FlashAttentionImpl<Device::CPU>::execute
// (src/backend/cpu/attention.cpp:39-120): Q [B][Hq][S][D], K/V [B][Hkv][S][D]
// bf16; out [B][Hq][S][D] bf16, as the reference writes it.
void ref_flash_attention(const void* Q, const void* K, const void* V, void* out, int32_t batch, int32_t n_q_heads,
                         int32_t n_kv_heads, int32_t seq_len, int32_t head_dim, float scale, int32_t causal) {
    Tensor q, k, v, o;
    q.data = const_cast<void*>(Q); k.data = const_cast<void*>(K); v.data = const_cast<void*>(V); o.data = out;
    for (Tensor* t : {&q, &k, &v, &o}) { t->device = Device::CPU; t->dtype = DataType::GGML_TYPE_BF16; }
    q.dims = {batch, n_q_heads, seq_len, head_dim};
    k.dims = {batch, n_kv_heads, seq_len, head_dim};
    v.dims = k.dims;
    o.dims = q.dims;
    o.src[0] = &q; o.src[1] = &k; o.src[2] = &v;
    o.op_params = {static_cast<float>(head_dim), scale, static_cast<float>(causal),
                   static_cast<float>(n_q_heads / n_kv_heads)};
    ops::FlashAttentionImpl<Device::CPU>::execute(&o, 0);
}

}  // extern "C"
