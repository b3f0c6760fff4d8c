// flash_attention_cuda.cpp — drop-in ops::FlashAttentionImpl<Device::CUDA>
// for the Genllm engine, on libgenllm_kv.so (include/genllm_kv.h).
//
// Replaces the definition in src/backend/cuda/attention.cu:317-399 (the
// declaration in include/backend/cuda/attention.h stays): the same tensors
// and op_params (head_dim, scale, causal, n_kv_groups), self-attention of
// each of the B sequences, now on the tcgen05 kernel instead of a warp-per-
// query SIMT kernel. Like the reference, the call is stream-ordered on the
// default stream of device dev_id.
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "backend/cuda/attention.h"
#include "genllm_kv.h"

namespace {

int32_t to_gkv_dtype(DataType d) {
    switch (d) {
        case DataType::GGML_TYPE_F32: return GKV_F32;
        case DataType::GGML_TYPE_F16: return GKV_F16;
        case DataType::GGML_TYPE_BF16: return GKV_BF16;
        default: throw std::runtime_error("flash_attention: unsupported dtype");
    }
}

}  // namespace

namespace ops {

void FlashAttentionImpl<Device::CUDA>::execute(Tensor* out, int32_t dev_id) {
    cudaSetDevice(dev_id);
    const Tensor* Q = out->src[0];
    const Tensor* K = out->src[1];
    const Tensor* V = out->src[2];
    const int32_t head_dim = static_cast<int32_t>(out->op_params[0]);
    const float scale = out->op_params[1];
    const int32_t causal = static_cast<int32_t>(out->op_params[2]);
    const int32_t st = gkv_flash_attention(
        Q->data, K->data, V->data, out->data, static_cast<int32_t>(Q->dims[0]), static_cast<int32_t>(Q->dims[1]),
        static_cast<int32_t>(K->dims[1]), static_cast<int32_t>(Q->dims[2]), head_dim, scale, causal,
        to_gkv_dtype(Q->dtype), to_gkv_dtype(out->dtype), nullptr);
    if (st != GKV_OK) throw std::runtime_error(std::string("flash_attention: ") + gkv_last_error());
}

}  // namespace ops

template struct ops::FlashAttentionImpl<Device::CUDA>;
