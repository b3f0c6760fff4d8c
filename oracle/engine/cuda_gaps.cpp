// cuda_gaps.cpp — test infrastructure for the engine build. The Genllm
// sources dispatch kernel::sigmoid to ops::SigmoidImpl<Device::CUDA>
// (src/core/kernels.cpp:63) but define it only for the CPU
// (include/backend/cpu/activation.h:27); the engine's CUDA build therefore
// does not link as shipped. Sigmoid is used only by the Qwen3.5 graph, not by
// Qwen3, so the missing specialization is provided as an error.
#include <stdexcept>

#include "cuda_gaps.h"

namespace ops {
void SigmoidImpl<Device::CUDA>::execute(Tensor*, int32_t) {
    throw std::runtime_error("sigmoid: no CUDA implementation in the Genllm sources (not on the Qwen3 path)");
}
}  // namespace ops
