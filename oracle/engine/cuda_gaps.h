// cuda_gaps.h — declares the one operator specialization the Genllm CUDA
// build lacks (see cuda_gaps.cpp); force-included into src/core/kernels.cpp.
#pragma once
#include "backend/cpu/activation.h"

namespace ops {
template <>
struct SigmoidImpl<Device::CUDA> {
    static void execute(Tensor* out, int32_t dev_id);
};
}  // namespace ops
