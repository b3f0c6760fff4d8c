// ref_ops_harness.cpp — C entry points that drive the UNMODIFIED reference
// CPU RMSNorm, RoPE and RoPE-cache ops.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles this file with the
// reference's src/backend/cpu/{normalization,rope}.cpp, read in place, into
// oracle/_ref/libgenllm_ref_ops.so, using the reference build's own CPU flags
// (CMakeLists.txt: -O3 for Release, -mavx2 -mf16c -mfma, C++23; the files use
// only `#pragma omp simd`, built with -fopenmp-simd), so
// that the float contractions the compiler applies are the reference's. It
// pins the C restatement (qk_rope_oracle.c) and makes golden fixtures; the
// product never links it.
#include <cstdint>

#include "backend/cpu/normalization.h"
#include "backend/cpu/rope.h"
#include "core/tensor.hpp"

extern "C" {

// ops::RmsNormImpl<CPU>::execute (src/backend/cpu/normalization.cpp:146-160)
// on `rows` rows of `dim` bf16 values with an fp32 weight of `dim`.
void ref_rms_norm(const void* x, const float* w, void* out, int64_t rows, int64_t dim, float eps) {
    Tensor tx, tw, to;
    tx.data = const_cast<void*>(x);
    tx.dtype = DataType::GGML_TYPE_BF16;
    tx.dims = {1, rows, dim, 0};
    tw.data = const_cast<float*>(w);
    tw.dtype = DataType::GGML_TYPE_F32;
    tw.dims = {dim, 0, 0, 0};
    to.data = out;
    to.dtype = DataType::GGML_TYPE_BF16;
    to.dims = tx.dims;
    to.src[0] = &tx;
    to.src[1] = &tw;
    to.op_params = {eps, 0, 0, 0};
    ops::RmsNormImpl<Device::CPU>::execute(&to, 0);
}

// ops::ApplyRopeImpl<CPU>::execute (src/backend/cpu/rope.cpp:73-110) on
// x [1][n_heads][seq][head_dim] bf16 with cos/sin [max_seq][head_dim] f32.
void ref_apply_rope(const void* x, void* out, const float* cos, const float* sin, int64_t n_heads, int64_t seq,
                    int64_t head_dim, int64_t start_pos, int64_t max_seq) {
    Tensor tx, tc, ts, to;
    tx.data = const_cast<void*>(x);
    tx.dtype = DataType::GGML_TYPE_BF16;
    tx.dims = {1, n_heads, seq, head_dim};
    tc.data = const_cast<float*>(cos);
    tc.dtype = DataType::GGML_TYPE_F32;
    tc.dims = {max_seq, head_dim, 0, 0};
    ts = tc;
    ts.data = const_cast<float*>(sin);
    to.data = out;
    to.dtype = DataType::GGML_TYPE_BF16;
    to.dims = tx.dims;
    to.src[0] = &tx;
    to.src[1] = &tc;
    to.src[2] = &ts;
    to.op_params = {static_cast<float>(head_dim), 0, static_cast<float>(start_pos), 0};
    ops::ApplyRopeImpl<Device::CPU>::execute(&to, 0);
}

// ops::RopeCacheImpl<CPU>::execute (src/backend/cpu/rope.cpp:112-140): the
// cos table when the tensor's name holds "_cos", else the sin table.
void ref_rope_cache(float theta, int32_t head_dim, int32_t max_seq, float* cos_out, float* sin_out) {
    Tensor tc, ts;
    tc.data = cos_out;
    tc.dtype = DataType::GGML_TYPE_F32;
    tc.dims = {max_seq, head_dim, 0, 0};
    tc.op_params = {theta, static_cast<float>(head_dim), static_cast<float>(max_seq), 0};
    tc.name = "rope_cos";
    ts = tc;
    ts.data = sin_out;
    ts.name = "rope_sin";
    ops::RopeCacheImpl<Device::CPU>::execute(&tc, 0);
    ops::RopeCacheImpl<Device::CPU>::execute(&ts, 0);
}

}  // extern "C"
