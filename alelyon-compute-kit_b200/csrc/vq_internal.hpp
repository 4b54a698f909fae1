// Entry points between the vq4 translation units: the dispatcher
// (vq_kernels.cu) routes an admitted plan to the unit that launches it.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "vq_plan.hpp"

namespace ack {

// vq_codec.cu: decode, encode, the shader AdamW (op 3) and the fused
// coded-state AdamW passes (ops 18-20); codebooks in constant-bank slots.
cudaError_t launch_encode(uint32_t group, const float* x, uint64_t n, const float* book, uint32_t* codes,
                          uint32_t* status, cudaStream_t s);
cudaError_t launch_decode(uint32_t group, const uint32_t* codes, const float* book, float* out, uint64_t n,
                          uint32_t* status, cudaStream_t s);
cudaError_t launch_adamw_shader(const Plan& p, void* const* ptr, cudaStream_t s);
cudaError_t launch_adamw_fused(const Plan& p, void* const* ptr, cudaStream_t s);

// vq_products.cu: the shader's packed-pair product (op 2), the dense and
// coded products (ops 16, 17) and the tile32 repack (op 23).
cudaError_t launch_matmul_exact(const Plan& p, void* const* ptr, cudaStream_t s);
cudaError_t launch_dense(const Plan& p, void* const* ptr, cudaStream_t s);
cudaError_t launch_coded(const Plan& p, void* const* ptr, cudaStream_t s);
cudaError_t launch_repack(const Plan& p, void* const* ptr, cudaStream_t s);

// vq_gemm_tc.cu: the dense product on the tensor cores (op 16, flag 8).
cudaError_t launch_dense_tc(const Plan& p, void* const* ptr, cudaStream_t s);

// vq_harness.cu: the expert harness's residual and gradient clip (ops 26, 27).
cudaError_t launch_residual(const Plan& p, void* const* ptr, cudaStream_t s);
cudaError_t launch_clip(const Plan& p, void* const* ptr, cudaStream_t s);

// vq_fit.cu: fit_codebook on the device (ops 24, 25).
cudaError_t launch_adamw_fit(const Plan& p, void* const* ptr, cudaStream_t s);
cudaError_t launch_fit_values(const Plan& p, void* const* ptr, cudaStream_t s);

}  // namespace ack
