// sm_100a kernels of the vq4/v1 path and their launcher.
//
//   decode        HBM-write-bound gather: 128-bit streaming stores, warp
//                 steps of 256 vectors whose code words arrive as one line
//                 and move by shuffle, the codebook in shared memory
//                 (vq4.comp op 1 / vq.py:117-121)
//   encode        certified nearest entry per vector (vq4.comp op 0 /
//                 vq.py:154-179): aligned input takes k_encode_tc (TMA tiles,
//                 tcgen05 tf32 filter, deferred FP32 refinement of the few
//                 near ties, float64 pass for what stays tied); otherwise
//                 k_encode (FP32 filter on the CUDA cores); lanes of a warp
//                 own consecutive vectors and pack nibbles with shuffles
//   matmul_exact  the shader's packed-pair product (vq4.comp:165-176):
//                 64x64 tiles dequantised into shared memory, each output
//                 summed in k order with separately rounded multiply and add
//   adamw         the shader's AdamW (vq4.comp:87-116), one value per thread
//   dense_lut     Y = X * decode(W)^T with W stored N x K: a per-group table
//                 P[m][t][e] = x[m, tg:tg+g] . c_e in shared memory, then one
//                 table lookup and add per (row, group); code tiles staged by
//                 cp.async into padded shared rows
//   coded_lut     C = decode(A) * decode(B)^T: a 16x16 table L = C_A C_B^T,
//                 one lookup and add per (row, column, group)
//   gemm_generic  any layout: 64x64 tiles dequantised into shared memory,
//                 FP32 FMA
//   adamw_*       fused coded-state AdamW: sampled values, whole-tensor entry
//                 usage, and decode -> AdamW -> encode of W', M', V'
//
// The kernels live in vq_codec.cu, vq_products.cu, vq_fit.cu and
// vq_noalloc.cu; this unit routes an admitted plan to them.
#include <cuda_runtime.h>

#include "vq_internal.hpp"
#include "vq_kernels.hpp"

namespace ack {

cudaError_t launch(const Plan& p, void* const* ptr, cudaStream_t s) {
  const uint32_t g = p.group;
  if (p.schema == 1) {
    switch (p.op) {
      case Op::Encode:
        return launch_encode(g, static_cast<const float*>(ptr[0]), p.m, static_cast<const float*>(ptr[1]),
                             static_cast<uint32_t*>(ptr[4]), static_cast<uint32_t*>(ptr[5]), s);
      case Op::Decode:
        return launch_decode(g, static_cast<const uint32_t*>(ptr[0]), static_cast<const float*>(ptr[1]),
                             static_cast<float*>(ptr[4]), p.m, static_cast<uint32_t*>(ptr[5]), s);
      case Op::Matmul:
        return launch_matmul_exact(p, ptr, s);
      case Op::AdamW:
        return launch_adamw_shader(p, ptr, s);
      default:
        return cudaErrorInvalidValue;
    }
  }
  switch (p.op) {
    case Op::Dense: return (p.flags & 8u) ? launch_dense_tc(p, ptr, s) : launch_dense(p, ptr, s);
    case Op::Coded: return launch_coded(p, ptr, s);
    case Op::AdamwSample:
    case Op::AdamwUsage:
    case Op::AdamwEncode: return launch_adamw_fused(p, ptr, s);
    case Op::EncodeLarge:
      return launch_encode(g, static_cast<const float*>(ptr[0]), p.m, static_cast<const float*>(ptr[1]),
                           static_cast<uint32_t*>(ptr[5]), static_cast<uint32_t*>(ptr[7]), s);
    case Op::DecodeLarge:
      return launch_decode(g, static_cast<const uint32_t*>(ptr[0]), static_cast<const float*>(ptr[1]),
                           static_cast<float*>(ptr[5]), p.m, static_cast<uint32_t*>(ptr[7]), s);
    case Op::Fit: return launch_fit_values(p, ptr, s);
    case Op::AdamwFit: return launch_adamw_fit(p, ptr, s);
    case Op::RepackTile32: return launch_repack(p, ptr, s);
    case Op::Residual: return launch_residual(p, ptr, s);
    case Op::ClipNorm: return launch_clip(p, ptr, s);
    default:
      return cudaErrorInvalidValue;
  }
}


}  // namespace ack
