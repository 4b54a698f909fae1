// The expert harness's host arithmetic on the device (ops 26, 27), so a
// train step keeps its residual and gradient in HBM:
//
//   op 26  r = prediction - decode(target), out = r * s (FP32), and the
//          float64 sum of r^2 (the MSE loss is that sum / count);
//          harness.py:189-193 (residual, loss, the 2 / size scaling)
//   op 27  norm = sqrt(sum g^2) in float64, scale = min(1, max / (norm +
//          1e-6)), out = g * fl32(scale); harness.py:196-200
//
// Both reductions are deterministic: a fixed grid for a given count, each
// block sums its values in a fixed order into one float64 partial, and one
// block adds the partials in index order. The residual and the scaling are
// single FP32 operations, rounded like the host's numpy arithmetic; the
// float64 sums differ from numpy's (pairwise) and BLAS's orders only in
// their last bits.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "vq_common.cuh"

namespace ack {
namespace {

constexpr int kRedThreads = 256;

uint32_t reduce_grid(uint64_t count) {
  const uint64_t want = (count + 4 * kRedThreads - 1) / (4 * kRedThreads);
  return uint32_t(std::max<uint64_t>(1, std::min<uint64_t>(want, kReducePartials)));
}

// The block's float64 sum of `v` over its threads, in a fixed order (warp
// trees, then the warps' sums in order by thread 0). Valid in thread 0.
__device__ double block_sum(double v) {
  __shared__ double warp_sums[kRedThreads / 32];
#pragma unroll
  for (int o = 16; o; o >>= 1) v = __dadd_rn(v, __shfl_down_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x / 32] = v;
  __syncthreads();
  double total = 0.0;
  if (threadIdx.x == 0)
    for (int w = 0; w < kRedThreads / 32; ++w) total = __dadd_rn(total, warp_sums[w]);
  return total;
}

template <int G>
__global__ void __launch_bounds__(kRedThreads) k_residual(const float* __restrict__ pred,
                                                          const uint32_t* __restrict__ codes,
                                                          const float* __restrict__ book, uint64_t count,
                                                          float scale, float* __restrict__ out,
                                                          double* __restrict__ partials,
                                                          uint32_t* __restrict__ status) {
  __shared__ float sb[16 * G];
  for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) sb[i] = book[i];
  __syncthreads();
  double acc = 0.0;
  uint32_t bits = 0;
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
    const float r = __fsub_rn(pred[i], sb[code_at(codes, i / G) * G + uint32_t(i % G)]);
    bits |= finite32(r) ? 0u : kNonfinite;
    acc = __fma_rn(double(r), double(r), acc);
    out[i] = __fmul_rn(r, scale);
  }
  flag_warp(status, bits);
  const double s = block_sum(acc);
  if (threadIdx.x == 0) partials[blockIdx.x] = s;
}

__global__ void __launch_bounds__(kRedThreads) k_sumsq(const float* __restrict__ x, uint64_t count,
                                                       double* __restrict__ partials) {
  double acc = 0.0;
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
    const double v = double(x[i]);
    acc = __fma_rn(v, v, acc);
  }
  const double s = block_sum(acc);
  if (threadIdx.x == 0) partials[blockIdx.x] = s;
}

// One block: the partials added in index order (each thread a strided
// subsequence, then the block's fixed tree). total[0] = the sum.
__global__ void __launch_bounds__(kRedThreads) k_sum_partials(const double* __restrict__ partials, uint32_t n,
                                                              double* __restrict__ total) {
  double acc = 0.0;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) acc = __dadd_rn(acc, partials[i]);
  const double s = block_sum(acc);
  if (threadIdx.x == 0) total[0] = s;
}

// `sumsq` holds sum g^2 (from k_sum_partials); every block derives norm and
// scale from it, thread 0 of block 0 writes stats = [norm, scale].
__global__ void __launch_bounds__(kRedThreads) k_clip(const float* __restrict__ x, uint64_t count, double max_norm,
                                                      const double* __restrict__ sumsq, double* __restrict__ stats,
                                                      float* __restrict__ out, uint32_t* __restrict__ status) {
  const double norm = __dsqrt_rn(sumsq[0]);
  const double scale = fmin(1.0, __ddiv_rn(max_norm, __dadd_rn(norm, 1e-6)));
  const float sf = __double2float_rn(scale);
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride)
    out[i] = __fmul_rn(x[i], sf);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (!(norm == norm) || norm > 1.7976931348623157e308) atomicOr(status, kNonfinite);
    stats[0] = norm;
    stats[1] = scale;
  }
}

}  // namespace

cudaError_t launch_residual(const Plan& p, void* const* ptr, cudaStream_t s) {
  const uint64_t count = p.m;
  const uint32_t grid = reduce_grid(count);
  float scale;
  memcpy(&scale, &p.aux0, sizeof(scale));
  double* partials = static_cast<double*>(ptr[4]);
  if ((reinterpret_cast<uintptr_t>(ptr[4]) | reinterpret_cast<uintptr_t>(ptr[6])) & 7u)
    return cudaErrorMisalignedAddress;  // float64 partials and sum
  const float* pred = static_cast<const float*>(ptr[0]);
  const uint32_t* codes = static_cast<const uint32_t*>(ptr[1]);
  const float* book = static_cast<const float*>(ptr[2]);
  float* out = static_cast<float*>(ptr[5]);
  uint32_t* status = static_cast<uint32_t*>(ptr[7]);
  switch (p.group) {
    case 8: k_residual<8><<<grid, kRedThreads, 0, s>>>(pred, codes, book, count, scale, out, partials, status); break;
    case 16: k_residual<16><<<grid, kRedThreads, 0, s>>>(pred, codes, book, count, scale, out, partials, status); break;
    default: k_residual<32><<<grid, kRedThreads, 0, s>>>(pred, codes, book, count, scale, out, partials, status);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k_sum_partials<<<1, kRedThreads, 0, s>>>(partials, grid, static_cast<double*>(ptr[6]));
  return cudaGetLastError();
}

cudaError_t launch_clip(const Plan& p, void* const* ptr, cudaStream_t s) {
  const uint64_t count = p.m;
  const uint32_t grid = reduce_grid(count);
  const uint64_t bits = uint64_t(p.aux0) | (uint64_t(p.aux1) << 32);
  double max_norm;
  static_assert(sizeof(max_norm) == sizeof(bits), "float64 bits");
  memcpy(&max_norm, &bits, sizeof(bits));
  const float* x = static_cast<const float*>(ptr[0]);
  double* partials = static_cast<double*>(ptr[4]);
  double* stats = static_cast<double*>(ptr[6]);
  if ((reinterpret_cast<uintptr_t>(ptr[4]) | reinterpret_cast<uintptr_t>(ptr[6])) & 7u)
    return cudaErrorMisalignedAddress;  // float64 partials and results
  k_sumsq<<<grid, kRedThreads, 0, s>>>(x, count, partials);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // the sum lands after the partials (the workspace holds kReducePartials + 1 values)
  double* sumsq = partials + kReducePartials;
  k_sum_partials<<<1, kRedThreads, 0, s>>>(partials, grid, sumsq);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k_clip<<<grid, kRedThreads, 0, s>>>(x, count, max_norm, sumsq, stats, static_cast<float*>(ptr[5]),
                                      static_cast<uint32_t*>(ptr[7]));
  return cudaGetLastError();
}

}  // namespace ack
