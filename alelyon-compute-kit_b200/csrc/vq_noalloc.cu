// The encode entry that allocates nothing (ack_vq_encode_noalloc).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "vq_common.cuh"
#include "vq_kernels.hpp"

namespace ack {

// ------------------------------------------------ encode without allocation --
// The encode of ack_vq_encode_noalloc: the same certified search as
// k_encode, for callers that may not allocate anything on the device (a
// host whose allocator owns all device memory, code running where an
// allocation would stall or be refused). Its only scratch, each tensor's
// book staged pair-interleaved with its BookMeta, lives in the fixed array
// below instead of the constant-bank slot ring (whose events are created on
// first use): kStaticEncodeBooks books of at most group 32, 139,264 bytes
// per device, held by every GPU that loads the library until exit.
namespace {

static __device__ __align__(256) float g_static_scratch[kStaticEncodeBooks * kStaticBookFloats];

// Block b stages book b of `books` into scratch entry b (every word of the
// entry that the encode reads is written, so no clearing is needed).
template <int G>
__global__ void k_static_stage(const float* __restrict__ books, float* __restrict__ scratch) {
  __shared__ BookMeta m;
  const int lane = threadIdx.x & 31;
  const float* book = books + uint64_t(blockIdx.x) * 16 * G;
  float* dst = scratch + uint64_t(blockIdx.x) * kStaticBookFloats;
  for (int i = lane; i < 16 * G; i += 32) dst[book_pos<G>(i / G, i % G)] = book[i];
  meta_compute<G>(book, m);
  __syncwarp();
  constexpr int kWords = sizeof(BookMeta) / 4;
  if (lane < kWords) reinterpret_cast<uint32_t*>(dst + kStaticMetaOffset)[lane] = reinterpret_cast<const uint32_t*>(&m)[lane];
}

// Tensor blockIdx.y: x + y n values, codes + y words; the grid's x
// dimension strides over its vectors (one per lane, 32 per warp step).
template <int G, bool VEC>
__global__ void __launch_bounds__(kThreads, 2) k_encode_static(const float* __restrict__ x, uint64_t n,
                                                               uint32_t* __restrict__ codes,
                                                               uint32_t* __restrict__ status,
                                                               const float* __restrict__ scratch) {
  using Book = SBook<G>;
  const uint32_t t = blockIdx.y;
  const float4* src = reinterpret_cast<const float4*>(scratch + uint64_t(t) * kStaticBookFloats);
  for (int i = threadIdx.x; i < kStaticBookFloats / 4; i += blockDim.x) s_static_book[i] = src[i];
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x == 0 && Book::bad()) atomicOr(status, kNonfinite);
  const uint64_t vectors = (n + G - 1) / G, full = n / G, words = (vectors + 7) / 8;
  const float* xt = x + uint64_t(t) * n;
  uint32_t* ct = codes + uint64_t(t) * words;
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t stride = uint64_t(gridDim.x) * (blockDim.x / 32) * 32;
  for (uint64_t base = (uint64_t(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32) * 32; base < vectors;
       base += stride) {
    const uint64_t v = base + lane;
    uint32_t idx = 0, bits = 0;
    if (v < full) {
      float xr[G];
      enc_load<G, VEC>(xt, v, full, xr);
      bool certified;
      const float* vsrc = xt + v * G;
      idx = enc_vector<G, Book>(xr, &certified, vsrc);
      if (certified)
        for (int j = 0; j < G; ++j) bits |= finite32(vsrc[j]) ? 0u : kNonfinite;
    } else if (v < vectors) {
      const int valid = int(n - v * G);  // the partial last vector (vq.py:171-172)
      const float* vsrc = xt + v * G;
      for (int j = 0; j < valid; ++j) bits |= finite32(vsrc[j]) ? 0u : kNonfinite;
      idx = enc_exact_mem<G, Book>(vsrc, valid, 0xffffu);
    }
    const uint32_t w = pack_nibbles(idx);
    const uint64_t word = (base >> 3) + (lane >> 3);
    if ((lane & 7) == 0 && word < words) ct[word] = w;
    flag_warp(status, bits);
  }
}

// Device address of g_static_scratch: looked up with cudaGetSymbolAddress
// the first time each device (current at the call) encodes here, then
// cached. The array's name in host code is only a host-side stand-in, never
// a device pointer.
float* static_scratch(cudaError_t* err) {
  static std::mutex mu;
  static float* addr[kMaxDevices] = {};
  int dev = 0;
  *err = current_device(&dev);
  if (*err != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    float* p = nullptr;
    *err = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_static_scratch);
    if (*err != cudaSuccess) return nullptr;
    addr[dev] = p;
  }
  return addr[dev];
}

template <int G>
cudaError_t encode_static_group(const float* x, uint64_t n, uint32_t batch, const float* books, uint32_t* codes,
                                uint32_t* status, float* scratch, cudaStream_t s) {
  k_static_stage<G><<<batch, 32, 0, s>>>(books, scratch);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const uint64_t vectors = (n + G - 1) / G;
  const bool vec = aligned16(x) && (n * sizeof(float)) % 16 == 0;
  const uint64_t cap = uint64_t(sm_count()) * resident_per_sm(k_encode_static<G, true>, 0);
  const uint64_t want = (vectors + kThreads - 1) / kThreads;
  const uint32_t gx = uint32_t(std::max<uint64_t>(1, std::min<uint64_t>(want, (cap + batch - 1) / batch)));
  const dim3 grid(gx, batch);
  if (vec) k_encode_static<G, true><<<grid, kThreads, 0, s>>>(x, n, codes, status, scratch);
  else k_encode_static<G, false><<<grid, kThreads, 0, s>>>(x, n, codes, status, scratch);
  return cudaGetLastError();
}

}  // namespace

cudaError_t encode_noalloc(const float* x, uint64_t n, uint32_t batch, const float* books, uint32_t group,
                           uint32_t* codes, uint32_t* status, cudaStream_t s) {
  cudaError_t err = cudaSuccess;
  float* scratch = static_scratch(&err);
  if (!scratch) return err;
  if (group == 8) return encode_static_group<8>(x, n, batch, books, codes, status, scratch, s);
  if (group == 16) return encode_static_group<16>(x, n, batch, books, codes, status, scratch, s);
  return encode_static_group<32>(x, n, batch, books, codes, status, scratch, s);
}


}  // namespace ack
