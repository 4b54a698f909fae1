// Kernel-side building blocks and host launch helpers shared by the vq4
// translation units (vq_codec.cu, vq_products.cu, vq_fit.cu, vq_noalloc.cu).
// Everything here has internal linkage: each unit gets its own copy.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "vq_device.cuh"
#include "vq_internal.hpp"

namespace ack {
namespace {

constexpr int kThreads = 256;

// The per-device caches of the launchers (symbol addresses, events, SM
// counts) are indexed by the CUDA device ordinal and kept for the life of
// the process; ordinals at or beyond kMaxDevices are refused.
constexpr int kMaxDevices = 64;

template <int G>
__device__ __forceinline__ void load_vector(const float* __restrict__ x, uint64_t v, float (&xr)[G]) {
  const float4* src = reinterpret_cast<const float4*>(x + v * G);
#pragma unroll
  for (int q = 0; q < G / 4; ++q) {
    const float4 t = __ldg(src + q);
    xr[4 * q + 0] = t.x;
    xr[4 * q + 1] = t.y;
    xr[4 * q + 2] = t.z;
    xr[4 * q + 3] = t.w;
  }
}

// At least 3/3/2 resident blocks for group 8/16/32 (measured best: more
// would spill the double buffer); the fused AdamW kernels
// hold more per thread.
template <int G>
constexpr int encode_min_blocks() { return G == 32 ? 2 : 3; }
template <int G>
constexpr int adamw_min_blocks() { return G == 8 ? 3 : (G == 16 ? 2 : 1); }

template <int G, bool VEC>
__device__ __forceinline__ void enc_load(const float* __restrict__ x, uint64_t v, uint64_t full, float (&xr)[G]) {
  if (v < full) {
    if (VEC) {
      load_vector<G>(x, v, xr);
    } else {
#pragma unroll
      for (int j = 0; j < G; ++j) xr[j] = x[v * G + j];
    }
  }
}

// ------------------------------------------------- fused coded-state AdamW --

struct AdamwBatch {
  const uint32_t* codes;  // [E][4][words]
  const float* books;     // [E][4][16G]
  const float* coefs;     // [E][7]
  uint64_t words;         // u32 words of one packed image
  uint32_t n;             // values per tensor
};

// AdamW outputs W', M', V' of the first `valid` values of vector v of
// expert e (zeros beyond `valid`).
template <int G>
__device__ __forceinline__ void adamw_vector3(const AdamwBatch& a, const float* __restrict__ sbooks,
                                              const AdamwCoefs& k, uint32_t e, uint64_t v, int valid, float (&w)[G],
                                              float (&m)[G], float (&var)[G], uint32_t* bits) {
  const uint32_t* base = a.codes + uint64_t(e) * 4 * a.words;
  uint32_t code[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) code[s] = code_at(base + s * a.words, v);
#pragma unroll
  for (int j = 0; j < G; ++j) {
    w[j] = m[j] = var[j] = 0.f;
    if (j < valid) {
      float nw, nm, nv;
      bool skip;
      *bits |= adamw_value(k, sbooks[0 * 16 * G + code[0] * G + j], sbooks[1 * 16 * G + code[1] * G + j],
                           sbooks[2 * 16 * G + code[2] * G + j], sbooks[3 * 16 * G + code[3] * G + j], &nw, &nm,
                           &nv, &skip);
      if (!skip) {
        w[j] = nw;
        m[j] = nm;
        var[j] = nv;
      }
    }
  }
}

// One of the three outputs (0: W', 1: M', 2: V'), for the whole-tensor
// usage pass, which needs one state only.
template <int G>
__device__ __forceinline__ void adamw_vector(const AdamwBatch& a, const float* __restrict__ sbooks,
                                             const AdamwCoefs& k, uint32_t e, uint64_t v, int valid, int state,
                                             float (&x)[G], uint32_t* bits) {
  const uint32_t* base = a.codes + uint64_t(e) * 4 * a.words;
  uint32_t code[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) code[s] = code_at(base + s * a.words, v);
#pragma unroll
  for (int j = 0; j < G; ++j) {
    x[j] = 0.f;
    if (j < valid) {
      float nw, nm, nv;
      bool skip;
      *bits |= adamw_value(k, sbooks[0 * 16 * G + code[0] * G + j], sbooks[1 * 16 * G + code[1] * G + j],
                           sbooks[2 * 16 * G + code[2] * G + j], sbooks[3 * 16 * G + code[3] * G + j], &nw, &nm,
                           &nv, &skip);
      if (!skip) x[j] = state == 0 ? nw : (state == 1 ? nm : nv);
    }
  }
}

constexpr int kStaticMetaOffset = 16 * 32;                       // floats
constexpr int kStaticBookFloats = kStaticMetaOffset + kMetaFloats;  // 544 per book

// The book of the block's tensor, copied from the scratch by each block.
__shared__ __align__(16) float4 s_static_book[kStaticBookFloats / 4];

template <int G>
struct SBook {
  static __device__ __forceinline__ float4 quad(int p, int h) { return s_static_book[(p * 2 * G) / 4 + h]; }
  static __device__ __forceinline__ float at(int e, int j) {
    return reinterpret_cast<const float*>(s_static_book)[book_pos<G>(e, j)];
  }
  static __device__ __forceinline__ float4 metaq(int i) { return s_static_book[kStaticMetaOffset / 4 + i]; }
  static __device__ __forceinline__ float2 qpair(int p) {
    const float4 t = metaq(p >> 1);
    return (p & 1) ? make_float2(t.z, t.w) : make_float2(t.x, t.y);
  }
  static __device__ __forceinline__ float cmax2() { return metaq(4).x; }
  static __device__ __forceinline__ uint32_t uniq() { return __float_as_uint(metaq(4).y); }
  static __device__ __forceinline__ bool bad() { return __float_as_uint(metaq(4).z) != 0; }
};

// ---------------------------------------------------------------- helpers --

int g_sm_count[kMaxDevices];

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (!g_sm_count[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    g_sm_count[dev] = v;
  }
  return g_sm_count[dev];
}

uint32_t grid_for(uint64_t items, int per_sm = 8) {
  const uint64_t want = (items + kThreads - 1) / kThreads;
  const uint64_t cap = uint64_t(sm_count()) * per_sm;
  return uint32_t(std::max<uint64_t>(1, std::min(want, cap)));
}

template <typename Kernel>
int resident_per_sm(Kernel k, size_t smem, int threads = kThreads) {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, threads, smem) != cudaSuccess || n < 1) n = 1;
  return n;
}

template <template <int> class F, typename... Args>
cudaError_t by_group(uint32_t g, Args&&... args) {
  switch (g) {
    case 8: return F<8>::run(args...);
    case 16: return F<16>::run(args...);
    default: return F<32>::run(args...);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The current device's ordinal, refused when it is beyond the caches.
cudaError_t current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e == cudaSuccess && (*dev < 0 || *dev >= kMaxDevices)) e = cudaErrorInvalidDevice;
  return e;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// link-time dependency on the driver library); null if unavailable.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace
}  // namespace ack
