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
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "vq_device.cuh"
#include "vq_kernels.hpp"

namespace ack {
namespace {

constexpr int kThreads = 256;

// ------------------------------------------------------------------ decode --

// Warp-cooperative decode, 16-byte aligned output. A warp step covers 256
// vectors: lane l loads code word l of the step (one coalesced 128-byte line,
// prefetched a step ahead) and writes output quads l + 32 k (each warp store
// a full 512-byte line). The word of quad Q comes by shuffle; its nibble
// position and the quad within the vector depend on the lane only.
template <int G>
__global__ void __launch_bounds__(kThreads) k_decode(const uint32_t* __restrict__ codes,
                                                     const float* __restrict__ book, float* __restrict__ out,
                                                     uint64_t n, uint32_t* __restrict__ status) {
  __shared__ __align__(16) float sb[16 * G];
  for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) sb[i] = book[i];
  __syncthreads();
  if (blockIdx.x == 0) {
    uint32_t bits = 0;
    for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) bits |= finite32(sb[i]) ? 0u : kNonfinite;
    flag_warp(status, bits);
  }
  const float4* sb4 = reinterpret_cast<const float4*>(sb);
  float4* out4 = reinterpret_cast<float4*>(out);
  constexpr uint32_t kQV = G / 4;          // float4 per vector
  constexpr uint32_t kQuads = 256 * kQV;   // quads per warp step
  constexpr uint32_t kPer = kQuads / 32;   // stores per lane per step
  const uint32_t lane = threadIdx.x & 31, qv = lane % kQV;
  const uint64_t nq = n / 4;               // complete quads
  const uint64_t steps = (nq + kQuads - 1) / kQuads, words = ((n + G - 1) / G + 7) / 8;
  const uint64_t warps = uint64_t(gridDim.x) * (blockDim.x / 32);
  uint64_t st = uint64_t(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  auto word = [&](uint64_t step) { return step < steps && step * 32 + lane < words ? __ldg(codes + step * 32 + lane) : 0u; };
  uint32_t cur = word(st);
  for (; st < steps; st += warps) {
    const uint32_t next = word(st + warps);
    const uint64_t q0 = st * kQuads;
    if (q0 + kQuads <= nq) {
#pragma unroll 4
      for (uint32_t k = 0; k < kPer; ++k) {
        const uint32_t Q = lane + 32 * k, v = Q / kQV;
        const uint32_t c = (__shfl_sync(0xffffffffu, cur, v >> 3) >> (4 * (v & 7))) & 15u;
        __stcs(out4 + q0 + Q, sb4[c * kQV + qv]);
      }
    } else {
      for (uint32_t k = 0; k < kPer; ++k) {
        const uint32_t Q = lane + 32 * k, v = Q / kQV;
        const uint32_t c = (__shfl_sync(0xffffffffu, cur, v >> 3) >> (4 * (v & 7))) & 15u;
        if (q0 + Q < nq) __stcs(out4 + q0 + Q, sb4[c * kQV + qv]);
      }
    }
    cur = next;
  }
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {  // the values after the last complete quad
    const uint64_t i = nq * 4 + threadIdx.x;
    out[i] = sb[code_at(codes, i / G) * G + uint32_t(i % G)];
  }
}

template <int G>
__global__ void __launch_bounds__(kThreads) k_decode_scalar(const uint32_t* __restrict__ codes,
                                                            const float* __restrict__ book, float* __restrict__ out,
                                                            uint64_t n, uint32_t* __restrict__ status) {
  __shared__ float sb[16 * G];
  for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) sb[i] = book[i];
  __syncthreads();
  if (blockIdx.x == 0) {
    uint32_t bits = 0;
    for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) bits |= finite32(sb[i]) ? 0u : kNonfinite;
    flag_warp(status, bits);
  }
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = sb[code_at(codes, i / G) * G + uint32_t(i % G)];
}

// ------------------------------------------------------------------ encode --

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

// Book staging area: the launcher's staging kernel writes the
// pair-interleaved image of a slot's books and their BookMeta here, then
// the stream copies it into the slot's constant bank.
__device__ __align__(16) float g_stage[kBookSlots][kSlotFloats];

// Stage `nb` row-major 16 x G books from `src` for slot `slot`: warp b writes
// book b pair-interleaved into g_stage[slot] and its BookMeta after the
// books (the slot layout CBook reads).
template <int G>
__global__ void k_stage_books(const float* __restrict__ src, int nb, int slot) {
  __shared__ BookMeta m[3];
  const int b = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (b >= nb) return;
  const float* book = src + b * 16 * G;
  float* dst = g_stage[slot] + b * 16 * G;
  for (int i = lane; i < 16 * G; i += 32) dst[book_pos<G>(i / G, i % G)] = book[i];
  meta_compute<G>(book, m[b]);
  __syncwarp();
  constexpr int kWords = sizeof(BookMeta) / 4;
  uint32_t* meta = reinterpret_cast<uint32_t*>(g_stage[slot] + kSlotBookFloats + b * kMetaFloats);
  if (lane < kWords) meta[lane] = reinterpret_cast<const uint32_t*>(&m[b])[lane];
}

// One encode step of a warp: 32 consecutive vectors from `base` (one per
// lane; `xr` holds the lane's complete vector), nibbles packed into 4 words
// with shuffles.
template <int G, int SLOT>
__device__ __forceinline__ void enc_step(const float* __restrict__ x, uint64_t n, uint64_t base,
                                         const float (&xr)[G], uint32_t* __restrict__ codes,
                                         uint32_t* __restrict__ status) {
  using Book = CBook<G, SLOT, 0>;
  const uint64_t vectors = (n + G - 1) / G, full = n / G, words = (vectors + 7) / 8;
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t v = base + lane;
  uint32_t idx = 0, bits = 0;
  if (v < full) {
    bool certified;
    const float* src = x + v * G;
    idx = enc_vector<G, Book>(xr, &certified, src);
    if (certified) {
      // the rare path: nonfinite values are flagged here, not on every
      // vector (read again from memory: the registers are free by now)
      for (int j = 0; j < G; ++j) bits |= finite32(src[j]) ? 0u : kNonfinite;
    }
  } else if (v < vectors) {
    // The partial last vector: compare its valid components only (vq.py:171-172).
    const int valid = int(n - v * G);
    const float* src = x + v * G;
    for (int j = 0; j < valid; ++j) bits |= finite32(src[j]) ? 0u : kNonfinite;
    idx = enc_exact_mem<G, Book>(src, valid, 0xffffu);
  }
  const uint32_t w = pack_nibbles(idx);
  const uint64_t word = (base >> 3) + (lane >> 3);
  if ((lane & 7) == 0 && word < words) codes[word] = w;
  flag_warp(status, bits);
}

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

// A persistent grid; each warp takes 32 consecutive vectors per step. The
// next step's vectors are loaded into registers while the current ones are
// filtered (two buffers, used in turn). VEC: x is 16-byte aligned.
template <int G, int SLOT, bool VEC>
__global__ void __launch_bounds__(kThreads, encode_min_blocks<G>()) k_encode(const float* __restrict__ x, uint64_t n,
                                                                             uint32_t* __restrict__ codes,
                                                                             uint32_t* __restrict__ status) {
  using Book = CBook<G, SLOT, 0>;
  if (blockIdx.x == 0 && threadIdx.x == 0 && Book::bad()) atomicOr(status, kNonfinite);
  const uint64_t vectors = (n + G - 1) / G, full = n / G;
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t stride = uint64_t(gridDim.x) * (blockDim.x / 32) * 32;
  uint64_t base = (uint64_t(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32) * 32;
  float xa[G], xb[G];
  enc_load<G, VEC>(x, base + lane, full, xa);
  for (; base < vectors; base += 2 * stride) {
    enc_load<G, VEC>(x, base + stride + lane, full, xb);
    enc_step<G, SLOT>(x, n, base, xa, codes, status);
    if (base + stride >= vectors) break;
    enc_load<G, VEC>(x, base + 2 * stride + lane, full, xa);
    enc_step<G, SLOT>(x, n, base + stride, xb, codes, status);
  }
}

// Group 32 with 16-byte aligned x: each warp step copies its 32 vectors
// (4 KB, contiguous) into a per-warp shared buffer with cp.async, 16 bytes
// per lane per instruction, double-buffered; quad L of a step sits at
// L ^ ((L >> 3) & 7), so both the copy and each lane's read of its own
// vector are free of bank conflicts. Fully coalesced global reads and no
// registers held for the prefetch.
__device__ __forceinline__ uint32_t enc_swizzle(uint32_t L) { return L ^ ((L >> 3) & 7u); }

template <int G, int SLOT>
__global__ void __launch_bounds__(kThreads, 3) k_encode_async(const float* __restrict__ x, uint64_t n,
                                                              uint32_t* __restrict__ codes,
                                                              uint32_t* __restrict__ status) {
  using Book = CBook<G, SLOT, 0>;
  constexpr int kQuads = 8 * G;  // 16-byte quads per warp step
  extern __shared__ __align__(16) float4 sx[];  // [warps][2][kQuads]
  if (blockIdx.x == 0 && threadIdx.x == 0 && Book::bad()) atomicOr(status, kNonfinite);
  const uint64_t vectors = (n + G - 1) / G, full = n / G;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x / 32;
  float4* buf0 = sx + size_t(warp) * 2 * kQuads;
  const uint64_t stride = uint64_t(gridDim.x) * (blockDim.x / 32) * 32;
  const uint64_t quads_full = full * (G / 4);
  uint64_t base = (uint64_t(blockIdx.x) * (blockDim.x / 32) + warp) * 32;
  auto issue = [&](uint64_t b, float4* buf) {
    const uint64_t q0 = b * (G / 4);
#pragma unroll
    for (int k = 0; k < G / 4; ++k) {
      const uint32_t L = lane + 32 * k;
      if (q0 + L < quads_full) {  // complete vectors only; the tail is read directly
        const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(buf + enc_swizzle(L)));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(x + (q0 + L) * 4) : "memory");
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (base < vectors) issue(base, buf0);
  for (int s = 0; base < vectors; base += stride, s ^= 1) {
    const float4* cur = buf0 + s * kQuads;
    if (base + stride < vectors) issue(base + stride, buf0 + (s ^ 1) * kQuads);
    else asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncwarp();
    float xr[G];
#pragma unroll
    for (int q = 0; q < G / 4; ++q) {
      const float4 t = cur[enc_swizzle(lane * (G / 4) + q)];
      xr[4 * q] = t.x;
      xr[4 * q + 1] = t.y;
      xr[4 * q + 2] = t.z;
      xr[4 * q + 3] = t.w;
    }
    __syncwarp();  // every lane holds its vector before the buffer is refilled
    enc_step<G, SLOT>(x, n, base, xr, codes, status);
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// ------------------------------------------------ encode on the tensor cores --
//
// k_encode_tc: the FP32 filter of enc_vector moved onto tcgen05. A producer
// warp streams tiles of 128 H vectors (raw FP32, TMA-swizzled into the UMMA
// K-major layout) into an S-stage ring; one thread issues
// tcgen05.mma.kind::tf32 of each 128-vector sub-tile against the book
// (rounded to tf32) into TMEM; C consumer quads (quad q owns the block's
// tiles k = q mod C and its own accumulator columns) read the 16 dot
// products of each vector with tcgen05.ld and certify the nearest entry.
//
// Certificate. The tensor core uses the top 19 bits of each x component
// (|x - x'| < 2^-10 |x|), the book is rounded to tf32 (2^-11), products are
// exact and accumulate in FP32. With f_e = ||c_e||^2 - 2 x.c_e and
// sum_j |x_j c_j| <= (||x||^2 + max ||c||^2) / 2, the computed f'_e obeys
// |f'_e - f_e| <= eps1 = kappa1 (||x||^2 + max ||c||^2) + 2^-118 with
// kappa1 = 2^-10 + 2^-11 + (G + 8) 2^-21 (the last term covers the FP32
// accumulation and the final fused multiply-add; the absolute floor covers
// flushed subnormal products). The float64 winner lies in
// {e : f'_e <= min f' + 2 eps1} minus duplicate rows; one entry left is the
// answer. Otherwise (a few per cent of vectors on smooth data) the vector
// joins its warp's queue and is refined later: the FP32 filter of enc_vector
// (its bound kappa2 = (G + 8) 2^-23) over those candidates only, then the
// float64 pass over what survives, the result OR-ed into the zero nibble the
// first pass stored. Nonfinite input or books take the float64 pass at once.
//
// Group 32 tightens the bound (Cfg::TIGHT, Cfg::RESID): the book enters as
// tf32 hi and lo halves (N = 32, summed), so only x is truncated, and that
// error is bounded by 2 ||x - trunc(x)|| max ||c|| (Cauchy-Schwarz; the
// tensor core's operand is trunc(x) or its nearer tf32 neighbour, so the
// residual is at most this) plus (g + 9) 2^-21 (||x||^2 + max ||c||^2) +
// 2^-118 for accumulation, the book remainder, rounding and flushed
// subnormals. That leaves about a quarter of the near ties.
//
// Every wait on an mbarrier is bounded; one that runs out sets kStalled and
// the block drains its own copies and returns.
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// FP32 -> tf32, round to nearest (ties away), as cvt.rna.tf32.f32.
__device__ __forceinline__ float tf32_rna(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return __uint_as_float(r);
}

// The UMMA K-major swizzle matching the TMA swizzle of a G-float row
// (32/64/128-byte rows: SWIZZLE_32B/64B/128B; 16-byte chunk bits [4,7)
// XOR-ed with row-group bits [7,10)).
template <int G>
struct Swz {
  static constexpr uint32_t kRow = G * 4;
  static constexpr uint32_t kMask = G == 8 ? 1u : (G == 16 ? 3u : 7u);
  static constexpr uint64_t kLayout = G == 8 ? 6u : (G == 16 ? 4u : 2u);  // descriptor layout type
  // byte offset of 16-byte chunk `kc` of row `r` in a 1024-byte aligned tile
  static __device__ __forceinline__ uint32_t off(uint32_t r, uint32_t kc) {
    const uint32_t l = r * kRow + kc * 16u;
    return l ^ (((l >> 7) & kMask) << 4);
  }
  // shared-memory matrix descriptor: start >> 4, leading byte offset 16 (unused
  // by swizzled K-major), stride byte offset = 8 rows, version 1, layout type
  static __device__ __forceinline__ uint64_t desc(uint32_t addr) {
    return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(((8u * kRow) >> 4) & 0x3FFFu) << 32) |
           (uint64_t(1) << 46) | (kLayout << 61);
  }
};

// Instruction descriptor: D FP32, A and B tf32, both K-major, N = 16, M = 128.
constexpr uint32_t kIdescM128N16 = (1u << 4) | (2u << 7) | (2u << 10) | ((16u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescM128N32 = (1u << 4) | (2u << 7) | (2u << 10) | ((32u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void mb_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mb_arrive(uint64_t* b) {
  asm volatile("{ .reg .b64 t; mbarrier.arrive.shared::cta.b64 t, [%0]; }" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mb_expect(uint64_t* b, uint32_t bytes) {
  asm volatile("{ .reg .b64 t; mbarrier.arrive.expect_tx.shared::cta.b64 t, [%0], %1; }" ::"r"(smem_u32(b)),
               "r"(bytes)
               : "memory");
}
// Wait for the phase of parity `parity` to complete; false after ~2^22 polls
// (each poll suspends for a hardware-chosen interval), never an endless spin.
__device__ __forceinline__ bool mb_wait(uint64_t* b, uint32_t parity) {
  for (uint32_t it = 0; it < (1u << 22); ++it) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

// Stages S, consumer quads C, sub-tiles of 128 vectors per tile H (one TMA
// box holds at most 256 rows). Measured on B200 for 2^30 values.
// TIGHT: the book as tf32 hi and lo halves (N = 32 columns, the two summed);
// RESID: the measured truncation residual of x in the bound instead of its
// worst case. Both pay on g32 (4.7% near ties on smooth data otherwise);
// on g16 and g8, with 2x and 4x the vectors per byte, the extra work per
// vector measured slower than the refinements it saves.
template <int G>
struct Cfg {
  static constexpr int S = 4, C = 2, H = G == 8 ? 4 : (G == 16 ? 2 : 1);
  static constexpr bool TIGHT = G == 32, RESID = G == 32;
  static constexpr uint32_t kN = TIGHT ? 32u : 16u;  // accumulator columns per sub-tile
  static constexpr int kThreads = 128 * C + 64, kBlocksPerSm = 2;
  static constexpr uint32_t kSub = 128u * G * 4u, kTile = kSub * H;
  static constexpr uint32_t kBoxRows = H > 2 ? 256u : 128u * H;
  static constexpr uint32_t kCols = C * H * kN <= 32 ? 32u : (C * H * kN <= 64 ? 64u : 128u);
  static constexpr uint32_t kCap = H == 1 ? 64u : (H == 2 ? 128u : 256u);  // >= 31 + 32 H: a tile never overflows it
  // dynamic shared memory: 1024-byte alignment slack, the ring, the tf32
  // book tile (kN rows, at most 4 KB), the FP32 book and its 16 squared norms
  static constexpr size_t kSmem = 1024 + size_t(S) * kTile + 4096 + 16 * G * 4 + 64;
};

// Deferred FP32 refinement of `count` (<= 32) queued vectors, one per lane,
// ring positions head + lane: x read again from memory, the FP32 filter of
// enc_vector over the tf32 candidates, the float64 pass if more than one
// survives; the index is OR-ed into the zero nibble the filter pass stored.
template <int G, class Book, uint32_t kCap>
__device__ __noinline__ void refine_queue(const float* __restrict__ x, uint32_t* __restrict__ codes,
                                          const uint64_t* qv, const uint32_t* qc, uint32_t head, uint32_t count,
                                          const float* sbk, const float* sq, uint32_t lane) {
  constexpr float kappa2 = float(G + 8) / 8388608.0f;
  __syncwarp();  // the nibble stores of the filter pass come first
  if (lane < count) {
    const uint32_t i = (head + lane) & (kCap - 1);
    const uint64_t v = qv[i];
    const uint32_t cand = qc[i];
    const float4* src = reinterpret_cast<const float4*>(x + v * G);
    float xr[G];
    float2 n2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int kc = 0; kc < G / 4; ++kc) {
      const float4 t = __ldg(src + kc);
      xr[4 * kc] = t.x;
      xr[4 * kc + 1] = t.y;
      xr[4 * kc + 2] = t.z;
      xr[4 * kc + 3] = t.w;
      n2 = __ffma2_rn(make_float2(t.x, t.y), make_float2(t.x, t.y), n2);
      n2 = __ffma2_rn(make_float2(t.z, t.w), make_float2(t.z, t.w), n2);
    }
    const float scale = n2.x + n2.y + Book::cmax2();
    const float inf = __int_as_float(0x7f800000);
    float f[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) f[e] = inf;
    float fb = inf;
    for (uint32_t m = cand; m; m &= m - 1u) {
      const int e = __ffs(m) - 1;
      const float* ce = sbk + e * G;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
      for (int kc = 0; kc < G / 4; ++kc) {
        const float4 c4 = *reinterpret_cast<const float4*>(ce + 4 * kc);
        a0 = fmaf(xr[4 * kc], c4.x, a0);
        a1 = fmaf(xr[4 * kc + 1], c4.y, a1);
        a2 = fmaf(xr[4 * kc + 2], c4.z, a2);
        a3 = fmaf(xr[4 * kc + 3], c4.w, a3);
      }
      const float fe = fmaf(-2.f, (a0 + a1) + (a2 + a3), sq[e]);
      fb = fminf(fb, fe);
#pragma unroll
      for (int t = 0; t < 16; ++t) f[t] = t == e ? fe : f[t];
    }
    const float thr = fmaf(2.f, fmaf(kappa2, scale, 1e-37f), fb);
    uint32_t c2 = 0;
#pragma unroll
    for (int e = 0; e < 16; ++e) c2 |= uint32_t(f[e] <= thr) << e;
    c2 &= cand;
    uint32_t idx;
    if (finite32(thr) && c2 != 0u && (c2 & (c2 - 1u)) == 0u)
      idx = uint32_t(__ffs(c2) - 1);
    else
      idx = enc_exact_mem<G, Book>(x + v * G, G, finite32(thr) && c2 ? c2 : cand);
    if (idx) atomicOr(codes + v / 8, idx << (4 * uint32_t(v % 8)));
  }
  __syncwarp();
}

}  // namespace tc

template <int G, int SLOT>
__global__ void __launch_bounds__(tc::Cfg<G>::kThreads, tc::Cfg<G>::kBlocksPerSm)
    k_encode_tc(const __grid_constant__ CUtensorMap tmap, const float* __restrict__ x, uint64_t n,
                uint32_t* __restrict__ codes, uint32_t* __restrict__ status) {
  using Book = CBook<G, SLOT, 0>;
  using W = tc::Swz<G>;
  using K = tc::Cfg<G>;
  constexpr int S = K::S, C = K::C, H = K::H, kChunks = G / 4;
  constexpr uint32_t kCap = K::kCap;
  extern __shared__ unsigned char tc_smem[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem) + 1023) & ~uintptr_t(1023));
  unsigned char* ring = base;
  unsigned char* bmat = base + S * K::kTile;             // 16 tf32 book rows, swizzled
  float* sbk = reinterpret_cast<float*>(bmat + 4096);    // the FP32 book, row-major
  float* sq = sbk + 16 * G;                               // its 16 squared norms
  __shared__ __align__(8) uint64_t full[S], sfree[S], done[C], afree[C];
  __shared__ uint32_t tmem_base;
  __shared__ uint64_t q_vec[4 * C][kCap];
  __shared__ uint32_t q_cand[4 * C][kCap];
  const uint32_t tid = threadIdx.x, warp = tid / 32, lane = tid & 31;
  const uint64_t vectors = (n + G - 1) / G, complete = n / G, words = (vectors + 7) / 8;
  const uint64_t tiles = (vectors + 128 * H - 1) / (128 * H);
  const uint32_t T = tiles > blockIdx.x ? uint32_t((tiles - blockIdx.x + gridDim.x - 1) / gridDim.x) : 0u;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_u32(&tmem_base)),
                 "r"(K::kCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      tc::mb_init(&full[s], 1);
      tc::mb_init(&sfree[s], 128 + 1);  // the owning quad's reads and the MMA's completion
    }
    for (int b = 0; b < C; ++b) {
      tc::mb_init(&done[b], 1);
      tc::mb_init(&afree[b], 128);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (tid < 16 * kChunks) {
    const uint32_t e = tid / kChunks, kc = tid % kChunks;
    float c[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) c[i] = Book::at(int(e), int(kc * 4 + i));
    float hi[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) hi[i] = tc::tf32_rna(c[i]);
    *reinterpret_cast<float4*>(bmat + W::off(e, kc)) = make_float4(hi[0], hi[1], hi[2], hi[3]);
    if constexpr (K::TIGHT)  // rows 16..31: the tf32 remainder, c - hi exact in FP32
      *reinterpret_cast<float4*>(bmat + W::off(16 + e, kc)) =
          make_float4(tc::tf32_rna(c[0] - hi[0]), tc::tf32_rna(c[1] - hi[1]), tc::tf32_rna(c[2] - hi[2]),
                      tc::tf32_rna(c[3] - hi[3]));
    *reinterpret_cast<float4*>(sbk + e * G + kc * 4) = make_float4(c[0], c[1], c[2], c[3]);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor core
  }
  if (tid < 4) *reinterpret_cast<float4*>(sq + 4 * tid) = Book::metaq(int(tid));
  if (blockIdx.x == 0 && tid == 0 && Book::bad()) atomicOr(status, kNonfinite);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  bool ok = true;

  if (warp == 4 * C) {
    // producer: one TMA tensor load (two for 512-row tiles) per tile
    if (lane == 0) {
      uint32_t issued = 0;
      for (uint32_t k = 0; k < T && ok; ++k) {
        const uint32_t s = k % S;
        if (k >= S && !(ok = tc::mb_wait(&sfree[s], ((k / S) - 1) & 1))) break;
        ++issued;
        tc::mb_expect(&full[s], K::kTile);
        const int32_t row = int32_t((blockIdx.x + uint64_t(k) * gridDim.x) * 128 * H);
#pragma unroll
        for (int part = 0; part < (H > 2 ? H / 2 : 1); ++part)
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
                  "r"(tc::smem_u32(ring + s * K::kTile + part * 2 * K::kSub)),
              "l"(&tmap), "r"(0), "r"(row + part * 256), "r"(tc::smem_u32(&full[s]))
              : "memory");
      }
      if (!ok) atomicOr(status, kStalled);
      // the loads in flight land before the block may exit
      for (uint32_t k = issued > uint32_t(S) ? issued - S : 0u; k < issued; ++k)
        if (!tc::mb_wait(&full[k % S], (k / S) & 1)) atomicOr(status, kStalled);
    }
  } else if (warp == 4 * C + 1) {
    // MMA issuer
    if (lane == 0) {
      const uint32_t b_addr = tc::smem_u32(bmat);
      for (uint32_t k = 0; k < T && ok; ++k) {
        const uint32_t s = k % S, q = k % C;
        if (!(ok = tc::mb_wait(&full[s], (k / S) & 1))) break;
        if (k >= C && !(ok = tc::mb_wait(&afree[q], ((k / C) - 1) & 1))) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (int h = 0; h < H; ++h) {
          const uint32_t d = tmem + (q * H + h) * K::kN;
          const uint32_t a = tc::smem_u32(ring + s * K::kTile + h * K::kSub);
#pragma unroll
          for (int ks = 0; ks < G / 8; ++ks)
            asm volatile(
                "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p; }" ::"r"(d),
                "l"(W::desc(a + ks * 32u)), "l"(W::desc(b_addr + ks * 32u)),
                "r"(K::TIGHT ? tc::kIdescM128N32 : tc::kIdescM128N16), "r"(uint32_t(ks))
                : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         tc::smem_u32(&done[q]))
                     : "memory");
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         tc::smem_u32(&sfree[s]))
                     : "memory");
      }
      if (!ok) atomicOr(status, kStalled);
      // the last MMAs complete before TMEM is released
      for (uint32_t k = T > uint32_t(C) ? T - C : 0u; ok && k < T; ++k)
        if (!tc::mb_wait(&done[k % C], (k / C) & 1)) atomicOr(status, kStalled);
    }
  } else {
    // consumer quad q: TMEM lanes 32 (warp % 4) .. + 31, one vector per lane per sub-tile
    const uint32_t q = warp / 4, row = tid & 127, wq = warp & 3;
    constexpr float kappa1 = 1.0f / 1024 + 1.0f / 2048 + float(G + 8) / 2097152.0f;
    constexpr float kappa_t = float(G + 9) / 2097152.0f;  // TIGHT: all but the x residual
    uint32_t qhead = 0, qtail = 0;
    for (uint32_t k = q; k < T && ok; k += C) {
      const uint32_t s = k % S;
      if (!(ok = tc::mb_wait(&full[s], (k / S) & 1))) break;
      if (!(ok = tc::mb_wait(&done[q], (k / C) & 1))) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll(G == 8 ? 2 : 1)
      for (int h = 0; h < H; ++h) {
        uint32_t r[K::kN];
        const uint32_t taddr = tmem + ((wq * 32u) << 16) + (q * H + h) * K::kN;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(taddr));
        if constexpr (K::TIGHT)
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
              : "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
                "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
                "=r"(r[30]), "=r"(r[31])
              : "r"(taddr + 16u));
        // ||x||^2 in enc_vector's order, from the swizzled tile (conflict-free);
        // TIGHT also ||x - trunc(x)||^2, x truncated to its top 19 bits: the
        // tensor core's operand is that or the nearer tf32 neighbour, so this
        // bounds its residual either way
        const unsigned char* tile = ring + s * K::kTile + h * K::kSub;
        float2 n2 = make_float2(0.f, 0.f), r2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int kc = 0; kc < kChunks; ++kc) {
          const float4 t = *reinterpret_cast<const float4*>(tile + W::off(row, kc));
          n2 = __ffma2_rn(make_float2(t.x, t.y), make_float2(t.x, t.y), n2);
          n2 = __ffma2_rn(make_float2(t.z, t.w), make_float2(t.z, t.w), n2);
          if constexpr (K::RESID) {
            const float2 a = make_float2(t.x - __uint_as_float(__float_as_uint(t.x) & 0xFFFFE000u),
                                         t.y - __uint_as_float(__float_as_uint(t.y) & 0xFFFFE000u));
            const float2 b = make_float2(t.z - __uint_as_float(__float_as_uint(t.z) & 0xFFFFE000u),
                                         t.w - __uint_as_float(__float_as_uint(t.w) & 0xFFFFE000u));
            r2 = __ffma2_rn(a, a, r2);
            r2 = __ffma2_rn(b, b, r2);
          }
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if constexpr (K::TIGHT) {
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            const float2 t = __fadd2_rn(make_float2(__uint_as_float(r[e]), __uint_as_float(r[e + 1])),
                                        make_float2(__uint_as_float(r[16 + e]), __uint_as_float(r[17 + e])));
            r[e] = __float_as_uint(t.x);
            r[e + 1] = __float_as_uint(t.y);
          }
        }
        const uint64_t vbase = (blockIdx.x + uint64_t(k) * gridDim.x) * 128 * H + h * 128;
        const uint64_t v = vbase + row;
        uint32_t idx = 0, bits = 0, cand = 0;
        bool defer = false;
        if (v < complete) {
          float f[16];
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            const float2 t = __ffma2_rn(make_float2(-2.f, -2.f),
                                        make_float2(__uint_as_float(r[2 * p]), __uint_as_float(r[2 * p + 1])),
                                        Book::qpair(p));
            f[2 * p] = t.x;
            f[2 * p + 1] = t.y;
          }
          float lo[8];
#pragma unroll
          for (int p = 0; p < 8; ++p) lo[p] = fminf(f[2 * p], f[2 * p + 1]);
#pragma unroll
          for (int w = 4; w; w >>= 1)
#pragma unroll
            for (int p = 0; p < w; ++p) lo[p] = fminf(lo[p], lo[p + w]);
          const float fb = lo[0];
          float eps;
          if constexpr (K::TIGHT && !K::RESID) {
            // x truncated (2^-10) against the exactly represented book
            eps = fmaf(1.0f / 1024 + kappa_t, n2.x + n2.y + Book::cmax2(), 0x1p-118f);
          } else if constexpr (K::RESID) {
            // 2 ||r|| max||c|| (rounded up, 2^-16 margin for the FP32 sum of
            // squares) + the accumulation, book-remainder, rounding and
            // flushed-subnormal terms
            const float rc = __fsqrt_ru(__fmul_ru(r2.x + r2.y, Book::cmax2()));
            eps = fmaf(2.0f + 0x1p-15f, rc, fmaf(kappa_t, n2.x + n2.y + Book::cmax2(), 0x1p-118f));
          } else {
            eps = fmaf(kappa1, n2.x + n2.y + Book::cmax2(), 0x1p-118f);
          }
          const float thr = fmaf(2.f, eps, fb);
#pragma unroll
          for (int e = 0; e < 16; ++e) cand |= uint32_t(f[e] <= thr) << e;
          cand &= Book::uniq();
          const bool clean = finite32(thr) && finite32(fb) && !Book::bad();
          if (clean && cand != 0u && (cand & (cand - 1u)) == 0u) {
            idx = uint32_t(__ffs(cand) - 1);
          } else if (clean && cand != 0u) {
            defer = true;
          } else {
            const float* src = x + v * G;
            for (int j = 0; j < G; ++j) bits |= finite32(src[j]) ? 0u : kNonfinite;
            idx = enc_exact_mem<G, Book>(src, G, clean ? cand : 0xffffu);
          }
        } else if (v < vectors) {
          // the partial last vector: its valid components only (vq.py:171-172)
          const int valid = int(n - v * G);
          const float* src = x + v * G;
          for (int j = 0; j < valid; ++j) bits |= finite32(src[j]) ? 0u : kNonfinite;
          idx = enc_exact_mem<G, Book>(src, valid, 0xffffu);
        }
        const uint32_t dm = __ballot_sync(0xffffffffu, defer);
        if (defer) {
          const uint32_t pos = (qtail + __popc(dm & ((1u << lane) - 1u))) & (kCap - 1);
          q_vec[warp][pos] = v;
          q_cand[warp][pos] = cand;
        }
        qtail += __popc(dm);
        const uint32_t w = pack_nibbles(idx);
        const uint64_t word = (vbase + wq * 32) / 8 + lane / 8;
        if ((lane & 7) == 0 && word < words) codes[word] = w;
        flag_warp(status, bits);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      tc::mb_arrive(&afree[q]);
      tc::mb_arrive(&sfree[s]);
      // refine off the pipeline's critical path, 32 vectors at a time
      while (qtail - qhead >= 32u) {
        tc::refine_queue<G, Book, kCap>(x, codes, q_vec[warp], q_cand[warp], qhead, 32u, sbk, sq, lane);
        qhead += 32u;
      }
    }
    if (ok && qtail != qhead)
      tc::refine_queue<G, Book, kCap>(x, codes, q_vec[warp], q_cand[warp], qhead, qtail - qhead, sbk, sq, lane);
    if (!ok) atomicOr(status, kStalled);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(K::kCols));
}

// ------------------------------------------- shader-exact packed-pair matmul --

template <int G>
__device__ __forceinline__ float dequant(const uint32_t* __restrict__ codes, const float* __restrict__ book,
                                         uint64_t logical) {
  return __ldg(book + code_at(codes, logical / G) * G + uint32_t(logical % G));
}

// C[M,N] = sum over inner of fl32(a*b) with separately rounded adds, k in
// order (vq4.comp:165-176). Flag bit 0: A stored K x M; bit 1: B stored N x K.
template <int G>
__global__ void __launch_bounds__(kThreads) k_matmul_exact(const uint32_t* __restrict__ ac,
                                                           const float* __restrict__ ab,
                                                           const uint32_t* __restrict__ bc,
                                                           const float* __restrict__ bb, float* __restrict__ c,
                                                           uint32_t M, uint32_t N, uint32_t K, uint32_t flags,
                                                           uint32_t* __restrict__ status) {
  constexpr int T = 64, KC = 16;
  __shared__ float As[KC][T + 1];
  __shared__ float Bs[KC][T + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const uint32_t row0 = blockIdx.y * T, col0 = blockIdx.x * T;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  if (blockIdx.x == 0 && blockIdx.y == 0) {
    uint32_t bits = 0;
    for (int i = threadIdx.x; i < 16 * G; i += blockDim.x)
      bits |= (finite32(ab[i]) && finite32(bb[i])) ? 0u : kNonfinite;
    flag_warp(status, bits);
  }
  for (uint32_t k0 = 0; k0 < K; k0 += KC) {
    for (int i = threadIdx.x; i < KC * T; i += blockDim.x) {
      const int kk = i / T, rr = i % T;
      const uint32_t k = k0 + kk, row = row0 + rr, col = col0 + rr;
      float a = 0.f, b = 0.f;
      if (k < K && row < M) a = dequant<G>(ac, ab, (flags & 1u) ? uint64_t(k) * M + row : uint64_t(row) * K + k);
      if (k < K && col < N) b = dequant<G>(bc, bb, (flags & 2u) ? uint64_t(col) * K + k : uint64_t(k) * N + col);
      As[kk][rr] = a;
      Bs[kk][rr] = b;
    }
    __syncthreads();
    const int kmax = min(KC, int(K - k0));
    for (int kk = 0; kk < kmax; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
    }
    __syncthreads();
  }
  uint32_t bits = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t row = row0 + ty * 4 + i, col = col0 + tx * 4 + j;
      if (row < M && col < N) {
        c[uint64_t(row) * N + col] = acc[i][j];
        // a nonfinite product or partial sum leaves the total nonfinite
        bits |= finite32(acc[i][j]) ? 0u : kNonfinite;
      }
    }
  flag_warp(status, bits);
}

// ------------------------------------------------------------------- AdamW --

__device__ __forceinline__ float state_value(const uint32_t* __restrict__ codes, const float* __restrict__ books,
                                             uint64_t words, int state, uint32_t group, uint64_t i) {
  const uint64_t v = i / group;
  const uint32_t code = code_at(codes + state * words, v);
  return books[state * 16 * group + code * group + uint32_t(i % group)];
}

// vq4.comp op 3: b0 = [W, M, V, G] packed images, b1 = their four books,
// b2 = seven coefficients; out = [W', M', V'] dense FP32.
__global__ void __launch_bounds__(kThreads) k_adamw(const uint32_t* __restrict__ codes,
                                                    const float* __restrict__ books,
                                                    const float* __restrict__ coefs, float* __restrict__ out,
                                                    uint32_t n, uint32_t group, uint32_t* __restrict__ status) {
  __shared__ float sbooks[4 * 16 * 32];
  for (int i = threadIdx.x; i < 64 * int(group); i += blockDim.x) sbooks[i] = books[i];
  __syncthreads();
  const AdamwCoefs k = load_coefs(coefs);
  if (blockIdx.x == 0) {
    uint32_t bits = 0;
    for (int i = threadIdx.x; i < 64 * int(group); i += blockDim.x) bits |= finite32(sbooks[i]) ? 0u : kNonfinite;
    flag_warp(status, bits);
  }
  const uint64_t words = (uint64_t(n) + group - 1) / group;
  const uint64_t wpad = (words + 7) / 8;
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    uint32_t bits = k.status;
    if (!bits) {
      const float w = state_value(codes, sbooks, wpad, 0, group, i);
      const float m = state_value(codes, sbooks, wpad, 1, group, i);
      const float v = state_value(codes, sbooks, wpad, 2, group, i);
      const float g = state_value(codes, sbooks, wpad, 3, group, i);
      float nw, nm, nv;
      bool skip;
      bits = adamw_value(k, w, m, v, g, &nw, &nm, &nv, &skip);
      if (!skip) {
        out[i] = nw;
        out[uint64_t(n) + i] = nm;
        out[2 * uint64_t(n) + i] = nv;
      }
    }
    if (bits) atomicOr(status, bits);
  }
}

// ------------------------------------------------ dense X times coded W^T --

// Y[b] = X[b] decode(W[b])^T with W stored N x K, vectors along K, K % G == 0.
//
// Per (rows of X, t-chunk of TC groups) a block builds the table
// P[m][t][e] = x[m, tG:tG+G] . c_e in shared memory; then each thread owns
// one row n of W and adds P[m][t][idx(n, t)] over the chunk: one lookup and
// one add per (row, group). The rows' codes arrive by cp.async into padded
// shared rows (conflict-free 16-byte reads), double-buffered. Nibbles are
// turned into byte offsets four at a time ((w << 2) & 0x3C3C3C3C holds 4*idx
// of the even nibbles, (w >> 2) & 0x3C3C3C3C of the odd ones) and extracted
// with one byte permute each; with TC a template constant every table offset
// is an immediate, so a lookup is one permute, one shared load and one add.
// A block works on `items_per_expert`-th of one expert's rows.
template <int G, int MC, int TC>
__global__ void __launch_bounds__(kThreads, 2) k_dense_lut(const float* __restrict__ X,
                                                           const uint32_t* __restrict__ codes,
                                                           const float* __restrict__ books, float* __restrict__ Y,
                                                           uint32_t M, uint32_t N, uint32_t K,
                                                           uint32_t items_per_expert, uint32_t batches_per_item,
                                                           uint64_t words_per_expert, uint32_t* __restrict__ status) {
  constexpr uint32_t kPitch = TC / 2 + 16;  // bytes of one staged row, padded
  constexpr uint32_t kStage = kThreads * kPitch;
  constexpr uint32_t kPieces = TC / 32;     // 16-byte pieces (32 groups) per staged row
  extern __shared__ __align__(16) unsigned char smem[];
  float* P = reinterpret_cast<float*>(smem);                       // [MC][TC][16]
  unsigned char* stage0 = smem + size_t(MC) * TC * 64;             // [2][kThreads][kPitch]
  __shared__ float sbook[16 * G];

  const uint32_t e = blockIdx.x / items_per_expert, part = blockIdx.x % items_per_expert;
  const uint32_t T = K / G;
  const uint32_t nbatches = (N + kThreads - 1) / kThreads;
  const uint32_t b0 = part * batches_per_item, b1 = min(nbatches, b0 + batches_per_item);
  if (b0 >= b1) return;  // the whole block leaves together
  const uint32_t r0 = b0 * kThreads, r1 = min(N, b1 * kThreads);
  const float* Xb = X + uint64_t(e) * M * K;
  const unsigned char* Cb = reinterpret_cast<const unsigned char*>(codes + uint64_t(e) * words_per_expert);
  float* Yb = Y + uint64_t(e) * M * N;
  for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) sbook[i] = books[uint64_t(e) * 16 * G + i];
  __syncthreads();
  if (part == 0) {
    uint32_t bits = 0;
    for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) bits |= finite32(sbook[i]) ? 0u : kNonfinite;
    flag_warp(status, bits);
  }
  const uint32_t nb = (r1 - r0 + kThreads - 1) / kThreads;

  for (uint32_t m0 = 0; m0 < M; m0 += MC) {
    const uint32_t mc = min(uint32_t(MC), M - m0);
    for (uint32_t t0 = 0; t0 < T; t0 += TC) {
      __syncthreads();  // the previous table and stages are no longer read
      for (uint32_t i = threadIdx.x; i < mc * TC; i += blockDim.x) {
        const uint32_t m = i / TC, t = i % TC;
        const float* xs = Xb + uint64_t(m0 + m) * K + uint64_t(t0 + t) * G;
        float xr[G];
#pragma unroll
        for (int j = 0; j < G; ++j) xr[j] = __ldg(xs + j);
        float* dst = P + (size_t(m) * TC + t) * 16;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          float acc = 0.f;
#pragma unroll
          for (int j = 0; j < G; ++j) acc = fmaf(xr[j], sbook[c * G + j], acc);
          dst[c] = acc;
        }
      }
      auto issue = [&](uint32_t batch, uint32_t buf) {
        const uint32_t rb = r0 + batch * kThreads;
        const uint32_t nrows = min(uint32_t(kThreads), r1 - rb);
        for (uint32_t i = threadIdx.x; i < nrows * kPieces; i += blockDim.x) {
          const uint32_t r = i / kPieces, pc = i % kPieces;
          const unsigned char* src = Cb + (uint64_t(rb + r) * T + t0) / 2 + pc * 16;
          const uint32_t saddr =
              static_cast<uint32_t>(__cvta_generic_to_shared(stage0 + buf * kStage + r * kPitch + pc * 16));
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(src));
        }
        asm volatile("cp.async.commit_group;\n" ::);
      };
      issue(0, 0);
      for (uint32_t batch = 0; batch < nb; ++batch) {
        const uint32_t buf = batch & 1;
        if (batch + 1 < nb) {
          issue(batch + 1, buf ^ 1);
          asm volatile("cp.async.wait_group 1;\n" ::);
        } else {
          asm volatile("cp.async.wait_group 0;\n" ::);
        }
        __syncthreads();
        const uint32_t row = r0 + batch * kThreads + threadIdx.x;
        if (row < r1) {
          float acc[MC][4];
#pragma unroll
          for (int m = 0; m < MC; ++m)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[m][q] = 0.f;
          const unsigned char* rowp = stage0 + buf * kStage + threadIdx.x * kPitch;
          const unsigned char* Pb = smem;
#pragma unroll
          for (int pc = 0; pc < int(kPieces); ++pc) {
            const uint4 q4 = *reinterpret_cast<const uint4*>(rowp + pc * 16);
            const uint32_t wd[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
              const uint32_t lo = (wd[wi] << 2) & 0x3C3C3C3Cu;  // 4 * nibbles 0, 2, 4, 6
              const uint32_t hi = (wd[wi] >> 2) & 0x3C3C3C3Cu;  // 4 * nibbles 1, 3, 5, 7
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint32_t olo = __byte_perm(lo, 0, 0x4440 + kk);
                const uint32_t ohi = __byte_perm(hi, 0, 0x4440 + kk);
                const int t = pc * 32 + wi * 8 + 2 * kk;
#pragma unroll
                for (int m = 0; m < MC; ++m) {
                  const unsigned char* pm = Pb + (size_t(m) * TC + t) * 64;
                  acc[m][(2 * kk) & 3] += *reinterpret_cast<const float*>(pm + olo);
                  acc[m][(2 * kk + 1) & 3] += *reinterpret_cast<const float*>(pm + 64 + ohi);
                }
              }
            }
          }
#pragma unroll
          for (int m = 0; m < MC; ++m) {
            if (m < int(mc)) {
              const float y = (acc[m][0] + acc[m][1]) + (acc[m][2] + acc[m][3]);
              float* dst = Yb + uint64_t(m0 + m) * N + row;
              *dst = t0 ? *dst + y : y;
            }
          }
        }
        __syncthreads();  // this stage may be overwritten by the next issue
      }
    }
  }
}

// Repack E canonical N x K images (vectors along K) into the tile32 layout:
// 16-byte unit c of row r goes to ((r / 32) * T/32 + c) * 32 + r % 32; rows
// past N in the last tile become zero codes.
__global__ void __launch_bounds__(kThreads) k_repack_tile32(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                            uint32_t N, uint32_t T, uint64_t src_units,
                                                            uint64_t dst_units, uint32_t batch) {
  const uint32_t ct = T / 32;  // 16-byte units per row
  const uint64_t total = dst_units * batch;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += uint64_t(gridDim.x) * blockDim.x) {
    const uint64_t e = i / dst_units, u = i % dst_units;
    const uint32_t lane = uint32_t(u % 32);
    const uint64_t tc = u / 32;
    const uint32_t c = uint32_t(tc % ct);
    const uint64_t row = (tc / ct) * 32 + lane;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < N) v = __ldg(src + e * src_units + row * ct + c);
    dst[i] = v;
  }
}

// Y[b] = X[b] decode(W[b])^T with W[b] in the tile32 layout. The same table
// and the same per-row lookup order as k_dense_lut (results are bitwise the
// same), but each warp reads its 32 rows' codes as coalesced 512-byte lines
// straight into registers: no shared-memory staging and no barrier inside a
// t-chunk.
//
// Persistent grid: the work units are (expert, 32-row tile), expert-major,
// and block b takes the contiguous range [U b / grid, U (b + 1) / grid), so
// every block gets the same number of tiles to within one whatever the
// expert count. Per expert segment of its range and per (m, t)-chunk a block
// builds the table once: the chunk of X arrives in shared memory in one
// round trip, lane e % 16 holds book row e in registers and a half-warp
// computes the 16 entries of one group.
//
// The table is P[t][m / 2][e][m % 2]: rows of X in pairs side by side per
// entry, so one 8-byte shared load fetches an entry for two rows (a
// half-warp phase of 16 distinct 8-byte entries is conflict-free; 16-byte
// loads measured slower, their quarter-warp phases conflict). The nibble
// masks yield 4 idx (MC = 1) or 8 idx (MC > 1) directly in each byte.
template <int G, int MC, int TC>
__global__ void __launch_bounds__(kThreads, 3) k_dense_t32(const float* __restrict__ X,
                                                           const uint4* __restrict__ codes,
                                                           const float* __restrict__ books, float* __restrict__ Y,
                                                           uint32_t M, uint32_t N, uint32_t K, uint32_t experts,
                                                           uint64_t units_per_expert, uint32_t* __restrict__ status) {
  constexpr int kPieces = TC / 32;
  extern __shared__ __align__(16) unsigned char smem[];
  static_assert(MC == 1 || MC == 2 || MC == 4, "one table load covers MC rows");
  float* P = reinterpret_cast<float*>(smem);  // [TC][MC/2][16][2], or [TC][16] for MC = 1
  float* Xs = P + MC * TC * 16;                // [TC * G]: one row's X chunk
  const uint32_t T = K / G, ct = T / 32;
  const uint32_t ntiles = (N + 31) / 32;
  const uint64_t total = uint64_t(experts) * ntiles;
  const bool x_vec = (reinterpret_cast<uintptr_t>(X) & 15u) == 0;
  const uint64_t u0 = total * blockIdx.x / gridDim.x, u1 = total * (blockIdx.x + 1) / gridDim.x;
  const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (uint64_t s0 = u0; s0 < u1;) {
    const uint32_t e = uint32_t(s0 / ntiles);
    const uint64_t s1 = min(u1, uint64_t(e + 1) * ntiles);
    const uint32_t tl0 = uint32_t(s0 - uint64_t(e) * ntiles), tl1 = uint32_t(s1 - uint64_t(e) * ntiles);
    const float* Xb = X + uint64_t(e) * M * K;
    const uint4* Cb = codes + uint64_t(e) * units_per_expert;
    float* Yb = Y + uint64_t(e) * M * N;
    float brow[G];  // book row lane % 16
    {
      const float* b = books + uint64_t(e) * 16 * G + (lane & 15) * G;
#pragma unroll
      for (int j = 0; j < G; ++j) brow[j] = __ldg(b + j);
    }
    if (tl0 == 0 && warp == 0) {  // the one block whose range starts the expert checks its book
      uint32_t bits = 0;
#pragma unroll
      for (int j = 0; j < G; ++j) bits |= finite32(brow[j]) ? 0u : kNonfinite;
      flag_warp(status, bits);
    }
    for (uint32_t m0 = 0; m0 < M; m0 += MC) {
      const uint32_t mc = min(uint32_t(MC), M - m0);
      for (uint32_t t0 = 0; t0 < T; t0 += TC) {
        for (uint32_t m = 0; m < mc; ++m) {
          // this row's X chunk into shared memory in one round trip, then
          // the 16 dots of each group: half-warp per group, lane = entry
          __syncthreads();  // the previous table / chunk is no longer read
          const float* xrow = Xb + uint64_t(m0 + m) * K + uint64_t(t0) * G;
          if (x_vec) {
            for (uint32_t i = threadIdx.x; i < TC * G / 4; i += kThreads)
              reinterpret_cast<float4*>(Xs)[i] = __ldg(reinterpret_cast<const float4*>(xrow) + i);
          } else {
            for (uint32_t i = threadIdx.x; i < TC * G; i += kThreads) Xs[i] = __ldg(xrow + i);
          }
          __syncthreads();
          for (uint32_t t = warp * 2 + (lane >> 4); t < TC; t += 2 * (kThreads / 32)) {
            const float4* xs = reinterpret_cast<const float4*>(Xs + t * G);
            float acc = 0.f;
#pragma unroll
            for (int q = 0; q < G / 4; ++q) {
              const float4 v = xs[q];
              acc = fmaf(v.x, brow[4 * q], acc);
              acc = fmaf(v.y, brow[4 * q + 1], acc);
              acc = fmaf(v.z, brow[4 * q + 2], acc);
              acc = fmaf(v.w, brow[4 * q + 3], acc);
            }
            P[size_t(t) * 16 * MC + (MC == 1 ? (lane & 15) : (m >> 1) * 32 + (lane & 15) * 2 + (m & 1))] = acc;
          }
        }
        __syncthreads();
        for (uint32_t tile = tl0 + warp; tile < tl1; tile += kThreads / 32) {
          const uint4* src = Cb + (uint64_t(tile) * ct + t0 / 32) * 32 + lane;
          uint4 q[kPieces];
#pragma unroll
          for (int pc = 0; pc < kPieces; ++pc) q[pc] = __ldg(src + pc * 32);
          // acc[m][0] = (sum 0, sum 1), acc[m][1] = (sum 2, sum 3): the even and
          // odd groups of a word pair add as one packed two-lane add
          float2 acc[MC][2];
#pragma unroll
          for (int m = 0; m < MC; ++m) acc[m][0] = acc[m][1] = make_float2(0.f, 0.f);
          const unsigned char* Pb = smem;
#pragma unroll
          for (int pc = 0; pc < kPieces; ++pc) {
            const uint32_t wd[4] = {q[pc].x, q[pc].y, q[pc].z, q[pc].w};
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
              // 4 MC * nibble of the even (lo) and odd (hi) nibbles, one per byte
              const uint32_t w = wd[wi];
              const uint32_t lo = MC == 1 ? (w << 2) & 0x3C3C3C3Cu : (w << 3) & 0x78787878u;
              const uint32_t hi = MC == 1 ? (w >> 2) & 0x3C3C3C3Cu : (w >> 1) & 0x78787878u;
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint32_t olo = __byte_perm(lo, 0, 0x4440 + kk);
                const uint32_t ohi = __byte_perm(hi, 0, 0x4440 + kk);
                const int t = pc * 32 + wi * 8 + 2 * kk;
                const unsigned char* pt = Pb + size_t(t) * 64 * MC;  // row t of the table
                float vl[MC], vh[MC];
                if constexpr (MC == 1) {
                  vl[0] = *reinterpret_cast<const float*>(pt + olo);
                  vh[0] = *reinterpret_cast<const float*>(pt + 64 + ohi);
                } else {
#pragma unroll
                  for (int mp = 0; mp < MC / 2; ++mp) {
                    const float2 a = *reinterpret_cast<const float2*>(pt + mp * 128 + olo);
                    const float2 b = *reinterpret_cast<const float2*>(pt + 64 * MC + mp * 128 + ohi);
                    vl[2 * mp] = a.x; vl[2 * mp + 1] = a.y; vh[2 * mp] = b.x; vh[2 * mp + 1] = b.y;
                  }
                }
#pragma unroll
                for (int m = 0; m < MC; ++m) acc[m][kk & 1] = __fadd2_rn(acc[m][kk & 1], make_float2(vl[m], vh[m]));
              }
            }
          }
          const uint32_t row = tile * 32 + lane;
          if (row < N) {
#pragma unroll
            for (int m = 0; m < MC; ++m) {
              if (m < int(mc)) {
                const float y = (acc[m][0].x + acc[m][0].y) + (acc[m][1].x + acc[m][1].y);
                float* dst = Yb + uint64_t(m0 + m) * N + row;
                *dst = t0 ? *dst + y : y;
              }
            }
          }
        }
      }
    }
    s0 = s1;
  }
}

// ------------------------------- dense X times coded W^T, M = 1: byte table --
//
// k_dense_pair: one lookup per code BYTE. For a K-chunk of 256 groups (128
// code bytes per row), Q[p][b] = P[2p][b & 15] + P[2p+1][b >> 4] with
// P[t][e] = x_t . c_e (256 x 16 FP32 dot products), 128 pairs x 256 bytes =
// 128 KB of shared memory. A warp takes 32 rows at a time; lane i loads word
// i of every row (one coalesced 128-byte line per row) and so always looks up
// pairs 4i..4i+3. Q is laid out so that lane i's entries live in bank i:
// word(i, j, b) = 64 b + 32 (j & 1) + i + 16384 (j >> 1) for pair 4i + j,
// and one byte permute of the code word with a per-lane base forms each
// byte address. Lane sums are folded across the warp by a 32 x 32
// transpose-reduction (31 shuffles), after which lane r holds row r.
//
// One block of 16 warps per SM, persistent over (expert, 32-row batch)
// units; the next unit range's x chunk and book are prefetched with
// cp.async while the current one is looked up. Each row sums its 128 pair
// values per chunk in a fixed order (pairs, then a tree over lanes); chunks
// add in order, so the result does not depend on the grid.
namespace pair {

constexpr int kWarps = 16, kThreads = kWarps * 32, kRows = 32;
constexpr uint32_t kQFloats = 128u * 256u;         // the byte table
constexpr uint32_t kPFloats = 256u * 16u + 32u;    // P, one pad word per 8 groups
__device__ __forceinline__ uint32_t p_index(uint32_t t, uint32_t c) { return t * 16u + c + (t >> 3); }

// Table, P and one x-chunk buffer (the next chunk is prefetched into it once
// P is built): 161 KB for g16, so the 164 KB shared-memory configuration
// leaves ~92 KB of L1 for the code loads in flight (the largest carveout
// measured 6% slower).
template <int G>
constexpr size_t smem_bytes() {
  return (size_t(kQFloats) + kPFloats + 256 * G + 16 * G) * sizeof(float);
}

}  // namespace pair

template <int G, bool ONE>  // ONE: K = 256 G, one chunk (32-word rows, a compile-time stride)
__global__ void __launch_bounds__(pair::kThreads, 1)
    k_dense_pair(const float* __restrict__ X, const uint32_t* __restrict__ codes, const float* __restrict__ books,
                 float* __restrict__ Y, uint32_t N, uint32_t K, uint32_t E, uint64_t words_per_expert,
                 uint32_t* __restrict__ status) {
  constexpr uint32_t kChunkX = 256u * G, kBook = 16u * G;
  extern __shared__ __align__(16) float pair_smem[];
  float* Q = pair_smem;
  float* P = Q + pair::kQFloats;
  float* xbuf = P + pair::kPFloats;  // x chunk, then the book
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t chunks = ONE ? 1u : K / kChunkX, row_words = ONE ? 32u : K / G / 8;
  const uint32_t nb = (N + pair::kRows - 1) / pair::kRows;  // 32-row batches per expert
  const uint64_t U = uint64_t(E) * nb;
  const uint64_t u0 = U * blockIdx.x / gridDim.x, u1 = U * (blockIdx.x + 1) / gridDim.x;
  if (u0 >= u1) return;
  // byte 0: 4 i (slots 0, 2) or 4 i + 128 (slots 1, 3); byte 2: 0 or 1 (x 64 KB)
  const uint32_t base = (lane * 4u) | ((lane * 4u + 128u) << 8) | (1u << 24);

  // the work list: (segment of one expert's units, chunk) in order
  auto seg_end = [&](uint64_t s) { return min(u1, (s / nb + 1) * nb); };
  auto prefetch = [&](uint64_t s, uint32_t c) {
    const uint32_t e = uint32_t(s / nb);
    float* dst = xbuf;
    const float* xs = X + uint64_t(e) * K + uint64_t(c) * kChunkX;
    const float* bs = books + uint64_t(e) * kBook;
    for (uint32_t i = tid; i < (kChunkX + kBook) / 4; i += pair::kThreads) {
      const float* src = i < kChunkX / 4 ? xs + 4 * i : bs + 4 * (i - kChunkX / 4);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(
                       __cvta_generic_to_shared(dst + 4 * i))),
                   "l"(src)
                   : "memory");
    }
  };
  uint64_t s0 = u0;
  uint32_t c = 0;
  prefetch(s0, 0);
  asm volatile("cp.async.commit_group;" ::: "memory");
  while (s0 < u1) {
    const uint64_t s1 = seg_end(s0);
    const uint32_t e = uint32_t(s0 / nb);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // this chunk's x and book are in; Q is no longer read
    const float* xs = xbuf;
    const float* bk = xs + kChunkX;
    if (c == 0 && s0 % nb == 0) {  // the expert's first unit reports a nonfinite book
      uint32_t bits = 0;
      for (uint32_t i = tid; i < kBook; i += pair::kThreads) bits |= finite32(bk[i]) ? 0u : kNonfinite;
      flag_warp(status, bits);
    }
    {
      // P[t][e]: thread owns entry tid % 16 (its book row in registers)
      const uint32_t ce = tid & 15;
      float br[G];
#pragma unroll
      for (int j = 0; j < G; ++j) br[j] = bk[ce * G + j];
      for (uint32_t t = tid >> 4; t < 256u; t += pair::kThreads / 16) {
        float a = 0.f;
#pragma unroll
        for (int j = 0; j < G; j += 4) {
          const float4 x4 = *reinterpret_cast<const float4*>(xs + t * G + j);
          a = fmaf(x4.x, br[j], a);
          a = fmaf(x4.y, br[j + 1], a);
          a = fmaf(x4.z, br[j + 2], a);
          a = fmaf(x4.w, br[j + 3], a);
        }
        P[pair::p_index(t, ce)] = a;
      }
    }
    __syncthreads();
    {
      // x is read: the next (segment, chunk)'s x and book, in flight during
      // the table build and the lookups
      uint64_t ns = s0;
      uint32_t nc = c + 1;
      if (nc == chunks) {
        nc = 0;
        ns = s1;
      }
      if (ns < u1) prefetch(ns, nc);
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
    // Q: a thread holds P[2p][0..15] and fills one high nibble; lane = slot i,
    // so both the P loads and the Q stores are conflict-free
    for (uint32_t task = tid; task < 128u * 16u; task += pair::kThreads) {
      const uint32_t i = task & 31, j = (task >> 5) & 3, hi = task >> 7;
      const uint32_t p = 4 * i + j;
      float lo[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) lo[k] = P[pair::p_index(2 * p, k)];
      const float hv = P[pair::p_index(2 * p + 1, hi)];
      float* q = Q + (j & 1u) * 32u + i + (j >> 1) * 16384u + hi * 16u * 64u;
#pragma unroll
      for (int k = 0; k < 16; ++k) q[k * 64] = lo[k] + hv;
    }
    __syncthreads();

    // codes of this (expert, chunk): a warp-uniform base, 32-bit lane offsets
    const uint32_t* cb = codes + uint64_t(e) * words_per_expert + uint64_t(c) * 32u;
    float* ye = Y + uint64_t(e) * N;
    uint64_t u = s0 + warp;
    uint32_t w[pair::kRows];
    const uint64_t first = uint64_t(e) * nb;  // units of this segment are one expert's
    auto load = [&](uint64_t unit) {
      const uint32_t n0 = uint32_t(unit - first) * pair::kRows;
      const uint32_t off = n0 * row_words + lane;
      if (n0 + pair::kRows <= N) {
#pragma unroll
        for (int r = 0; r < pair::kRows; ++r) w[r] = __ldcs(cb + off + uint32_t(r) * row_words);
      } else {
#pragma unroll
        for (int r = 0; r < pair::kRows; ++r) w[r] = n0 + r < N ? __ldcs(cb + off + uint32_t(r) * row_words) : 0u;
      }
    };
    if (u < s1) load(u);
    for (; u < s1; u += pair::kWarps) {
      const uint32_t n0 = uint32_t(u - first) * pair::kRows;
      float v[pair::kRows];
#pragma unroll
      for (int r = 0; r < pair::kRows; ++r) {
        const char* qb = reinterpret_cast<const char*>(Q);
        const float q0 = *reinterpret_cast<const float*>(qb + __byte_perm(w[r], base, 0x6604));
        const float q1 = *reinterpret_cast<const float*>(qb + __byte_perm(w[r], base, 0x6615));
        const float q2 = *reinterpret_cast<const float*>(qb + __byte_perm(w[r], base, 0x6724));
        const float q3 = *reinterpret_cast<const float*>(qb + __byte_perm(w[r], base, 0x6735));
        v[r] = (q0 + q1) + (q2 + q3);
      }
      if (u + pair::kWarps < s1) load(u + pair::kWarps);  // in flight during the folding
      // fold lanes: each step halves the rows a lane keeps; after five, lane l holds row l
#pragma unroll
      for (int off = pair::kRows / 2; off; off >>= 1) {
        const bool up = lane & off;
#pragma unroll
        for (int k = 0; k < off; ++k) {
          const float send = up ? v[k] : v[k + off];
          const float keep = up ? v[k + off] : v[k];
          v[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      if (n0 + lane < N) {  // lane l now holds row n0 + l
        float* y = ye + n0 + lane;
        *y = c == 0 ? v[0] : *y + v[0];
      }
    }
    // advance: the next chunk of this segment, or the next segment
    if (++c == chunks) {
      c = 0;
      s0 = s1;
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// ------------------------------------------ coded A times coded B^T (LUT) --

// C[m, n] = sum_t L[a(m,t)][b(n,t)] with L = C_A C_B^T (16 x 16, each entry
// summed in float64 and rounded once). A stored M x K, B stored N x K,
// K % G == 0 and (K/G) % 8 == 0 so every row starts on a code word. A block
// owns kCodedRows rows of A (the same for all its warps, so A's indices are
// block-uniform) and 8 x 32 x kCodedCols columns; each lane kCodedRows x
// kCodedCols outputs. Every lookup of an instruction reads one 16-entry row
// of L: distinct columns hit distinct banks, equal columns broadcast. (16 x 4
// per lane measured fastest of 8x8, 4x8, 8x4, 4x4, 16x4, 4x16.)
constexpr int kCodedRows = 16, kCodedCols = 4;

template <int G>
__global__ void __launch_bounds__(kThreads, 2) k_coded_lut(const uint32_t* __restrict__ ac,
                                                           const float* __restrict__ ab,
                                                           const uint32_t* __restrict__ bc,
                                                           const float* __restrict__ bb, float* __restrict__ C,
                                                           uint32_t M, uint32_t N, uint32_t K,
                                                           uint32_t* __restrict__ status) {
  __shared__ float L[16 * 16];
  __shared__ float sa[16 * 32], sbk[16 * 32];
  for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) {
    sa[i] = ab[i];
    sbk[i] = bb[i];
  }
  __syncthreads();
  {
    const int e = threadIdx.x / 16, f = threadIdx.x % 16;
    double s = 0.0;
    for (int j = 0; j < G; ++j) s = __dadd_rn(s, __dmul_rn(double(sa[e * G + j]), double(sbk[f * G + j])));
    L[e * 16 + f] = __double2float_rn(s);
  }
  if (blockIdx.x == 0 && blockIdx.y == 0) {
    uint32_t bits = 0;
    for (int i = threadIdx.x; i < 16 * G; i += blockDim.x)
      bits |= (finite32(sa[i]) && finite32(sbk[i])) ? 0u : kNonfinite;
    flag_warp(status, bits);
  }
  __syncthreads();
  constexpr int RI = kCodedRows, RJ = kCodedCols;
  const uint32_t TW = K / G / 8;  // code words per row
  const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t row0 = blockIdx.x * RI;  // rows on x: up to 2^16 row blocks
  const uint32_t col0 = blockIdx.y * (8 * 32 * RJ) + warp * (32 * RJ) + lane;
  const uint32_t* bcol[RJ];
#pragma unroll
  for (int j = 0; j < RJ; ++j) bcol[j] = bc + uint64_t(min(col0 + 32 * j, N - 1)) * TW;
  float acc[RI][RJ];
#pragma unroll
  for (int i = 0; i < RI; ++i)
#pragma unroll
    for (int j = 0; j < RJ; ++j) acc[i][j] = 0.f;
  for (uint32_t tw = 0; tw < TW; ++tw) {
    uint32_t aw[RI], bw[RJ];
#pragma unroll
    for (int i = 0; i < RI; ++i) aw[i] = __ldg(ac + uint64_t(min(row0 + i, M - 1)) * TW + tw);
#pragma unroll
    for (int j = 0; j < RJ; ++j) bw[j] = __ldg(bcol[j] + tw);
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const float* Lr[RI];
#pragma unroll
      for (int i = 0; i < RI; ++i) Lr[i] = L + (((aw[i] >> (4 * s)) & 15u) << 4);
      uint32_t b1[RJ];
#pragma unroll
      for (int j = 0; j < RJ; ++j) b1[j] = (bw[j] >> (4 * s)) & 15u;
#pragma unroll
      for (int i = 0; i < RI; ++i)
#pragma unroll
        for (int j = 0; j < RJ; ++j) acc[i][j] += Lr[i][b1[j]];
    }
  }
  uint32_t bits = 0;
#pragma unroll
  for (int i = 0; i < RI; ++i)
#pragma unroll
    for (int j = 0; j < RJ; ++j) {
      const uint32_t r = row0 + i, c = col0 + 32 * j;
      if (r < M && c < N) {
        C[uint64_t(r) * N + c] = acc[i][j];
        bits |= finite32(acc[i][j]) ? 0u : kNonfinite;
      }
    }
  flag_warp(status, bits);
}

// --------------------------------------------- generic tiled product (FMA) --

// Operand sources of the generic product: a dense FP32 row-major matrix, or a
// coded image with its layout flag.
struct Operand {
  const float* dense;      // non-null: dense row-major (rows x K)
  const uint32_t* codes;   // coded image
  const float* book;
  int stored_transposed;   // coded: A stored K x M (for A) or B stored N x K (for B)
};

template <int G>
__device__ __forceinline__ float op_a(const Operand& a, uint32_t row, uint32_t k, uint32_t M, uint32_t K) {
  if (a.dense) return __ldg(a.dense + uint64_t(row) * K + k);
  const uint64_t logical = a.stored_transposed ? uint64_t(k) * M + row : uint64_t(row) * K + k;
  return dequant<G>(a.codes, a.book, logical);
}
template <int G>
__device__ __forceinline__ float op_b(const Operand& b, uint32_t k, uint32_t col, uint32_t N, uint32_t K) {
  const uint64_t logical = b.stored_transposed ? uint64_t(col) * K + k : uint64_t(k) * N + col;
  return dequant<G>(b.codes, b.book, logical);
}

// C_z[M,N] = A_z B_z over blockIdx.z; per-z offsets in elements/words.
template <int G>
__global__ void __launch_bounds__(kThreads) k_gemm_generic(Operand A, Operand B, float* __restrict__ C, uint32_t M,
                                                           uint32_t N, uint32_t K, uint64_t a_dense_z,
                                                           uint64_t b_words_z, uint32_t* __restrict__ status) {
  constexpr int T = 64, KC = 16;
  __shared__ float As[KC][T + 4];
  __shared__ float Bs[KC][T + 4];
  const uint32_t z = blockIdx.z;
  if (A.dense) A.dense += z * a_dense_z;
  B.codes += z * b_words_z;
  B.book += uint64_t(z) * 16 * G;
  C += uint64_t(z) * M * N;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const uint32_t row0 = blockIdx.y * T, col0 = blockIdx.x * T;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  if (blockIdx.x == 0 && blockIdx.y == 0) {
    uint32_t bits = 0;
    for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) {
      bits |= finite32(B.book[i]) ? 0u : kNonfinite;
      if (!A.dense) bits |= finite32(A.book[i]) ? 0u : kNonfinite;
    }
    flag_warp(status, bits);
  }
  for (uint32_t k0 = 0; k0 < K; k0 += KC) {
    for (int i = threadIdx.x; i < KC * T; i += blockDim.x) {
      const int kk = i / T, rr = i % T;
      const uint32_t k = k0 + kk, row = row0 + rr, col = col0 + rr;
      As[kk][rr] = (k < K && row < M) ? op_a<G>(A, row, k, M, K) : 0.f;
      Bs[kk][rr] = (k < K && col < N) ? op_b<G>(B, k, col, N, K) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < KC; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  uint32_t bits = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t row = row0 + ty * 4 + i, col = col0 + tx * 4 + j;
      if (row < M && col < N) {
        C[uint64_t(row) * N + col] = acc[i][j];
        bits |= finite32(acc[i][j]) ? 0u : kNonfinite;
      }
    }
  flag_warp(status, bits);
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

// out[e][state][s][j]: AdamW values of the calibration sample vectors.
template <int G>
__global__ void __launch_bounds__(kThreads) k_adamw_sample(AdamwBatch a, const uint32_t* __restrict__ sample,
                                                           uint32_t S, float* __restrict__ out,
                                                           uint32_t* __restrict__ status) {
  __shared__ float sbooks[4 * 16 * G];
  const uint32_t e = blockIdx.y;
  for (int i = threadIdx.x; i < 64 * G; i += blockDim.x) sbooks[i] = a.books[uint64_t(e) * 64 * G + i];
  __syncthreads();
  const AdamwCoefs k = load_coefs(a.coefs + 7 * e);
  const uint64_t total = uint64_t(S) * G;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t s = uint32_t(i / G), j = uint32_t(i % G);
    const uint64_t v = sample[s];
    uint32_t bits = k.status;
    if (v >= uint64_t(a.n) / G) bits |= kLayout;  // a position outside the complete vectors
    float nw = 0.f, nm = 0.f, nv = 0.f;
    if (!bits) {
      const uint32_t* base = a.codes + uint64_t(e) * 4 * a.words;
      float st[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) st[q] = sbooks[q * 16 * G + code_at(base + q * a.words, v) * G + j];
      bool skip;
      bits = adamw_value(k, st[0], st[1], st[2], st[3], &nw, &nm, &nv, &skip);
    }
    float* o = out + uint64_t(e) * 3 * total;
    o[i] = nw;
    o[total + i] = nm;
    o[2 * total + i] = nv;
    if (bits) atomicOr(status, bits);
  }
}

// Entries a trial book (constant slot SLOT, book 0) selects over the
// complete vectors of one updated state (the whole-tensor pass of
// fit_codebook, vq.py:219-222). One vector per thread.
template <int G, int SLOT>
__global__ void __launch_bounds__(kThreads, adamw_min_blocks<G>()) k_adamw_usage(AdamwBatch a, uint32_t expert,
                                                                                 uint32_t state,
                                                                                 uint32_t* __restrict__ out,
                                                                                 uint32_t* __restrict__ status) {
  using Book = CBook<G, SLOT, 0>;
  __shared__ float sbooks[4 * 16 * G];
  __shared__ uint32_t hist[16];
  for (int i = threadIdx.x; i < 64 * G; i += blockDim.x) sbooks[i] = a.books[uint64_t(expert) * 64 * G + i];
  if (threadIdx.x < 16) hist[threadIdx.x] = 0;
  __syncthreads();
  const AdamwCoefs k = load_coefs(a.coefs + 7 * expert);
  const uint64_t full = a.n / G;
  const uint64_t v = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  uint32_t bits = k.status;
  if (v < full && !bits) {
    float x[G];
    adamw_vector<G>(a, sbooks, k, expert, v, G, int(state), x, &bits);
    bool certified;
    atomicAdd(&hist[enc_vector<G, Book>(x, &certified)], 1u);
  }
  flag_warp(status, bits);
  __syncthreads();
  if (threadIdx.x < 16 && hist[threadIdx.x]) atomicAdd(out + threadIdx.x, hist[threadIdx.x]);
}

// decode -> AdamW -> encode of W', M', V' of one expert with their new books
// (constant slot SLOT, books 0, 1, 2), one vector per thread, and a count of
// weight values whose decoded value changed.
template <int G, int SLOT>
__global__ void __launch_bounds__(kThreads, adamw_min_blocks<G>()) k_adamw_encode(AdamwBatch a, uint32_t e,
                                                                                  uint32_t* __restrict__ out_codes,
                                                                                  uint32_t* __restrict__ changed,
                                                                                  uint32_t* __restrict__ status) {
  using BW = CBook<G, SLOT, 0>;
  using BM = CBook<G, SLOT, 1>;
  using BV = CBook<G, SLOT, 2>;
  __shared__ float sbooks[4 * 16 * G];
  for (int i = threadIdx.x; i < 64 * G; i += blockDim.x) sbooks[i] = a.books[uint64_t(e) * 64 * G + i];
  __syncthreads();
  const AdamwCoefs k = load_coefs(a.coefs + 7 * e);
  if (blockIdx.x == 0 && threadIdx.x == 0 && (BW::bad() || BM::bad() || BV::bad())) atomicOr(status, kNonfinite);
  const uint64_t vectors = (uint64_t(a.n) + G - 1) / G;
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t base = uint64_t(blockIdx.x) * blockDim.x + (threadIdx.x & ~31u);
  const uint64_t v = base + lane;
  uint32_t changes = 0;
  uint32_t idx[3] = {0, 0, 0}, bits = k.status;
  if (v < vectors && !bits) {
    const int valid = int(min(uint64_t(G), uint64_t(a.n) - v * G));
    bool certified;
    if (G <= 16) {
      // the AdamW arithmetic (two divisions and a square root per value) once
      float w[G], m[G], var[G];
      adamw_vector3<G>(a, sbooks, k, e, v, valid, w, m, var, &bits);
      idx[0] = valid == G ? enc_vector<G, BW>(w, &certified) : enc_exact<G, BW>(w, valid, 0xffffu);
      idx[1] = valid == G ? enc_vector<G, BM>(m, &certified) : enc_exact<G, BM>(m, valid, 0xffffu);
      idx[2] = valid == G ? enc_vector<G, BV>(var, &certified) : enc_exact<G, BV>(var, valid, 0xffffu);
    } else {
      // group 32: one state at a time keeps one vector of values live
      float x[G];
      adamw_vector<G>(a, sbooks, k, e, v, valid, 0, x, &bits);
      idx[0] = valid == G ? enc_vector<G, BW>(x, &certified) : enc_exact<G, BW>(x, valid, 0xffffu);
      adamw_vector<G>(a, sbooks, k, e, v, valid, 1, x, &bits);
      idx[1] = valid == G ? enc_vector<G, BM>(x, &certified) : enc_exact<G, BM>(x, valid, 0xffffu);
      adamw_vector<G>(a, sbooks, k, e, v, valid, 2, x, &bits);
      idx[2] = valid == G ? enc_vector<G, BV>(x, &certified) : enc_exact<G, BV>(x, valid, 0xffffu);
    }
    // vq.py:402: decoded new weight against decoded old weight, value by value
    const uint32_t old = code_at(a.codes + uint64_t(e) * 4 * a.words, v);
    for (int j = 0; j < valid; ++j) changes += BW::at(int(idx[0]), j) != sbooks[old * G + j];
  }
#pragma unroll
  for (int s = 0; s < 3; ++s) {
    const uint32_t word_bits = pack_nibbles(idx[s]);
    const uint64_t word = (base >> 3) + (lane >> 3);
    if ((lane & 7) == 0 && word < a.words) out_codes[(uint64_t(e) * 3 + s) * a.words + word] = word_bits;
  }
  flag_warp(status, bits);
  for (int o = 16; o; o >>= 1) changes += __shfl_xor_sync(0xffffffffu, changes, o);
  if (lane == 0 && changes) atomicAdd(changed + e, changes);
}

// ---------------------------------------------------------------- helpers --

int g_sm_count[64];

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
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

// The constant-bank slots of one device. A launch holds the ring's lock from
// choosing its slot to recording the slot's event: it makes its stream wait
// for the slot's previous launch (on whatever stream that ran), copies its
// book(s) into the slot on its own stream, launches, and records the event.
struct SlotRing {
  std::mutex mu;
  uint32_t next = 0;
  cudaEvent_t done[kBookSlots] = {};
};
SlotRing g_rings[64];

// Device address of g_stage, looked up once per device.
float* stage_address(cudaError_t* err) {
  static std::mutex mu;
  static float* addr[64] = {};
  int dev = 0;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev & 63]) *err = cudaGetSymbolAddress(reinterpret_cast<void**>(&addr[dev & 63]), g_stage);
  return addr[dev & 63];
}

// One launch's hold on a slot: waits for the slot's previous user, stages
// `nb` books of group `group` from `src` (device memory) into it, and on
// release records the slot's event.
class BookSlot {
 public:
  BookSlot(cudaStream_t stream, const void* src, int nb, uint32_t group) : stream_(stream) {
    int dev = 0;
    cudaGetDevice(&dev);
    ring_ = &g_rings[dev & 63];
    lock_ = std::unique_lock<std::mutex>(ring_->mu);
    index_ = int(ring_->next++ % kBookSlots);
    cudaEvent_t& ev = ring_->done[index_];
    err_ = ev ? cudaStreamWaitEvent(stream, ev, 0) : cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    float* stage = nullptr;
    if (err_ == cudaSuccess) stage = stage_address(&err_);
    if (err_ != cudaSuccess) return;
    const float* books = static_cast<const float*>(src);
    if (group == 8) k_stage_books<8><<<1, 32 * nb, 0, stream>>>(books, nb, index_);
    else if (group == 16) k_stage_books<16><<<1, 32 * nb, 0, stream>>>(books, nb, index_);
    else k_stage_books<32><<<1, 32 * nb, 0, stream>>>(books, nb, index_);
    err_ = cudaGetLastError();
    if (err_ == cudaSuccess)  // books and their meta: the whole slot
      err_ = cudaMemcpyToSymbolAsync(c_books, stage + size_t(index_) * kSlotFloats, kSlotFloats * sizeof(float),
                                     size_t(index_) * kSlotFloats * sizeof(float), cudaMemcpyDeviceToDevice, stream);
  }
  ~BookSlot() {
    if (lock_.owns_lock()) release();
  }
  int index() const { return index_; }
  cudaError_t error() const { return err_; }
  cudaError_t release() {
    cudaError_t e = cudaEventRecord(ring_->done[index_], stream_);
    lock_.unlock();
    return e;
  }

 private:
  cudaStream_t stream_;
  SlotRing* ring_ = nullptr;
  std::unique_lock<std::mutex> lock_;
  int index_ = 0;
  cudaError_t err_ = cudaSuccess;
};

#define ACK_SLOT_SWITCH(slot, LAUNCH) \
  switch (slot) {                     \
    case 0: LAUNCH(0); break;         \
    case 1: LAUNCH(1); break;         \
    case 2: LAUNCH(2); break;         \
    case 3: LAUNCH(3); break;         \
    case 4: LAUNCH(4); break;         \
    case 5: LAUNCH(5); break;         \
    case 6: LAUNCH(6); break;         \
    default: LAUNCH(7); break;        \
  }

template <int G>
struct RunDecode {
  static cudaError_t run(const uint32_t* codes, const float* book, float* out, uint64_t n, uint32_t* status,
                         cudaStream_t s) {
    if (aligned16(out)) {
      // 16 blocks of 8 warps per SM (two rounds of residency), measured best
      const uint64_t steps = (n / 4 + 256 * (G / 4) - 1) / (256 * (G / 4));
      const uint64_t grid = std::max<uint64_t>(1, std::min<uint64_t>((steps + 7) / 8, uint64_t(sm_count()) * 16));
      k_decode<G><<<uint32_t(grid), kThreads, 0, s>>>(codes, book, out, n, status);
    } else {
      k_decode_scalar<G><<<grid_for(n), kThreads, 0, s>>>(codes, book, out, n, status);
    }
    return cudaGetLastError();
  }
};

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

// The tensor map of x as rows of G floats (its complete vectors), boxes of
// the encode tile's rows, swizzled to the rows' width.
template <int G>
bool encode_tensor_map(const float* x, uint64_t complete, CUtensorMap* map) {
  const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return false;
  const cuuint64_t dims[2] = {cuuint64_t(G), cuuint64_t(complete)};
  const cuuint64_t strides[1] = {cuuint64_t(G) * sizeof(float)};
  const cuuint32_t box[2] = {cuuint32_t(G), tc::Cfg<G>::kBoxRows};
  const cuuint32_t elem[2] = {1, 1};
  const CUtensorMapSwizzle sw =
      G == 8 ? CU_TENSOR_MAP_SWIZZLE_32B : (G == 16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int G>
struct RunEncode {
  static cudaError_t run(const float* x, uint64_t n, const float* book, uint32_t* codes, uint32_t* status,
                         cudaStream_t s) {
    const uint64_t vectors = (n + G - 1) / G;
    const bool vec = aligned16(x);
    // tensor-core path: 16-byte aligned rows, at least one complete vector,
    // row coordinates within the TMA's signed 32 bits
    if (vec && n / G >= 1 && vectors < (uint64_t(1) << 31) - 1024) {
      CUtensorMap map;
      if (encode_tensor_map<G>(x, n / G, &map)) return run_tc(map, x, n, book, codes, status, s);
    }
    if constexpr (G == 32) {
      if (vec) return run_async(x, n, book, codes, status, s);
    }
    const uint64_t grid = grid_for(vectors, resident_per_sm(k_encode<G, 0, true>, 0));
    BookSlot slot(s, book, 1, G);
    if (slot.error() != cudaSuccess) return slot.error();
#define ACK_LAUNCH_ENCODE(S)                                                                 \
  if (vec) k_encode<G, S, true><<<uint32_t(grid), kThreads, 0, s>>>(x, n, codes, status);  \
  else k_encode<G, S, false><<<uint32_t(grid), kThreads, 0, s>>>(x, n, codes, status)
    ACK_SLOT_SWITCH(slot.index(), ACK_LAUNCH_ENCODE)
#undef ACK_LAUNCH_ENCODE
    const cudaError_t e = cudaGetLastError();
    const cudaError_t r = slot.release();
    return e != cudaSuccess ? e : r;
  }

  static cudaError_t run_tc(const CUtensorMap& map, const float* x, uint64_t n, const float* book, uint32_t* codes,
                            uint32_t* status, cudaStream_t s) {
    using K = tc::Cfg<G>;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
#define ACK_TC_ATTR(S)                                                                                      \
  if (attr == cudaSuccess)                                                                                  \
    attr = cudaFuncSetAttribute(k_encode_tc<G, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(K::kSmem)); \
  if (attr == cudaSuccess)                                                                                  \
    attr = cudaFuncSetAttribute(k_encode_tc<G, S>, cudaFuncAttributePreferredSharedMemoryCarveout,          \
                                int(cudaSharedmemCarveoutMaxShared));
      ACK_TC_ATTR(0) ACK_TC_ATTR(1) ACK_TC_ATTR(2) ACK_TC_ATTR(3)
      ACK_TC_ATTR(4) ACK_TC_ATTR(5) ACK_TC_ATTR(6) ACK_TC_ATTR(7)
#undef ACK_TC_ATTR
    });
    if (attr != cudaSuccess) return attr;
    const uint64_t vectors = (n + G - 1) / G;
    const uint64_t tiles = (vectors + 128 * K::H - 1) / (128 * K::H);
    // two blocks per SM by design (registers and shared memory both allow
    // exactly two); blocks are independent, so an SM that holds fewer only
    // runs the rest later
    const uint32_t grid = uint32_t(std::min<uint64_t>(tiles, uint64_t(sm_count()) * K::kBlocksPerSm));
    BookSlot slot(s, book, 1, G);
    if (slot.error() != cudaSuccess) return slot.error();
#define ACK_LAUNCH_ENCODE(S) k_encode_tc<G, S><<<grid, K::kThreads, K::kSmem, s>>>(map, x, n, codes, status)
    ACK_SLOT_SWITCH(slot.index(), ACK_LAUNCH_ENCODE)
#undef ACK_LAUNCH_ENCODE
    const cudaError_t e = cudaGetLastError();
    const cudaError_t r = slot.release();
    return e != cudaSuccess ? e : r;
  }

  // group 32, aligned x: coalesced cp.async staging (k_encode_async)
  static cudaError_t run_async(const float* x, uint64_t n, const float* book, uint32_t* codes, uint32_t* status,
                               cudaStream_t s) {
    const uint64_t vectors = (n + G - 1) / G;
    constexpr size_t smem = size_t(kThreads / 32) * 2 * 8 * G * 16;
    cudaError_t err = cudaSuccess;
#define ACK_ASYNC_ATTR(S)                                                                                       \
  if (err == cudaSuccess)                                                                                       \
    err = cudaFuncSetAttribute(k_encode_async<G, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    ACK_ASYNC_ATTR(0) ACK_ASYNC_ATTR(1) ACK_ASYNC_ATTR(2) ACK_ASYNC_ATTR(3)
    ACK_ASYNC_ATTR(4) ACK_ASYNC_ATTR(5) ACK_ASYNC_ATTR(6) ACK_ASYNC_ATTR(7)
#undef ACK_ASYNC_ATTR
    if (err != cudaSuccess) return err;
    const uint64_t grid = grid_for(vectors, resident_per_sm(k_encode_async<G, 0>, smem));
    BookSlot slot(s, book, 1, G);
    if (slot.error() != cudaSuccess) return slot.error();
#define ACK_LAUNCH_ENCODE(S) k_encode_async<G, S><<<uint32_t(grid), kThreads, smem, s>>>(x, n, codes, status)
    ACK_SLOT_SWITCH(slot.index(), ACK_LAUNCH_ENCODE)
#undef ACK_LAUNCH_ENCODE
    const cudaError_t e = cudaGetLastError();
    const cudaError_t r = slot.release();
    return e != cudaSuccess ? e : r;
  }
};

template <int G>
struct RunMatmulExact {
  static cudaError_t run(const Plan& p, void* const* ptr, cudaStream_t s) {
    dim3 grid(uint32_t((p.n + 63) / 64), uint32_t((p.m + 63) / 64));
    k_matmul_exact<G><<<grid, kThreads, 0, s>>>(
        static_cast<const uint32_t*>(ptr[0]), static_cast<const float*>(ptr[1]), static_cast<const uint32_t*>(ptr[2]),
        static_cast<const float*>(ptr[3]), static_cast<float*>(ptr[4]), uint32_t(p.m), uint32_t(p.n), uint32_t(p.k),
        p.flags, static_cast<uint32_t*>(ptr[5]));
    return cudaGetLastError();
  }
};

// Rows of W per work item, in 256-row batches: the fewest waves of resident
// blocks, each item's table build counted as 0.3 of a batch.
uint32_t balance_batches(uint32_t nbatches, uint32_t experts, uint64_t resident) {
  double best = 1e300;
  uint32_t pick = nbatches;
  for (uint32_t b = 1; b <= nbatches; ++b) {
    const uint64_t items = uint64_t(experts) * ((nbatches + b - 1) / b);
    const uint64_t waves = (items + resident - 1) / resident;
    const double cost = double(waves) * (b + 0.3);
    if (cost < best - 1e-9) {
      best = cost;
      pick = b;
    }
  }
  return pick;
}

template <int G, int MC, int TC>
cudaError_t launch_dense_lut(const float* X, const uint32_t* codes, const float* books, float* Y, uint32_t M,
                             uint32_t N, uint32_t K, uint32_t batch, uint64_t words, uint32_t* status,
                             cudaStream_t s) {
  const size_t smem = size_t(MC) * TC * 64 + 2 * size_t(kThreads) * (TC / 2 + 16);
  cudaError_t err = cudaFuncSetAttribute(k_dense_lut<G, MC, TC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(smem));
  if (err != cudaSuccess) return err;
  const uint64_t resident = uint64_t(sm_count()) * resident_per_sm(k_dense_lut<G, MC, TC>, smem);
  const uint32_t nbatches = (N + kThreads - 1) / kThreads;
  const uint32_t per_item = balance_batches(nbatches, batch, resident);
  const uint32_t items = (nbatches + per_item - 1) / per_item;
  k_dense_lut<G, MC, TC><<<uint32_t(uint64_t(items) * batch), kThreads, smem, s>>>(
      X, codes, books, Y, M, N, K, items, per_item, words, status);
  return cudaGetLastError();
}

template <int G, int MC>
cudaError_t launch_dense_mc(const float* X, const uint32_t* codes, const float* books, float* Y, uint32_t M,
                            uint32_t N, uint32_t K, uint32_t batch, uint64_t words, uint32_t* status, cudaStream_t s) {
  const uint32_t T = K / G;
  // t-chunk sizes (the tile32 launcher uses the same, so both layouts sum alike)
  if (MC <= 2 && T % 256 == 0) return launch_dense_lut<G, MC, (MC <= 2 ? 256 : 128)>(X, codes, books, Y, M, N, K, batch, words, status, s);
  if (T % 128 == 0) return launch_dense_lut<G, MC, 128>(X, codes, books, Y, M, N, K, batch, words, status, s);
  return launch_dense_lut<G, MC, 32>(X, codes, books, Y, M, N, K, batch, words, status, s);
}

template <int G, int MC, int TC>
cudaError_t launch_dense_t32(const float* X, const uint4* codes, const float* books, float* Y, uint32_t M,
                             uint32_t N, uint32_t K, uint32_t batch, uint32_t* status, cudaStream_t s) {
  const size_t smem = size_t(MC) * TC * 64 + size_t(TC) * G * 4;
  cudaError_t err = cudaFuncSetAttribute(k_dense_t32<G, MC, TC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(smem));
  if (err != cudaSuccess) return err;
  const uint64_t resident = uint64_t(sm_count()) * resident_per_sm(k_dense_t32<G, MC, TC>, smem);
  const uint64_t tiles = uint64_t(batch) * ((N + 31) / 32);
  // one persistent wave, at least one tile per warp per block
  const uint64_t grid = std::max<uint64_t>(1, std::min<uint64_t>(resident, (tiles + 7) / 8));
  const uint64_t units = tile32_bytes(N, K, G) / 16;
  k_dense_t32<G, MC, TC><<<uint32_t(grid), kThreads, smem, s>>>(X, codes, books, Y, M, N, K, batch, units, status);
  return cudaGetLastError();
}

template <int G, int MC>
cudaError_t launch_t32_mc(const float* X, const uint4* codes, const float* books, float* Y, uint32_t M, uint32_t N,
                          uint32_t K, uint32_t batch, uint32_t* status, cudaStream_t s) {
  // the t-chunk sizes of the canonical path for the same M (the per-row sums
  // then match it bit for bit): 256 groups for M <= 2, 128 beyond
  const uint32_t T = K / G;
  if (T % 256 == 0 && MC <= 2) return launch_dense_t32<G, MC, (MC <= 2 ? 256 : 128)>(X, codes, books, Y, M, N, K, batch, status, s);
  if (T % 128 == 0) return launch_dense_t32<G, MC, 128>(X, codes, books, Y, M, N, K, batch, status, s);
  return launch_dense_t32<G, MC, 32>(X, codes, books, Y, M, N, K, batch, status, s);
}

// M = 1 with K a multiple of 256 g: the byte-table kernel, one block per SM.
// Worth its 128 KB table per (expert, K-chunk) only with enough rows: at
// least 4 batches of 32 rows per block and 256 rows per expert.
template <int G>
bool dense_pair_fits(uint32_t M, uint32_t N, uint32_t K, uint32_t batch, const float* X, const float* books) {
  const uint64_t units = uint64_t(batch) * ((N + pair::kRows - 1) / pair::kRows);
  return M == 1 && K % (256u * G) == 0 && N >= 256 && units >= 4ull * uint64_t(sm_count()) && aligned16(X) &&
         aligned16(books) && uint64_t(N) * (K / G / 8) < (uint64_t(1) << 31);  // 32-bit word offsets
}

template <int G>
cudaError_t launch_dense_pair(const float* X, const uint32_t* codes, const float* books, float* Y, uint32_t N,
                              uint32_t K, uint32_t batch, uint64_t words, uint32_t* status, cudaStream_t s) {
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    // no carveout preference: the driver takes the smallest shared-memory
    // configuration that fits, the rest stays L1 for the code stream
    for (auto fn : {k_dense_pair<G, true>, k_dense_pair<G, false>})
      if (attr == cudaSuccess)
        attr = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(pair::smem_bytes<G>()));
  });
  if (attr != cudaSuccess) return attr;
  const uint64_t units = uint64_t(batch) * ((N + pair::kRows - 1) / pair::kRows);
  const uint32_t grid = uint32_t(std::min<uint64_t>(units, uint64_t(sm_count())));
  if (K == 256u * G)
    k_dense_pair<G, true><<<grid, pair::kThreads, pair::smem_bytes<G>(), s>>>(X, codes, books, Y, N, K, batch, words,
                                                                               status);
  else
    k_dense_pair<G, false><<<grid, pair::kThreads, pair::smem_bytes<G>(), s>>>(X, codes, books, Y, N, K, batch, words,
                                                                                status);
  return cudaGetLastError();
}

template <int G>
struct RunDense {
  static cudaError_t run(const Plan& p, void* const* ptr, cudaStream_t s) {
    const float* X = static_cast<const float*>(ptr[0]);
    const uint32_t* codes = static_cast<const uint32_t*>(ptr[1]);
    const float* books = static_cast<const float*>(ptr[2]);
    float* Y = static_cast<float*>(ptr[5]);
    uint32_t* status = static_cast<uint32_t*>(ptr[7]);
    const uint32_t M = uint32_t(p.m), N = uint32_t(p.n), K = uint32_t(p.k);
    const uint64_t words = packed_words(uint64_t(N) * K, G);
    const bool nt = (p.flags & 2u) != 0;
    if (p.flags & 4u) {
      if (!aligned16(codes)) return cudaErrorMisalignedAddress;
      const uint4* c4 = reinterpret_cast<const uint4*>(codes);
      if (M == 1) return launch_t32_mc<G, 1>(X, c4, books, Y, M, N, K, p.batch, status, s);
      if (M == 2) return launch_t32_mc<G, 2>(X, c4, books, Y, M, N, K, p.batch, status, s);
      return launch_t32_mc<G, 4>(X, c4, books, Y, M, N, K, p.batch, status, s);  // M > 4: chunks of 4 rows
    }
    if (nt && dense_pair_fits<G>(M, N, K, p.batch, X, books))
      return launch_dense_pair<G>(X, codes, books, Y, N, K, p.batch, words, status, s);
    if (nt && K % G == 0 && (K / G) % 32 == 0 && aligned16(codes) && (words * 4) % 16 == 0) {
      if (M == 1) return launch_dense_mc<G, 1>(X, codes, books, Y, M, N, K, p.batch, words, status, s);
      if (M == 2) return launch_dense_mc<G, 2>(X, codes, books, Y, M, N, K, p.batch, words, status, s);
      if (M <= 4) return launch_dense_mc<G, 4>(X, codes, books, Y, M, N, K, p.batch, words, status, s);
      return launch_dense_mc<G, 8>(X, codes, books, Y, M, N, K, p.batch, words, status, s);
    }
    Operand A{X, nullptr, nullptr, 0};
    Operand B{nullptr, codes, books, nt ? 1 : 0};
    dim3 grid((N + 63) / 64, (M + 63) / 64, p.batch);
    k_gemm_generic<G><<<grid, kThreads, 0, s>>>(A, B, Y, M, N, K, uint64_t(M) * K, words, status);
    return cudaGetLastError();
  }
};

template <int G>
struct RunCoded {
  static cudaError_t run(const Plan& p, void* const* ptr, cudaStream_t s) {
    const uint32_t* ac = static_cast<const uint32_t*>(ptr[0]);
    const float* ab = static_cast<const float*>(ptr[1]);
    const uint32_t* bc = static_cast<const uint32_t*>(ptr[2]);
    const float* bb = static_cast<const float*>(ptr[3]);
    float* C = static_cast<float*>(ptr[5]);
    uint32_t* status = static_cast<uint32_t*>(ptr[7]);
    const uint32_t M = uint32_t(p.m), N = uint32_t(p.n), K = uint32_t(p.k);
    if (p.flags == 2u && K % G == 0 && (K / G) % 8 == 0) {
      dim3 grid((M + kCodedRows - 1) / kCodedRows, (N + 8 * 32 * kCodedCols - 1) / (8 * 32 * kCodedCols));
      k_coded_lut<G><<<grid, kThreads, 0, s>>>(ac, ab, bc, bb, C, M, N, K, status);
      return cudaGetLastError();
    }
    Operand A{nullptr, ac, ab, int(p.flags & 1u)};
    Operand B{nullptr, bc, bb, int((p.flags >> 1) & 1u)};
    dim3 grid((N + 63) / 64, (M + 63) / 64, 1);
    k_gemm_generic<G><<<grid, kThreads, 0, s>>>(A, B, C, M, N, K, 0, 0, status);
    return cudaGetLastError();
  }
};

template <int G>
struct RunAdamwFused {
  static cudaError_t run(const Plan& p, void* const* ptr, cudaStream_t s) {
    AdamwBatch a;
    a.codes = static_cast<const uint32_t*>(ptr[0]);
    a.books = static_cast<const float*>(ptr[1]);
    a.coefs = static_cast<const float*>(ptr[2]);
    a.words = packed_words(p.m, G);
    a.n = uint32_t(p.m);
    uint32_t* status = static_cast<uint32_t*>(ptr[7]);
    const uint64_t vectors = (p.m + G - 1) / G;
    if (p.op == Op::AdamwSample) {
      const uint64_t items = uint64_t(p.aux0) * G;
      dim3 grid(std::max<uint32_t>(1, std::min<uint32_t>(uint32_t((items + kThreads - 1) / kThreads), 64)), p.batch);
      k_adamw_sample<G><<<grid, kThreads, 0, s>>>(a, static_cast<const uint32_t*>(ptr[3]), p.aux0,
                                                   static_cast<float*>(ptr[5]), status);
      return cudaGetLastError();
    }
    if (p.op == Op::AdamwUsage) {
      cudaError_t err = cudaMemsetAsync(ptr[5], 0, 16 * sizeof(uint32_t), s);
      if (err != cudaSuccess) return err;
      const uint32_t grid = uint32_t((p.m / G + kThreads - 1) / kThreads);
      BookSlot slot(s, ptr[3], 1, G);
      if (slot.error() != cudaSuccess) return slot.error();
      uint32_t* out = static_cast<uint32_t*>(ptr[5]);
#define ACK_LAUNCH_USAGE(S) k_adamw_usage<G, S><<<grid, kThreads, 0, s>>>(a, p.aux1, p.aux0, out, status)
      ACK_SLOT_SWITCH(slot.index(), ACK_LAUNCH_USAGE)
#undef ACK_LAUNCH_USAGE
      const cudaError_t e = cudaGetLastError();
      const cudaError_t r = slot.release();
      return e != cudaSuccess ? e : r;
    }
    cudaError_t err = cudaMemsetAsync(ptr[6], 0, size_t(p.batch) * sizeof(uint32_t), s);
    if (err != cudaSuccess) return err;
    const uint32_t grid = uint32_t((vectors + kThreads - 1) / kThreads);
    const float* new_books = static_cast<const float*>(ptr[3]);
    uint32_t* out = static_cast<uint32_t*>(ptr[5]);
    uint32_t* changed = static_cast<uint32_t*>(ptr[6]);
    for (uint32_t e = 0; e < p.batch; ++e) {
      BookSlot slot(s, new_books + uint64_t(e) * 3 * 16 * G, 3, G);
      if (slot.error() != cudaSuccess) return slot.error();
#define ACK_LAUNCH_ADAMW(S) k_adamw_encode<G, S><<<grid, kThreads, 0, s>>>(a, e, out, changed, status)
      ACK_SLOT_SWITCH(slot.index(), ACK_LAUNCH_ADAMW)
#undef ACK_LAUNCH_ADAMW
      const cudaError_t le = cudaGetLastError();
      const cudaError_t r = slot.release();
      if (le != cudaSuccess) return le;
      if (r != cudaSuccess) return r;
    }
    return cudaSuccess;
  }
};

// Ops 24 and 25, defined with the shared-memory book access at the end of this file.
cudaError_t run_adamw_fit(const Plan& p, void* const* ptr, cudaStream_t s);
cudaError_t run_fit_values(const Plan& p, void* const* ptr, cudaStream_t s);

}  // namespace

cudaError_t launch(const Plan& p, void* const* ptr, cudaStream_t s) {
  const uint32_t g = p.group;
  if (p.schema == 1) {
    switch (p.op) {
      case Op::Encode:
        return by_group<RunEncode>(g, static_cast<const float*>(ptr[0]), p.m, static_cast<const float*>(ptr[1]),
                                   static_cast<uint32_t*>(ptr[4]), static_cast<uint32_t*>(ptr[5]), s);
      case Op::Decode:
        return by_group<RunDecode>(g, static_cast<const uint32_t*>(ptr[0]), static_cast<const float*>(ptr[1]),
                                   static_cast<float*>(ptr[4]), p.m, static_cast<uint32_t*>(ptr[5]), s);
      case Op::Matmul:
        return by_group<RunMatmulExact>(g, p, ptr, s);
      case Op::AdamW:
        k_adamw<<<grid_for(p.m), kThreads, 0, s>>>(static_cast<const uint32_t*>(ptr[0]),
                                                   static_cast<const float*>(ptr[1]), static_cast<const float*>(ptr[2]),
                                                   static_cast<float*>(ptr[4]), uint32_t(p.m), g,
                                                   static_cast<uint32_t*>(ptr[5]));
        return cudaGetLastError();
      default:
        return cudaErrorInvalidValue;
    }
  }
  switch (p.op) {
    case Op::Dense: return by_group<RunDense>(g, p, ptr, s);
    case Op::Coded: return by_group<RunCoded>(g, p, ptr, s);
    case Op::AdamwSample:
    case Op::AdamwUsage:
    case Op::AdamwEncode: return by_group<RunAdamwFused>(g, p, ptr, s);
    case Op::EncodeLarge:
      return by_group<RunEncode>(g, static_cast<const float*>(ptr[0]), p.m, static_cast<const float*>(ptr[1]),
                                 static_cast<uint32_t*>(ptr[5]), static_cast<uint32_t*>(ptr[7]), s);
    case Op::DecodeLarge:
      return by_group<RunDecode>(g, static_cast<const uint32_t*>(ptr[0]), static_cast<const float*>(ptr[1]),
                                 static_cast<float*>(ptr[5]), p.m, static_cast<uint32_t*>(ptr[7]), s);
    case Op::Fit:
      if (!aligned16(ptr[4])) return cudaErrorMisalignedAddress;  // the gathered sample is read in quads
      return run_fit_values(p, ptr, s);
    case Op::AdamwFit:
      if (!aligned16(ptr[3])) return cudaErrorMisalignedAddress;  // sample rows are read in 16-byte quads
      return run_adamw_fit(p, ptr, s);
    case Op::RepackTile32: {
      if (!aligned16(ptr[0]) || !aligned16(ptr[5])) return cudaErrorMisalignedAddress;
      const uint32_t T = uint32_t(p.k / g);
      const uint64_t src_units = packed_bytes(p.m * p.k, g) / 16, dst_units = tile32_bytes(p.m, p.k, g) / 16;
      k_repack_tile32<<<grid_for(dst_units * p.batch), kThreads, 0, s>>>(
          static_cast<const uint4*>(ptr[0]), static_cast<uint4*>(ptr[5]), uint32_t(p.m), T, src_units, dst_units,
          p.batch);
      return cudaGetLastError();
    }
    default:
      return cudaErrorInvalidValue;
  }
}

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

constexpr int kStaticMetaOffset = 16 * 32;                       // floats
constexpr int kStaticBookFloats = kStaticMetaOffset + kMetaFloats;  // 544 per book
static __device__ __align__(256) float g_static_scratch[kStaticEncodeBooks * kStaticBookFloats];

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
  static float* addr[64] = {};
  int dev = 0;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
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

// ------------------------------------------------- codebook fit on the device --
// fit_codebook (vq.py:182-257) for W', M', V' of a VQAdamW step, warm-started
// from the current books, bit for bit the CPU fit on the same sample:
//   assign  the sample's nearest entries (the certified search, book in
//           shared memory), entry counts, and whether the kept-entry rule
//           needs the whole tensor (warm start, sample smaller than the
//           tensor, an empty entry that no lower row duplicates)
//   usage   entries the whole updated tensor selects, only where needed
//   update  each entry with a sample vector: the float64 mean of its
//           vectors summed in sample order (numpy's mean over axis 0),
//           rounded to float32; each other entry not kept: the sample vector
//           farthest from the book as updated so far (float64 squared
//           distances summed in numpy's pairwise order, first maximum)
// One block per fitted book (problem p = expert * 3 + state).
namespace {

struct FitArgs {
  AdamwBatch a;
  const float* samples;  // [E][3][S][G]
  uint32_t S;
  float* books;          // [E][3][16][G]: the books being fitted
  unsigned char* ws;     // per problem: idx[S padded] | counts[16] | usage[16] | flag
  uint64_t stride;       // workspace bytes per problem
  uint32_t warm;         // warm start: the kept-entry rule applies
};

__device__ __forceinline__ uint8_t* fit_idx(const FitArgs& f, uint32_t p) { return f.ws + uint64_t(p) * f.stride; }
__device__ __forceinline__ uint32_t* fit_words(const FitArgs& f, uint32_t p) {
  return reinterpret_cast<uint32_t*>(f.ws + uint64_t(p) * f.stride + (uint64_t(f.S) + 15) / 16 * 16);
}  // [0..16) counts, [16..32) usage, [32] flag

// The row-major 16 x G book `book` into the block's shared SBook (values
// pair-interleaved, BookMeta by warp 0); ends with a barrier.
template <int G>
__device__ void sbook_stage(const float* __restrict__ book) {
  float* dst = reinterpret_cast<float*>(s_static_book);
  for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) dst[book_pos<G>(i / G, i % G)] = book[i];
  if (threadIdx.x < 32) meta_compute<G>(book, *reinterpret_cast<BookMeta*>(dst + kStaticMetaOffset));
  __syncthreads();
}

template <int G>
__global__ void k_fit_init(const float* __restrict__ books_in, float* __restrict__ books, uint32_t problems) {
  const uint32_t p = blockIdx.x, e = p / 3, w = p % 3;
  for (int i = threadIdx.x; i < 16 * G; i += blockDim.x)
    books[uint64_t(p) * 16 * G + i] = books_in[(uint64_t(e) * 4 + w) * 16 * G + i];
}

template <int G>
__global__ void __launch_bounds__(256, 2) k_fit_assign(FitArgs f, uint64_t complete, uint32_t* __restrict__ status) {
  using Book = SBook<G>;
  __shared__ uint32_t cnt[16];
  const uint32_t p = blockIdx.x;
  if (threadIdx.x < 16) cnt[threadIdx.x] = 0;
  sbook_stage<G>(f.books + uint64_t(p) * 16 * G);
  uint8_t* idx = fit_idx(f, p);
  uint32_t bits = Book::bad() ? kNonfinite : 0u;
  for (uint32_t i = threadIdx.x; i < f.S; i += blockDim.x) {
    asm volatile("" ::: "memory");  // re-read the book from shared memory each vector (no hoisting into registers)
    const float* src = f.samples + (uint64_t(p) * f.S + i) * G;
    float x[G];
#pragma unroll
    for (int q = 0; q < G / 4; ++q) {
      const float4 t = reinterpret_cast<const float4*>(src)[q];
      x[4 * q] = t.x;
      x[4 * q + 1] = t.y;
      x[4 * q + 2] = t.z;
      x[4 * q + 3] = t.w;
    }
    bool certified;
    const uint32_t e = enc_vector<G, Book>(x, &certified, src);
    if (certified)
      for (int j = 0; j < G; ++j) bits |= finite32(src[j]) ? 0u : kNonfinite;
    idx[i] = uint8_t(e);
    atomicAdd(&cnt[e], 1u);
  }
  flag_warp(status, bits);
  __syncthreads();
  uint32_t* words = fit_words(f, p);
  if (threadIdx.x < 16) {
    words[threadIdx.x] = cnt[threadIdx.x];
    words[16 + threadIdx.x] = 0;  // usage, filled by k_fit_usage when needed
  }
  if (threadIdx.x == 0) {
    uint32_t empty = 0;
    for (int e = 0; e < 16; ++e) empty |= cnt[e] ? 0u : (1u << e);
    const uint32_t reachable = empty & Book::uniq();
    words[32] = (f.warm && f.S < complete && reachable) ? 1u : 0u;
  }
}

template <int G>
__global__ void __launch_bounds__(256, 2) k_fit_usage(FitArgs f, uint32_t* __restrict__ status) {
  using Book = SBook<G>;
  const uint32_t p = blockIdx.y, e = p / 3, w = p % 3;
  uint32_t* words = fit_words(f, p);
  if (!words[32]) return;  // the whole block: this book keeps no entry
  __shared__ float sbooks[4 * 16 * G];
  __shared__ uint32_t hist[16];
  for (int i = threadIdx.x; i < 64 * G; i += blockDim.x) sbooks[i] = f.a.books[uint64_t(e) * 64 * G + i];
  if (threadIdx.x < 16) hist[threadIdx.x] = 0;
  sbook_stage<G>(f.books + uint64_t(p) * 16 * G);
  const AdamwCoefs k = load_coefs(f.a.coefs + 7 * e);
  const uint64_t full = f.a.n / G;
  uint32_t bits = k.status;
  if (!k.status) {
    for (uint64_t v = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < full; v += uint64_t(gridDim.x) * blockDim.x) {
      asm volatile("" ::: "memory");  // the book stays in shared memory
      float x[G];
      adamw_vector<G>(f.a, sbooks, k, e, v, G, int(w), x, &bits);
      bool certified;
      atomicAdd(&hist[enc_vector<G, Book>(x, &certified)], 1u);
    }
  }
  flag_warp(status, bits);
  __syncthreads();
  if (threadIdx.x < 16 && hist[threadIdx.x]) atomicAdd(words + 16 + threadIdx.x, hist[threadIdx.x]);
}

// sum over j of (s_j - b_j)^2 in float64, in numpy's pairwise order for G
// contiguous values: eight running sums, then a fixed tree.
template <int G>
__device__ __forceinline__ double fit_gap(const float* __restrict__ s, const float* __restrict__ b) {
  double r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const double d = __dsub_rn(double(s[j]), double(b[j]));
    r[j] = __dmul_rn(d, d);
  }
#pragma unroll
  for (int i = 8; i < G; i += 8)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const double d = __dsub_rn(double(s[i + j]), double(b[i + j]));
      r[j] = __dadd_rn(r[j], __dmul_rn(d, d));
    }
  return __dadd_rn(__dadd_rn(__dadd_rn(r[0], r[1]), __dadd_rn(r[2], r[3])),
                   __dadd_rn(__dadd_rn(r[4], r[5]), __dadd_rn(r[6], r[7])));
}

// Dynamic shared memory: S u16 sample indices, grouped by nearest entry in
// sample order (a stable counting sort), so each entry's mean reads only its
// own vectors.
template <int G>
__global__ void __launch_bounds__(512) k_fit_update(FitArgs f) {
  __shared__ float book[16 * G], mean[16 * G];
  __shared__ uint32_t cnt[16], kept, base[17];
  __shared__ double red_gap[16];
  __shared__ uint32_t red_idx[16];
  extern __shared__ uint16_t order[];
  const uint32_t p = blockIdx.x, warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  float* out = f.books + uint64_t(p) * 16 * G;
  for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) book[i] = out[i];
  const uint32_t* words = fit_words(f, p);
  if (threadIdx.x < 16) cnt[threadIdx.x] = words[threadIdx.x];
  if (threadIdx.x == 0) {
    uint32_t k = 0;
    if (words[32])
      for (int e = 0; e < 16; ++e) k |= words[16 + e] ? (1u << e) : 0u;
    kept = k;
  }
  __syncthreads();
  const float* sample = f.samples + uint64_t(p) * f.S * G;
  // stable counting sort of the sample by nearest entry (warp 0, 32 at a time)
  if (warp == 0) {
    if (lane == 0) {
      uint32_t run = 0;
      for (int e = 0; e < 16; ++e) {
        base[e] = run;
        run += cnt[e];
      }
      base[16] = run;
    }
    __syncwarp();
    const uint8_t* idx = fit_idx(f, p);
    const uint32_t below = (1u << lane) - 1u;
    for (uint32_t c = 0; c < f.S; c += 32) {
      const uint32_t i = c + lane;
      const uint32_t e = i < f.S ? idx[i] : 16u;
      const uint32_t peers = __match_any_sync(0xffffffffu, e);
      const uint32_t at = base[e] + __popc(peers & below);
      if (e < 16) order[at] = uint16_t(i);
      __syncwarp();
      if (e < 16 && (peers & below) == 0) base[e] += __popc(peers);  // the group's lowest lane
      __syncwarp();
    }
  }
  __syncthreads();
  // means: warp = entry, lane = component, its vectors in sample order
  {
    const uint32_t e = warp, n = cnt[e];
    if (lane < G && n) {
      const uint16_t* mine = order + (base[e] - n);  // base[e] now ends entry e's run
      double s = 0.0;
      for (uint32_t k = 0; k < n; ++k) s = __dadd_rn(s, double(sample[uint64_t(mine[k]) * G + lane]));
      mean[e * G + lane] = __double2float_rn(__ddiv_rn(s, double(n)));
    }
  }
  __syncthreads();
  for (int e = 0; e < 16; ++e) {  // in entry order: a reseed sees the entries before it updated
    if (cnt[e]) {
      if (threadIdx.x < G) book[e * G + threadIdx.x] = mean[e * G + threadIdx.x];
      __syncthreads();
    } else if (!((kept >> e) & 1u)) {
      double best = -1.0;
      uint32_t at = 0xffffffffu;
      for (uint32_t i = threadIdx.x; i < f.S; i += blockDim.x) {
        double gap = fit_gap<G>(sample + uint64_t(i) * G, book);
#pragma unroll 1
        for (int c = 1; c < 16; ++c) gap = fmin(gap, fit_gap<G>(sample + uint64_t(i) * G, book + c * G));
        if (gap > best) {
          best = gap;
          at = i;
        }
      }
      // the first maximum over the block: larger gap, then the lower index
      for (int o = 16; o; o >>= 1) {
        const double og = __shfl_xor_sync(0xffffffffu, best, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, at, o);
        if (og > best || (og == best && oi < at)) {
          best = og;
          at = oi;
        }
      }
      if (lane == 0) {
        red_gap[warp] = best;
        red_idx[warp] = at;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int w = 1; w < 16; ++w)
          if (red_gap[w] > red_gap[0] || (red_gap[w] == red_gap[0] && red_idx[w] < red_idx[0])) {
            red_gap[0] = red_gap[w];
            red_idx[0] = red_idx[w];
          }
      }
      __syncthreads();
      if (threadIdx.x < G) book[e * G + threadIdx.x] = sample[uint64_t(red_idx[0]) * G + threadIdx.x];
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) out[i] = book[i];
}

inline size_t fit_update_smem(uint32_t S) { return (size_t(S) * 2 + 15) / 16 * 16; }

template <int G>
cudaError_t fit_update_attr(uint32_t S) {
  return cudaFuncSetAttribute(k_fit_update<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(fit_update_smem(S)));
}

template <int G>
cudaError_t run_fit_group(const Plan& p, void* const* ptr, cudaStream_t s) {
  FitArgs f;
  f.a.codes = static_cast<const uint32_t*>(ptr[0]);
  f.a.books = static_cast<const float*>(ptr[1]);
  f.a.coefs = static_cast<const float*>(ptr[2]);
  f.a.words = packed_words(p.m, G);
  f.a.n = uint32_t(p.m);
  f.samples = static_cast<const float*>(ptr[3]);
  f.S = p.aux0;
  f.ws = static_cast<unsigned char*>(ptr[4]);
  f.stride = fit_workspace_stride(p.aux0);
  f.books = static_cast<float*>(ptr[5]);
  f.warm = 1;
  uint32_t* status = static_cast<uint32_t*>(ptr[7]);
  const uint32_t problems = p.batch * 3;
  const uint64_t complete = p.m / G;
  cudaError_t err = fit_update_attr<G>(f.S);
  if (err != cudaSuccess) return err;
  k_fit_init<G><<<problems, 128, 0, s>>>(f.a.books, f.books, problems);
  const uint32_t usage_blocks =
      uint32_t(std::max<uint64_t>(1, std::min<uint64_t>((complete + 255) / 256, uint64_t(sm_count()) * 4)));
  for (uint32_t it = 0; it < p.aux1; ++it) {
    k_fit_assign<G><<<problems, 256, 0, s>>>(f, complete, status);
    k_fit_usage<G><<<dim3(usage_blocks, problems), 256, 0, s>>>(f, status);
    k_fit_update<G><<<problems, 512, fit_update_smem(f.S), s>>>(f);
  }
  return cudaGetLastError();
}

cudaError_t run_adamw_fit(const Plan& p, void* const* ptr, cudaStream_t s) {
  if (p.group == 8) return run_fit_group<8>(p, ptr, s);
  if (p.group == 16) return run_fit_group<16>(p, ptr, s);
  return run_fit_group<32>(p, ptr, s);
}

// Op 25: one tensor's fit. The sample is gathered into the workspace; the
// book starts from the caller's (warm) or from 16 sample rows (cold).
template <int G>
__global__ void k_fit_gather(const float* __restrict__ values, const uint32_t* __restrict__ positions, uint32_t S,
                             float* __restrict__ sample) {
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < uint64_t(S) * G;
       i += uint64_t(gridDim.x) * blockDim.x)
    sample[i] = values[uint64_t(positions[i / G]) * G + i % G];
}

template <int G>
__global__ void k_fit_start(const float* __restrict__ init, const float* __restrict__ sample,
                            const uint32_t* __restrict__ rows, float* __restrict__ book) {
  for (int i = threadIdx.x; i < 16 * G; i += blockDim.x)
    book[i] = init ? init[i] : sample[uint64_t(rows[i / G]) * G + i % G];
}

// Entries the whole tensor's complete vectors select with the current book
// (the kept-entry rule), where the assign pass asked for it.
template <int G>
__global__ void __launch_bounds__(256, 2) k_fit_usage_values(FitArgs f, const float* __restrict__ values, uint64_t full,
                                                          uint32_t* __restrict__ status) {
  using Book = SBook<G>;
  uint32_t* words = fit_words(f, 0);
  if (!words[32]) return;
  __shared__ uint32_t hist[16];
  if (threadIdx.x < 16) hist[threadIdx.x] = 0;
  sbook_stage<G>(f.books);
  uint32_t bits = 0;
  for (uint64_t v = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < full; v += uint64_t(gridDim.x) * blockDim.x) {
    asm volatile("" ::: "memory");  // the book stays in shared memory
    float x[G];
#pragma unroll
    for (int j = 0; j < G; ++j) x[j] = values[v * G + j];
    bool certified;
    const uint32_t e = enc_vector<G, Book>(x, &certified, values + v * G);
    if (certified)
      for (int j = 0; j < G; ++j) bits |= finite32(values[v * G + j]) ? 0u : kNonfinite;
    atomicAdd(&hist[e], 1u);
  }
  flag_warp(status, bits);
  __syncthreads();
  if (threadIdx.x < 16 && hist[threadIdx.x]) atomicAdd(words + 16 + threadIdx.x, hist[threadIdx.x]);
}

template <int G>
cudaError_t run_fit_values_group(const Plan& p, void* const* ptr, cudaStream_t s) {
  const float* values = static_cast<const float*>(ptr[0]);
  const float* init = (p.flags & 1u) ? static_cast<const float*>(ptr[1]) : nullptr;
  const uint32_t* positions = static_cast<const uint32_t*>(ptr[2]);
  unsigned char* ws = static_cast<unsigned char*>(ptr[4]);
  const uint32_t S = p.aux0;
  const uint64_t sample_bytes = uint64_t(S) * G * 4;  // a multiple of 16
  FitArgs f{};
  f.samples = reinterpret_cast<const float*>(ws);
  f.S = S;
  f.books = static_cast<float*>(ptr[5]);
  f.ws = ws + sample_bytes;
  f.stride = fit_workspace_stride(S);
  f.warm = init ? 1u : 0u;
  uint32_t* status = static_cast<uint32_t*>(ptr[7]);
  const uint64_t full = p.m / G;
  cudaError_t err = fit_update_attr<G>(S);
  if (err != cudaSuccess) return err;
  k_fit_gather<G><<<grid_for(uint64_t(S) * G), kThreads, 0, s>>>(values, positions, S, reinterpret_cast<float*>(ws));
  k_fit_start<G><<<1, 256, 0, s>>>(init, f.samples, positions + S, f.books);
  const uint32_t usage_blocks =
      uint32_t(std::max<uint64_t>(1, std::min<uint64_t>((full + 255) / 256, uint64_t(sm_count()) * 4)));
  for (uint32_t it = 0; it < p.aux1; ++it) {
    k_fit_assign<G><<<1, 256, 0, s>>>(f, full, status);
    k_fit_usage_values<G><<<usage_blocks, 256, 0, s>>>(f, values, full, status);
    k_fit_update<G><<<1, 512, fit_update_smem(f.S), s>>>(f);
  }
  return cudaGetLastError();
}

cudaError_t run_fit_values(const Plan& p, void* const* ptr, cudaStream_t s) {
  if (p.group == 8) return run_fit_values_group<8>(p, ptr, s);
  if (p.group == 16) return run_fit_values_group<16>(p, ptr, s);
  return run_fit_values_group<32>(p, ptr, s);
}

}  // namespace

}  // namespace ack
