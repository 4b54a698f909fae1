// vq4 codec kernels and their launchers: decode, encode (tensor-core and
// CUDA-core paths), the shader AdamW (op 3) and the fused coded-state AdamW
// passes. The only unit that reads the constant-bank codebook slots.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <mutex>

#define ACK_VQ_CONSTANT_BOOKS
#include "vq_common.cuh"
#include "vq_tc.cuh"

namespace ack {
namespace {

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
// joins its warp's queue and is refined later: enc_vector's FP32 filter over
// all 16 entries (its bound kappa2 = (G + 8) 2^-23), then the float64 pass
// over what survives, the result OR-ed into the zero nibble the first pass
// stored. Nonfinite input or books take the float64 pass at once.
//
// Schedule. A consumer warp takes its quad's tiles in turn: it loads a pair
// of sub-tiles' accumulators under one wait, releases the stage and the
// accumulator once the tile's last loads have landed (so the next TMA load
// and MMA run while it certifies), certifies the pair in one branch-free
// block, then stores the code words. A quad's four warps flush their queues
// at the same tiles.
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

using namespace ::ack::tc;  // the primitives of vq_tc.cuh

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
  // queue ring per warp: flushed whenever it holds more than kCap - 32 H, so
  // one tile's deferrals always fit; on smooth data a scheduled flush (every
  // kFlush of the quad's tiles) finds 50-70 entries
  static constexpr uint32_t kCap = 256u;
  static constexpr uint32_t kFlush = 32;
  // dynamic shared memory: 1024-byte alignment slack, the ring, the tf32
  // book tile (kN rows, at most 4 KB)
  static constexpr size_t kSmem = 1024 + size_t(S) * kTile + 4096;
};

// Deferred FP32 refinement of `count` (<= 32) queued vectors, one per lane,
// ring positions head + lane: x read again from memory, then enc_vector (the
// FP32 filter over all 16 entries with its bound, packed FMAs against the
// constant-bank book, no divergence across lanes) and its float64 pass if
// more than one entry survives; the index is OR-ed into the zero nibble the
// filter pass stored.
template <int G, class Book, uint32_t kCap>
__device__ __noinline__ void refine_queue(const float* __restrict__ x, uint32_t* __restrict__ codes,
                                          const uint32_t* qv, uint32_t head, uint32_t count, uint32_t lane) {
  __syncwarp();  // the nibble stores of the filter pass come first
  if (lane < count) {
    const uint64_t v = qv[(head + lane) & (kCap - 1)];
    const float* src = x + v * G;
    float xr[G];
#pragma unroll
    for (int kc = 0; kc < G / 4; ++kc) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(src) + kc);
      xr[4 * kc] = t.x;
      xr[4 * kc + 1] = t.y;
      xr[4 * kc + 2] = t.z;
      xr[4 * kc + 3] = t.w;
    }
    bool exact;
    const uint32_t idx = enc_vector<G, Book, true>(xr, &exact, src);
    if (idx) atomicOr(codes + v / 8, idx << (4 * uint32_t(v % 8)));
  }
  __syncwarp();
}

}  // namespace tc

template <int G, int SLOT>
__global__ void __launch_bounds__(tc::Cfg<G>::kThreads, tc::Cfg<G>::kBlocksPerSm)
    k_encode_tc(const __grid_constant__ CUtensorMap tmap, const float* __restrict__ x, uint64_t n,
                uint32_t* __restrict__ codes, uint32_t* __restrict__ status, uint32_t stall_test) {
  using Book = CBook<G, SLOT, 0>;
  using W = tc::Swz<G>;
  using K = tc::Cfg<G>;
  constexpr int S = K::S, C = K::C, H = K::H, kChunks = G / 4;
  constexpr uint32_t kCap = K::kCap;
  extern __shared__ unsigned char tc_smem[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem) + 1023) & ~uintptr_t(1023));
  unsigned char* ring = base;
  unsigned char* bmat = base + S * K::kTile;             // 16 tf32 book rows, swizzled
  __shared__ __align__(8) uint64_t full[S], sfree[S], done[C], afree[C];
  __shared__ uint32_t tmem_base;
  __shared__ uint32_t q_vec[4 * C][kCap];  // vector indices (below 2^31 on this path)
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
    // consumers arrive once per warp (a quad's four warps): per-lane
    // arrivals on one mbarrier serialise
    for (int s = 0; s < S; ++s) {
      tc::mb_init(&full[s], 1);
      tc::mb_init(&sfree[s], 4 + 1);  // the owning quad's reads and the MMA's completion
    }
    for (int b = 0; b < C; ++b) {
      tc::mb_init(&done[b], 1);
      tc::mb_init(&afree[b], 4);
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
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor core
  }
  if (blockIdx.x == 0 && tid == 0 && Book::bad()) atomicOr(status, kNonfinite);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  bool ok = true;
  // stall_test (host-injected, test only): 1 = the producer issues no load,
  // 2 = the consumers take no accumulator; the pipeline waits then run out
  // after kTestPolls, set kStalled, and the drains below still complete
  const uint32_t lim = stall_test ? tc::kTestPolls : tc::kPolls;

  if (warp == 4 * C) {
    // producer: one TMA tensor load (two for 512-row tiles) per tile
    if (lane == 0) {
      uint32_t issued = 0;
      for (uint32_t k = 0; k < T && ok && stall_test != 1; ++k) {
        const uint32_t s = k % S;
        if (k >= S && !(ok = tc::mb_wait(&sfree[s], ((k / S) - 1) & 1, lim))) break;
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
      uint32_t committed = 0;
      for (uint32_t k = 0; k < T && ok; ++k) {
        const uint32_t s = k % S, q = k % C;
        if (!(ok = tc::mb_wait(&full[s], (k / S) & 1, lim))) break;
        if (k >= C && !(ok = tc::mb_wait(&afree[q], ((k / C) - 1) & 1, lim))) break;
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
        ++committed;
      }
      if (!ok) atomicOr(status, kStalled);
      // Every committed MMA completes before TMEM is released, on the stall
      // path too. Batch k was issued only after batch k - C's accumulator was
      // freed (so its done phase had completed): done[k % C] is at batch k's
      // phase or one past it, and its parity names that phase unambiguously.
      for (uint32_t k = committed > uint32_t(C) ? committed - C : 0u; k < committed; ++k)
        if (!tc::mb_wait(&done[k % C], (k / C) & 1)) atomicOr(status, kStalled);
    }
  } else {
    // consumer quad q: TMEM lanes 32 (warp % 4) .. + 31, one vector per lane per sub-tile
    const uint32_t q = warp / 4, row = tid & 127, wq = warp & 3;
    constexpr float kappa1 = 1.0f / 1024 + 1.0f / 2048 + float(G + 8) / 2097152.0f;
    constexpr float kappa_t = float(G + 9) / 2097152.0f;  // TIGHT: all but the x residual
    uint32_t qhead = 0, qtail = 0;
    constexpr uint32_t kChunk = 32u;  // queued vectors refined together (one per lane)
    uint32_t bits = 0;                // nonfinite inputs seen, flagged once when the warp is done
    for (uint32_t k = q; k < T && ok && stall_test != 2; k += C) {
      const uint32_t s = k % S;
      const uint64_t vtile = (blockIdx.x + uint64_t(k) * gridDim.x) * 128 * H;  // the tile's first vector
      // warp-uniform outcomes: tcgen05.ld below is .sync.aligned
      if (!(ok = __all_sync(0xffffffffu, tc::mb_wait(&full[s], (k / S) & 1, lim)))) break;
      if (!(ok = __all_sync(0xffffffffu, tc::mb_wait(&done[q], (k / C) & 1, lim)))) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      // sub-tiles are read in pairs: both accumulators' loads are in flight
      // under one wait, and the two certificates interleave
      constexpr int HP = H >= 2 ? 2 : 1;
#pragma unroll
      for (int h0 = 0; h0 < H; h0 += HP) {
        uint32_t r[HP][K::kN];
        float2 n2[HP], r2[HP];
#pragma unroll
        for (int hp = 0; hp < HP; ++hp) {
          const uint32_t taddr = tmem + ((wq * 32u) << 16) + (q * H + h0 + hp) * K::kN;
          tc::tmem_ld16(r[hp], taddr);
          if constexpr (K::TIGHT) tc::tmem_ld16(r[hp] + 16, taddr + 16u);
          // ||x||^2 in enc_vector's order, from the swizzled tile (conflict-free);
          // TIGHT also ||x - trunc(x)||^2, x truncated to its top 19 bits: the
          // tensor core's operand is that or the nearer tf32 neighbour, so this
          // bounds its residual either way
          const unsigned char* tile = ring + s * K::kTile + (h0 + hp) * K::kSub;
          n2[hp] = r2[hp] = make_float2(0.f, 0.f);
#pragma unroll
          for (int kc = 0; kc < kChunks; ++kc) {
            const float4 t = *reinterpret_cast<const float4*>(tile + W::off(row, kc));
            n2[hp] = __ffma2_rn(make_float2(t.x, t.y), make_float2(t.x, t.y), n2[hp]);
            n2[hp] = __ffma2_rn(make_float2(t.z, t.w), make_float2(t.z, t.w), n2[hp]);
            if constexpr (K::RESID) {
              const float2 a = make_float2(t.x - __uint_as_float(__float_as_uint(t.x) & 0xFFFFE000u),
                                           t.y - __uint_as_float(__float_as_uint(t.y) & 0xFFFFE000u));
              const float2 b = make_float2(t.z - __uint_as_float(__float_as_uint(t.z) & 0xFFFFE000u),
                                           t.w - __uint_as_float(__float_as_uint(t.w) & 0xFFFFE000u));
              r2[hp] = __ffma2_rn(a, a, r2[hp]);
              r2[hp] = __ffma2_rn(b, b, r2[hp]);
            }
          }
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (h0 + HP == H) {
          // the tile's accumulator and stage are read (TMEM into registers,
          // the norms from the tile): release both now, so the next load and
          // MMA into them run while this warp certifies
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            tc::mb_arrive(&afree[q]);
            tc::mb_arrive(&sfree[s]);
          }
        }
        // the pair's certificates: all arithmetic first, in one branch-free
        // block, so the two vectors' dependency chains interleave
        uint32_t cand[HP];
        bool clean[HP];
#pragma unroll
        for (int hp = 0; hp < HP; ++hp) {
          if constexpr (K::TIGHT) {
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const float2 t = __fadd2_rn(make_float2(__uint_as_float(r[hp][e]), __uint_as_float(r[hp][e + 1])),
                                          make_float2(__uint_as_float(r[hp][16 + e]), __uint_as_float(r[hp][17 + e])));
              r[hp][e] = __float_as_uint(t.x);
              r[hp][e + 1] = __float_as_uint(t.y);
            }
          }
          const float nx = n2[hp].x + n2[hp].y;
          float f[16];
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            const float2 t = __ffma2_rn(make_float2(-2.f, -2.f),
                                        make_float2(__uint_as_float(r[hp][2 * p]), __uint_as_float(r[hp][2 * p + 1])),
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
            eps = fmaf(1.0f / 1024 + kappa_t, nx + Book::cmax2(), 0x1p-118f);
          } else if constexpr (K::RESID) {
            // 2 ||r|| max||c|| (rounded up, 2^-16 margin for the FP32 sum of
            // squares) + the accumulation, book-remainder, rounding and
            // flushed-subnormal terms
            const float rc = __fsqrt_ru(__fmul_ru(r2[hp].x + r2[hp].y, Book::cmax2()));
            eps = fmaf(2.0f + 0x1p-15f, rc, fmaf(kappa_t, nx + Book::cmax2(), 0x1p-118f));
          } else {
            eps = fmaf(kappa1, nx + Book::cmax2(), 0x1p-118f);
          }
          const float thr = fmaf(2.f, eps, fb);
          // f_e <= thr as the sign of thr - f_e (one packed FMA a pair; the
          // sign of a rounded difference is exact, and a zero difference is
          // +0 since thr = fb + 2 eps with eps > 0 is never -0), the 16 sign
          // bits collected by funnel shifts in two chains of 8: bit e of
          // `over` is set iff f_e > thr. A NaN f_e leaves `clean` false, so
          // its unspecified sign never counts.
          uint32_t over_lo = 0, over_hi = 0;
#pragma unroll
          for (int p = 3; p >= 0; --p) {
            const float2 d = __ffma2_rn(make_float2(f[2 * p], f[2 * p + 1]), make_float2(-1.f, -1.f),
                                        make_float2(thr, thr));
            over_lo = __funnelshift_l(__float_as_uint(d.y), over_lo, 1);
            over_lo = __funnelshift_l(__float_as_uint(d.x), over_lo, 1);
            const float2 u = __ffma2_rn(make_float2(f[2 * p + 8], f[2 * p + 9]), make_float2(-1.f, -1.f),
                                        make_float2(thr, thr));
            over_hi = __funnelshift_l(__float_as_uint(u.y), over_hi, 1);
            over_hi = __funnelshift_l(__float_as_uint(u.x), over_hi, 1);
          }
          cand[hp] = ~((over_hi << 8) | over_lo) & Book::uniq();
          clean[hp] = finite32(thr) && finite32(fb) && !Book::bad();
        }
        // then the outcomes: a single candidate is the answer; several are
        // queued for the refinement; the rest (nonfinite input, the partial
        // last vector) take the float64 pass now
        uint32_t idx[HP];
        bool defer[HP];
        const uint64_t vbase0 = vtile + h0 * 128;
#pragma unroll
        for (int hp = 0; hp < HP; ++hp) {
          const uint64_t v = vbase0 + hp * 128 + row;
          const uint32_t c = cand[hp];
          idx[hp] = 0;
          defer[hp] = false;
          if (v < complete) {
            if (clean[hp] && c != 0u && (c & (c - 1u)) == 0u) {
              idx[hp] = uint32_t(__ffs(c) - 1);
            } else if (clean[hp] && c != 0u) {
              defer[hp] = true;
            } else {
              const float* src = x + v * G;
              for (int j = 0; j < G; ++j) bits |= finite32(src[j]) ? 0u : kNonfinite;
              idx[hp] = enc_exact_mem<G, Book>(src, G, clean[hp] ? c : 0xffffu);
            }
          } else if (v < vectors) {
            // the partial last vector: its valid components only (vq.py:171-172)
            const int valid = int(n - v * G);
            const float* src = x + v * G;
            for (int j = 0; j < valid; ++j) bits |= finite32(src[j]) ? 0u : kNonfinite;
            idx[hp] = enc_exact_mem<G, Book>(src, valid, 0xffffu);
          }
        }
#pragma unroll
        for (int hp = 0; hp < HP; ++hp) {
          const uint32_t dm = __ballot_sync(0xffffffffu, defer[hp]);
          if (defer[hp]) {
            const uint32_t pos = (qtail + __popc(dm & ((1u << lane) - 1u))) & (kCap - 1);
            q_vec[warp][pos] = uint32_t(vbase0 + hp * 128 + row);
          }
          qtail += __popc(dm);
        }
        // OR the nibbles of the 8 lanes that share a code word, both vectors'
        // shuffles interleaved
        uint32_t wd[HP];
#pragma unroll
        for (int hp = 0; hp < HP; ++hp) wd[hp] = idx[hp] << (4u * (lane & 7u));
#pragma unroll
        for (int o = 1; o < 8; o <<= 1)
#pragma unroll
          for (int hp = 0; hp < HP; ++hp) wd[hp] |= __shfl_xor_sync(0xffffffffu, wd[hp], o);
#pragma unroll
        for (int hp = 0; hp < HP; ++hp) {
          const uint64_t word = (vbase0 + hp * 128 + wq * 32) / 8 + lane / 8;
          if ((lane & 7) == 0 && word < words) codes[word] = wd[hp];
        }
      }
      // Refine off the pipeline's critical path, kChunk vectors at a time. The
      // four warps of a quad flush at the same tiles (every kFlush of the
      // quad's tiles), so their refinements overlap instead of holding the
      // quad's stages one warp after another; a queue that might not hold
      // the next tile's deferrals flushes at once.
      const uint32_t taken = (k - q) / C + 1;  // tiles this quad has certified
      if (taken % K::kFlush == 0 || qtail - qhead > kCap - 32u * H) {
        while (qtail != qhead) {
          const uint32_t cnt = min(kChunk, qtail - qhead);
          tc::refine_queue<G, Book, kCap>(x, codes, q_vec[warp], qhead, cnt, lane);
          qhead += cnt;
        }
      }
    }
    for (; ok && qtail != qhead; qhead += min(kChunk, qtail - qhead))
      tc::refine_queue<G, Book, kCap>(x, codes, q_vec[warp], qhead, min(kChunk, qtail - qhead), lane);
    flag_warp(status, bits);
    if (!ok) atomicOr(status, kStalled);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(K::kCols));
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

// The constant-bank slots of one device. A launch holds the ring's lock from
// choosing its slot to recording the slot's event. Before its copy into the
// constant bank it makes its stream wait for the latest launch of EVERY slot
// (on whatever streams they ran): CUDA leaves undefined a write to a
// __constant__ variable while any running grid reads it, so no c_books
// reader may still run when the copy lands. Launches on one stream lose
// nothing by this (stream order already holds); launches on several streams
// run their book-reading kernels one after another.
//
// Rings, like the other per-device caches of this file, are kept for the
// life of the process and indexed by the CUDA device ordinal (at most
// kMaxDevices): a device reset (cudaDeviceReset) after first use is not
// supported, since the cached events and symbol addresses belong to the
// context it destroys.
struct SlotRing {
  std::mutex mu;
  uint32_t next = 0;
  cudaEvent_t done[kBookSlots] = {};
};
SlotRing g_rings[kMaxDevices];

// Device address of g_stage, looked up once per device.
float* stage_address(cudaError_t* err) {
  static std::mutex mu;
  static float* addr[kMaxDevices] = {};
  int dev = 0;
  *err = current_device(&dev);
  if (*err != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) *err = cudaGetSymbolAddress(reinterpret_cast<void**>(&addr[dev]), g_stage);
  return *err == cudaSuccess ? addr[dev] : nullptr;
}

// One launch's hold on a slot: waits for every slot's latest user, stages
// `nb` books of group `group` from `src` (device memory) into its slot, and
// on release records the slot's event.
class BookSlot {
 public:
  BookSlot(cudaStream_t stream, const void* src, int nb, uint32_t group) : stream_(stream) {
    int dev = 0;
    err_ = current_device(&dev);
    if (err_ != cudaSuccess) return;
    ring_ = &g_rings[dev];
    lock_ = std::unique_lock<std::mutex>(ring_->mu);
    index_ = int(ring_->next++ % kBookSlots);
    for (int i = 0; i < kBookSlots && err_ == cudaSuccess; ++i)
      if (ring_->done[i]) err_ = cudaStreamWaitEvent(stream, ring_->done[i], 0);
    cudaEvent_t& ev = ring_->done[index_];
    if (err_ == cudaSuccess && !ev) err_ = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
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
    cudaError_t e = cudaSuccess;
    if (ring_ && ring_->done[index_]) e = cudaEventRecord(ring_->done[index_], stream_);
    if (lock_.owns_lock()) lock_.unlock();
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

// The host-injected stall test of the next k_encode_tc launch (test only,
// armed through ack_inject_fault): 0 none, 1 or 2 as the kernel describes.
std::atomic<uint32_t> g_encode_stall_test{0};
uint32_t take_encode_stall_test() { return g_encode_stall_test.exchange(0); }

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
    const uint32_t stall_test = take_encode_stall_test();
#define ACK_LAUNCH_ENCODE(S) \
  k_encode_tc<G, S><<<grid, K::kThreads, K::kSmem, s>>>(map, x, n, codes, status, stall_test)
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


}  // namespace

cudaError_t launch_encode(uint32_t group, const float* x, uint64_t n, const float* book, uint32_t* codes,
                          uint32_t* status, cudaStream_t s) {
  return by_group<RunEncode>(group, x, n, book, codes, status, s);
}

cudaError_t launch_decode(uint32_t group, const uint32_t* codes, const float* book, float* out, uint64_t n,
                          uint32_t* status, cudaStream_t s) {
  return by_group<RunDecode>(group, codes, book, out, n, status, s);
}

cudaError_t launch_adamw_shader(const Plan& p, void* const* ptr, cudaStream_t s) {
  k_adamw<<<grid_for(p.m), kThreads, 0, s>>>(static_cast<const uint32_t*>(ptr[0]), static_cast<const float*>(ptr[1]),
                                             static_cast<const float*>(ptr[2]), static_cast<float*>(ptr[4]),
                                             uint32_t(p.m), p.group, static_cast<uint32_t*>(ptr[5]));
  return cudaGetLastError();
}

cudaError_t launch_adamw_fused(const Plan& p, void* const* ptr, cudaStream_t s) {
  return by_group<RunAdamwFused>(p.group, p, ptr, s);
}

}  // namespace ack

namespace ack {
void set_encode_stall_test(uint32_t mode) { g_encode_stall_test.store(mode); }
}  // namespace ack
