// vq4 product kernels and their launchers: the shader's packed-pair product
// (op 2), dense activations times coded weights (op 16: byte-pair table,
// tile32 and canonical LUT kernels, generic fallback), coded times coded
// (op 17: 16x16 LUT) and the tile32 repack (op 23).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "vq_common.cuh"
#include "vq_kernels.hpp"
#include "vq_tc.cuh"

namespace ack {
namespace {

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
  uint32_t ybits = 0;  // nonfinite outputs (from x, or overflow)
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
              const float v = t0 ? *dst + y : y;
              *dst = v;
              ybits |= finite32(v) ? 0u : kNonfinite;  // a nonfinite partial sum stays nonfinite
            }
          }
        }
        __syncthreads();  // this stage may be overwritten by the next issue
      }
    }
  }
  flag_warp(status, ybits);
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
  uint32_t ybits = 0;  // nonfinite outputs (from x, or overflow)
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
                const float v = t0 ? *dst + y : y;
                *dst = v;
                ybits |= finite32(v) ? 0u : kNonfinite;  // a nonfinite partial sum stays nonfinite
              }
            }
          }
        }
      }
    }
    s0 = s1;
  }
  flag_warp(status, ybits);
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
// cp.async (completion tracked by an mbarrier) while the current one is
// looked up, and the warps that finish their lookups first build the next
// P from them, so only the Q build stands between two segments' lookups
// (two block barriers per segment). Each row sums its 128 pair
// values per chunk in a fixed order (pairs, then a tree over lanes); chunks
// add in order, so the result does not depend on the grid.
namespace pair {

constexpr int kWarps = 16, kThreads = kWarps * 32, kRows = 32;
constexpr uint32_t kQFloats = 128u * 256u;         // the byte table
constexpr uint32_t kPFloats = 256u * 16u + 32u;    // P, one pad word per 8 groups
__device__ __forceinline__ uint32_t p_index(uint32_t t, uint32_t c) { return t * 16u + c + (t >> 3); }

// The book's 16 rows sit G + 4 floats apart in shared memory, so the 16
// threads that each read one row as float4s hit 16 distinct bank quads.
template <int G>
constexpr uint32_t kBookStride = G + 4;

// Table, P and one x-chunk buffer (the next chunk is prefetched into it once
// P is built): 161 KB for g16, so the 164 KB shared-memory configuration
// leaves ~92 KB of L1 for the code loads in flight (the largest carveout
// measured 6% slower).
template <int G>
constexpr size_t smem_bytes() {
  return (size_t(kQFloats) + kPFloats + 256 * G + 16 * kBookStride<G>) * sizeof(float);
}

}  // namespace pair

template <int G, bool ONE>  // ONE: K = 256 G, one chunk (32-word rows, a compile-time stride)
__global__ void __launch_bounds__(pair::kThreads, 1)
    k_dense_pair(const float* __restrict__ X, const uint32_t* __restrict__ codes, const float* __restrict__ books,
                 float* __restrict__ Y, uint32_t N, uint32_t K, uint32_t E, uint64_t words_per_expert,
                 uint32_t* __restrict__ status, const __grid_constant__ PeerY peers) {
  constexpr uint32_t kChunkX = 256u * G, kBook = 16u * G, kBs = pair::kBookStride<G>;
  extern __shared__ __align__(16) float pair_smem[];
  __shared__ uint64_t xfull;  // phase k: the k-th prefetched x chunk and book have landed
  __shared__ uint32_t ptask;  // the next P task of the build under way
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
  if (tid == 0) {
    tc::mb_init(&xfull, pair::kThreads);  // one cp.async arrival per thread per phase
    ptask = 0;
  }
  __syncthreads();

  // the work list: (segment of one expert's units, chunk) in order
  auto seg_end = [&](uint64_t s) { return min(u1, (s / nb + 1) * nb); };
  // every thread copies its share of the x chunk and book of (s, c) into
  // xbuf and arrives on xfull when its copies have landed
  uint32_t xph = 1;  // parity of the last phase prefetched
  auto prefetch = [&](uint64_t s, uint32_t c) {
    const uint32_t e = uint32_t(s / nb);
    float* dst = xbuf;
    const float* xs = X + uint64_t(e) * K + uint64_t(c) * kChunkX;
    const float* bs = books + uint64_t(e) * kBook;
    for (uint32_t i = tid; i < (kChunkX + kBook) / 4; i += pair::kThreads) {
      // x pieces land contiguously; book piece q (row q / (G/4)) at the padded row stride
      const uint32_t q = i - kChunkX / 4;
      const float* src = i < kChunkX / 4 ? xs + 4 * i : bs + 4 * q;
      float* d = i < kChunkX / 4 ? dst + 4 * i : dst + kChunkX + (q / (G / 4)) * kBs + 4 * (q % (G / 4));
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(tc::smem_u32(d)), "l"(src) : "memory");
    }
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(tc::smem_u32(&xfull)) : "memory");
    xph ^= 1u;
  };
  uint32_t ybits = 0;  // nonfinite outputs (from x, or overflow)
  // P[t][e] = x_t . c_e of the last prefetched (segment, chunk), in tasks of
  // 8 groups that any warp takes once its lookups are done: the warps that
  // finish a segment early build the next one's P while the rest look up.
  // `first_unit`: the chunk opens an expert, whose nonfinite book is reported.
  auto build_p = [&](bool first_unit) {
    bool have_book = false;
    float br[G];  // book row lane % 16
    for (;;) {
      uint32_t task = 0;
      if (lane == 0) task = atomicAdd(&ptask, 1u);
      task = __shfl_sync(0xffffffffu, task, 0);
      if (task >= 256u / 8u) break;
      if (!have_book) {
        if (!tc::mb_wait(&xfull, xph) && lane == 0) atomicOr(status, kStalled);
        const float* bk = xbuf + kChunkX + (lane & 15) * kBs;
#pragma unroll
        for (int j = 0; j < G; j += 4) {
          const float4 b4 = *reinterpret_cast<const float4*>(bk + j);
          br[j] = b4.x;
          br[j + 1] = b4.y;
          br[j + 2] = b4.z;
          br[j + 3] = b4.w;
        }
        if (first_unit) {
          uint32_t bits = 0;
#pragma unroll
          for (int j = 0; j < G; ++j) bits |= finite32(br[j]) ? 0u : kNonfinite;
          flag_warp(status, bits);
        }
        have_book = true;
      }
#pragma unroll
      for (uint32_t it = 0; it < 4; ++it) {
        const uint32_t t = task * 8u + 2u * it + (lane >> 4);
        float a = 0.f;
#pragma unroll
        for (int j = 0; j < G; j += 4) {
          const float4 x4 = *reinterpret_cast<const float4*>(xbuf + t * G + j);
          a = fmaf(x4.x, br[j], a);
          a = fmaf(x4.y, br[j + 1], a);
          a = fmaf(x4.z, br[j + 2], a);
          a = fmaf(x4.w, br[j + 3], a);
        }
        P[pair::p_index(t, lane & 15)] = a;
      }
    }
  };
  uint64_t s0 = u0;
  uint32_t c = 0;
  prefetch(s0, 0);
  build_p(s0 % nb == 0);
  uint32_t w[pair::kRows];
  // one 32-row batch of code words: rows n0.. of an expert, `wp` this lane's
  // word of row n0
  auto load_rows = [&](const uint32_t* wp, uint32_t n0) {
    if (n0 + pair::kRows <= N) {
#pragma unroll
      for (int r = 0; r < pair::kRows; ++r) w[r] = __ldcs(wp + uint32_t(r) * row_words);
    } else {
#pragma unroll
      for (int r = 0; r < pair::kRows; ++r) w[r] = n0 + r < N ? __ldcs(wp + uint32_t(r) * row_words) : 0u;
    }
  };
  constexpr uint32_t kStepRows = pair::kWarps * pair::kRows;  // rows between a warp's batches
  bool preloaded = false;  // w already holds this warp's first batch of the current (segment, chunk)
  while (s0 < u1) {
    const uint64_t s1 = seg_end(s0);
    const uint32_t e = uint32_t(s0 / nb);
    // the next (segment, chunk)
    uint64_t ns = s0;
    uint32_t nc = c + 1;
    if (nc == chunks) {
      nc = 0;
      ns = s1;
    }
    const bool more = ns < u1;
    // codes of this (expert, chunk): a warp-uniform base, 32-bit lane offsets
    const uint32_t* cb = codes + uint64_t(e) * words_per_expert + uint64_t(c) * 32u;
    float* ye = Y + uint64_t(e) * N;
    const uint64_t first = uint64_t(e) * nb;  // units of this segment are one expert's
    // this warp's batches: rows n0, n0 + kStepRows, ... below nend, the lane's
    // word pointer advanced with them
    const uint32_t nend = uint32_t(s1 - first) * pair::kRows;
    uint32_t n0 = uint32_t(s0 + warp - first) * pair::kRows;
    const uint32_t* wp = cb + n0 * row_words + lane;
    // the first batch's code words are in flight during the table build (or
    // were issued during this warp's last batch of the previous segment)
    if (!preloaded && n0 < nend) load_rows(wp, n0);
    preloaded = false;
    __syncthreads();  // P of this chunk is built: Q, x and the book are no longer read
    if (tid == 0) ptask = 0;
    // the next chunk's x and book, in flight during the table build and the lookups
    if (more) prefetch(ns, nc);
    // Q: a thread holds P[2p][0..15] of one pair p = 4 i + j (lane = slot i)
    // and fills four of its high nibbles, so both the P loads and the Q
    // stores are conflict-free and P[2p] is read once
    {
      static_assert(pair::kThreads == 512, "four high nibbles per thread");
      const uint32_t i = tid & 31, j = (tid >> 5) & 3, h0 = tid >> 7;
      const uint32_t p = 4 * i + j;
      float lo[16], hv[4];
#pragma unroll
      for (int k = 0; k < 16; ++k) lo[k] = P[pair::p_index(2 * p, k)];
#pragma unroll
      for (int h = 0; h < 4; ++h) hv[h] = P[pair::p_index(2 * p + 1, h0 + 4 * h)];
      float* qp = Q + (j & 1u) * 32u + i + (j >> 1) * 16384u + h0 * 16u * 64u;
#pragma unroll
      for (int h = 0; h < 4; ++h)
#pragma unroll
        for (int k = 0; k < 16; ++k) qp[h * 4 * 16 * 64 + k * 64] = lo[k] + hv[h];
    }
    __syncthreads();  // Q is built; P is free for the next chunk

    for (; n0 < nend; n0 += kStepRows, wp += kStepRows * row_words) {
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
      if (n0 + kStepRows < nend) {
        load_rows(wp + kStepRows * row_words, n0 + kStepRows);  // in flight during the folding
      } else if (more && ns + warp < seg_end(ns)) {
        // this warp's last batch here: the first batch of the next (segment,
        // chunk) goes in flight now, through the fold, the P build, the
        // barrier and the next table build
        const uint32_t en = uint32_t(ns / nb);
        const uint32_t nn0 = uint32_t(ns + warp - uint64_t(en) * nb) * pair::kRows;
        load_rows(codes + uint64_t(en) * words_per_expert + uint64_t(nc) * 32u + nn0 * row_words + lane, nn0);
        preloaded = true;
      }
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
        const float nv = (ONE || c == 0) ? v[0] : *y + v[0];
        *y = nv;
        ybits |= finite32(nv) ? 0u : kNonfinite;  // a nonfinite partial sum stays nonfinite
        if (ONE || c + 1 == chunks)  // the finished value, into every peer's slot too (NVLink stores)
          for (uint32_t i = 0; i < peers.n; ++i) peers.dst[i][uint64_t(e) * N + n0 + lane] = nv;
      }
    }
    // this warp's lookups are done: help build the next chunk's P
    if (more) build_p(nc == 0 && ns % nb == 0);
    c = nc;
    s0 = ns;
  }
  flag_warp(status, ybits);
  if (peers.n) __threadfence_system();  // the peer stores are visible before the block exits
  asm volatile("cp.async.wait_all;" ::: "memory");
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
      // the A rows' table rows are warp-uniform: lane l holds entry l % 16 of
      // each, and a lookup is a shuffle from the lane of B's code
      uint32_t b1[RJ];
#pragma unroll
      for (int j = 0; j < RJ; ++j) b1[j] = (bw[j] >> (4 * s)) & 15u;
#pragma unroll
      for (int i = 0; i < RI; ++i) {
        const float row = L[(((aw[i] >> (4 * s)) & 15u) << 4) + (lane & 15u)];
#pragma unroll
        for (int j = 0; j < RJ; ++j) acc[i][j] += __shfl_sync(0xffffffffu, row, b1[j]);
      }
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
                              uint32_t K, uint32_t batch, uint64_t words, uint32_t* status, cudaStream_t s,
                              const PeerY& peers = PeerY{{}, 0}) {
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
                                                                               status, peers);
  else
    k_dense_pair<G, false><<<grid, pair::kThreads, pair::smem_bytes<G>(), s>>>(X, codes, books, Y, N, K, batch, words,
                                                                                status, peers);
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
struct RunDensePeers {
  static cudaError_t run(const Plan& p, void* const* ptr, const PeerY& peers, cudaStream_t s) {
    const float* X = static_cast<const float*>(ptr[0]);
    const uint32_t* codes = static_cast<const uint32_t*>(ptr[1]);
    const float* books = static_cast<const float*>(ptr[2]);
    const uint32_t M = uint32_t(p.m), N = uint32_t(p.n), K = uint32_t(p.k);
    if ((p.flags & ~2u) != 0 || !(p.flags & 2u) || !dense_pair_fits<G>(M, N, K, p.batch, X, books))
      return cudaErrorNotSupported;
    return launch_dense_pair<G>(X, codes, books, static_cast<float*>(ptr[5]), N, K, p.batch,
                                packed_words(uint64_t(N) * K, G), static_cast<uint32_t*>(ptr[7]), s, peers);
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


}  // namespace

cudaError_t launch_matmul_exact(const Plan& p, void* const* ptr, cudaStream_t s) {
  return by_group<RunMatmulExact>(p.group, p, ptr, s);
}

cudaError_t launch_dense(const Plan& p, void* const* ptr, cudaStream_t s) {
  return by_group<RunDense>(p.group, p, ptr, s);
}

cudaError_t launch_coded(const Plan& p, void* const* ptr, cudaStream_t s) {
  return by_group<RunCoded>(p.group, p, ptr, s);
}

cudaError_t launch_repack(const Plan& p, void* const* ptr, cudaStream_t s) {
  const uint32_t g = p.group;
  if (!aligned16(ptr[0]) || !aligned16(ptr[5])) return cudaErrorMisalignedAddress;
  const uint32_t T = uint32_t(p.k / g);
  const uint64_t src_units = packed_bytes(p.m * p.k, g) / 16, dst_units = tile32_bytes(p.m, p.k, g) / 16;
  k_repack_tile32<<<grid_for(dst_units * p.batch), kThreads, 0, s>>>(
      static_cast<const uint4*>(ptr[0]), static_cast<uint4*>(ptr[5]), uint32_t(p.m), T, src_units, dst_units,
      p.batch);
  return cudaGetLastError();
}

}  // namespace ack

namespace ack {
cudaError_t dense_peers(const Plan& p, void* const* ptr, const PeerY& peers, cudaStream_t s) {
  if (p.op != Op::Dense || peers.n > kMaxPeers) return cudaErrorNotSupported;
  switch (p.group) {
    case 8: return RunDensePeers<8>::run(p, ptr, peers, s);
    case 16: return RunDensePeers<16>::run(p, ptr, peers, s);
    case 32: return RunDensePeers<32>::run(p, ptr, peers, s);
    default: return cudaErrorNotSupported;
  }
}
}  // namespace ack
