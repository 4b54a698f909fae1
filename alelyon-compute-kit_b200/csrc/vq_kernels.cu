// sm_100a kernels of the vq4/v1 path and their launcher.
//
//   decode        HBM-write-bound gather: 128-bit streaming stores, the
//                 codebook in shared memory (vq4.comp op 1 / vq.py:117-121)
//   encode        certified nearest entry per vector: FP32 filter on the CUDA
//                 cores, float64 pass only for near ties; lanes of a warp own
//                 consecutive vectors and pack nibbles with shuffles
//                 (vq4.comp op 0 / vq.py:154-179)
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
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "vq_device.cuh"
#include "vq_kernels.hpp"

namespace ack {
namespace {

constexpr int kThreads = 256;

// ------------------------------------------------------------------ decode --

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
  constexpr uint32_t kQ = G / 4;  // float4 per vector
  const uint64_t nq = n / 4;
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  uint64_t q = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; q + 3 * stride < nq; q += 4 * stride) {
    uint32_t c[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) c[u] = code_at(codes, (q + u * stride) / kQ);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint64_t qq = q + u * stride;
      __stcs(out4 + qq, sb4[c[u] * kQ + uint32_t(qq % kQ)]);
    }
  }
  for (; q < nq; q += stride) __stcs(out4 + q, sb4[code_at(codes, q / kQ) * kQ + uint32_t(q % kQ)]);
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const uint64_t i = nq * 4 + threadIdx.x;
    out[i] = sb[code_at(codes, i / G) * G + uint32_t(i % G)];
  }
}

// Scalar variant for an output that is not 16-byte aligned (device-pointer callers).
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

template <int G>
__global__ void __launch_bounds__(kThreads) k_encode(const float* __restrict__ x, uint64_t n,
                                                     const float* __restrict__ book, uint32_t* __restrict__ codes,
                                                     uint32_t* __restrict__ status, int aligned) {
  __shared__ EncBook<G> eb;
  enc_book_setup<G>(eb, book);
  if (blockIdx.x == 0 && threadIdx.x == 0 && eb.bad) atomicOr(status, kNonfinite);
  const uint64_t vectors = (n + G - 1) / G;
  const uint64_t full = n / G;
  const uint64_t words = (vectors + 7) / 8;
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warps = uint64_t(gridDim.x) * (blockDim.x / 32);
  for (uint64_t base = (uint64_t(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32) * 32; base < vectors;
       base += warps * 32) {
    const uint64_t v = base + lane;
    uint32_t idx = 0, bits = 0;
    float xr[G];
    if (v < full) {
      if (aligned) {
        load_vector<G>(x, v, xr);
      } else {
#pragma unroll
        for (int j = 0; j < G; ++j) xr[j] = x[v * G + j];
      }
#pragma unroll
      for (int j = 0; j < G; ++j) bits |= finite32(xr[j]) ? 0u : kNonfinite;
      bool certified;
      idx = enc_vector<G>(xr, eb, &certified);
    } else if (v < vectors) {
      // The partial last vector: compare its valid components only (vq.py:171-172).
      const int valid = int(n - v * G);
#pragma unroll
      for (int j = 0; j < G; ++j) xr[j] = j < valid ? x[v * G + j] : 0.f;
#pragma unroll
      for (int j = 0; j < G; ++j) bits |= (j < valid && !finite32(xr[j])) ? kNonfinite : 0u;
      idx = enc_exact<G>(xr, valid, 0xffffu, eb.rows);
    }
    const uint32_t w = pack_nibbles(idx);
    const uint64_t word = (base >> 3) + (lane >> 3);
    if ((lane & 7) == 0 && word < words) codes[word] = w;
    flag_warp(status, bits);
  }
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

// Shared-memory plan of k_dense_lut: the table P[MC][TC][16] then two code
// stages of 256 rows x (TC/2 + 16) bytes.
__host__ __device__ constexpr uint32_t lut_row_pitch(uint32_t tc) { return tc / 2 + 16; }

template <int G, int MC>
__global__ void __launch_bounds__(kThreads, 1) k_dense_lut(const float* __restrict__ X,
                                                           const uint32_t* __restrict__ codes,
                                                           const float* __restrict__ books, float* __restrict__ Y,
                                                           uint32_t M, uint32_t N, uint32_t K, uint32_t rows_per_block,
                                                           uint32_t TC, uint64_t words_per_expert,
                                                           uint32_t* __restrict__ status) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* P = reinterpret_cast<float*>(smem);
  unsigned char* stage0 = smem + size_t(MC) * TC * 16 * 4;
  const uint32_t pitch = lut_row_pitch(TC);
  const size_t stage_bytes = size_t(kThreads) * pitch;  // stage b starts at stage0 + b * stage_bytes
  __shared__ float sbook[16 * 32];

  const uint32_t b = blockIdx.y;
  const uint32_t T = K / G;
  const float* Xb = X + uint64_t(b) * M * K;
  const uint32_t* Cb = codes + uint64_t(b) * words_per_expert;
  float* Yb = Y + uint64_t(b) * M * N;
  for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) sbook[i] = books[uint64_t(b) * 16 * G + i];
  __syncthreads();
  if (blockIdx.x == 0) {
    uint32_t bits = 0;
    for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) bits |= finite32(sbook[i]) ? 0u : kNonfinite;
    flag_warp(status, bits);
  }
  const uint32_t r0 = blockIdx.x * rows_per_block;
  const uint32_t r1 = min(N, r0 + rows_per_block);

  for (uint32_t m0 = 0; m0 < M; m0 += MC) {
    const uint32_t mc = min(uint32_t(MC), M - m0);
    for (uint32_t t0 = 0; t0 < T; t0 += TC) {
      const uint32_t tc = min(TC, T - t0);
      __syncthreads();  // the previous table is no longer read
      // P[m][t][e] = sum_j x[m0+m, (t0+t)*G + j] * c[e][j]
      for (uint32_t i = threadIdx.x; i < mc * tc; i += blockDim.x) {
        const uint32_t m = i / tc, t = i % tc;
        const float* xs = Xb + uint64_t(m0 + m) * K + uint64_t(t0 + t) * G;
        float xr[G];
#pragma unroll
        for (int j = 0; j < G; ++j) xr[j] = __ldg(xs + j);
        float* dst = P + (size_t(m) * TC + t) * 16;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < G; ++j) s = fmaf(xr[j], sbook[e * G + j], s);
          dst[e] = s;
        }
      }
      __syncthreads();
      // rows in batches of 256, one row per thread; code tiles double-buffered
      const uint32_t batches = (r1 - r0 + kThreads - 1) / kThreads;
      auto issue = [&](uint32_t batch, int buf) {
        const uint32_t rb = r0 + batch * kThreads;
        const uint32_t nrows = min(uint32_t(kThreads), r1 - rb);
        const uint32_t pieces = tc / 32;  // 16-byte pieces of this chunk in one row
        for (uint32_t i = threadIdx.x; i < nrows * pieces; i += blockDim.x) {
          const uint32_t r = i / pieces, pc = i % pieces;
          const unsigned char* src = reinterpret_cast<const unsigned char*>(Cb) +
                                     (uint64_t(rb + r) * T + t0) / 2 + uint64_t(pc) * 16;
          unsigned char* dst = stage0 + buf * stage_bytes + size_t(r) * pitch + pc * 16;
          const uint32_t saddr = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(src));
        }
        asm volatile("cp.async.commit_group;\n" ::);
      };
      if (batches) issue(0, 0);
      for (uint32_t batch = 0; batch < batches; ++batch) {
        const int buf = batch & 1;
        if (batch + 1 < batches) {
          issue(batch + 1, buf ^ 1);
          asm volatile("cp.async.wait_group 1;\n" ::);
        } else {
          asm volatile("cp.async.wait_group 0;\n" ::);
        }
        __syncthreads();
        const uint32_t row = r0 + batch * kThreads + threadIdx.x;
        if (row < r1) {
          float acc[MC];
#pragma unroll
          for (int m = 0; m < MC; ++m) acc[m] = 0.f;
          const uint4* src = reinterpret_cast<const uint4*>(stage0 + buf * stage_bytes + size_t(threadIdx.x) * pitch);
          for (uint32_t piece = 0; piece < tc / 32; ++piece) {
            const uint4 q4 = src[piece];
            const uint32_t wds[4] = {q4.x, q4.y, q4.z, q4.w};
            const float* Pp = P + size_t(piece) * 32 * 16;
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
              const uint32_t w = wds[wi];
#pragma unroll
              for (int s = 0; s < 8; ++s) {
                const uint32_t off = (wi * 8 + s) * 16 + ((w >> (4 * s)) & 15u);
#pragma unroll
                for (int m = 0; m < MC; ++m)
                  if (m < int(mc)) acc[m] += Pp[size_t(m) * TC * 16 + off];
              }
            }
          }
#pragma unroll
          for (int m = 0; m < MC; ++m) {
            if (m < int(mc)) {
              float* y = Yb + uint64_t(m0 + m) * N + row;
              *y = t0 ? *y + acc[m] : acc[m];
            }
          }
        }
        __syncthreads();  // this stage may be overwritten by the next issue
      }
    }
  }
}

// ------------------------------------------ coded A times coded B^T (LUT) --

// C[m, n] = sum_t L[a(m,t)][b(n,t)] with L = C_A C_B^T (16 x 16, each entry
// summed in float64 and rounded once). A stored M x K, B stored N x K,
// K % G == 0 and (K/G) % 8 == 0 so every row starts on a code word. A warp
// owns 8 rows (warp-uniform A codes) and 256 columns (8 per lane), so every
// lookup of an instruction reads one 16-entry row of L: distinct columns hit
// distinct banks, equal columns broadcast.
template <int G>
__global__ void __launch_bounds__(kThreads) k_coded_lut(const uint32_t* __restrict__ ac,
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
  const uint32_t TW = K / G / 8;  // code words per row
  const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // block tile: 64 rows (8 warps x 8 rows) x 256 columns
  const uint32_t row0 = blockIdx.y * 64 + warp * 8;
  const uint32_t col0 = blockIdx.x * 256 + lane;
  const uint32_t* arow[8];
  const uint32_t* bcol[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) arow[i] = ac + uint64_t(min(row0 + i, M - 1)) * TW;
#pragma unroll
  for (int j = 0; j < 8; ++j) bcol[j] = bc + uint64_t(min(col0 + 32 * j, N - 1)) * TW;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  for (uint32_t tw = 0; tw < TW; ++tw) {
    uint32_t aw[8], bw[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) aw[i] = __ldg(arow[i] + tw);
#pragma unroll
    for (int j = 0; j < 8; ++j) bw[j] = __ldg(bcol[j] + tw);
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      uint32_t a16[8], b1[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a16[i] = ((aw[i] >> (4 * s)) & 15u) << 4;
#pragma unroll
      for (int j = 0; j < 8; ++j) b1[j] = (bw[j] >> (4 * s)) & 15u;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] += L[a16[i] + b1[j]];
    }
  }
  uint32_t bits = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
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

template <int G>
__device__ __forceinline__ void adamw_vector(const AdamwBatch& a, const float* __restrict__ sbooks,
                                             const AdamwCoefs& k, uint32_t e, uint64_t v, int valid,
                                             float (&w)[G], float (&m)[G], float (&var)[G], uint32_t* bits) {
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

// Entries a trial book selects over the complete vectors of one updated state
// (the whole-tensor pass of fit_codebook, vq.py:219-222).
template <int G>
__global__ void __launch_bounds__(kThreads) k_adamw_usage(AdamwBatch a, uint32_t expert, uint32_t state,
                                                          const float* __restrict__ trial, uint32_t* __restrict__ out,
                                                          uint32_t* __restrict__ status) {
  __shared__ float sbooks[4 * 16 * G];
  __shared__ EncBook<G> eb;
  __shared__ uint32_t hist[16];
  for (int i = threadIdx.x; i < 64 * G; i += blockDim.x) sbooks[i] = a.books[uint64_t(expert) * 64 * G + i];
  if (threadIdx.x < 16) hist[threadIdx.x] = 0;
  enc_book_setup<G>(eb, trial);
  const AdamwCoefs k = load_coefs(a.coefs + 7 * expert);
  const uint64_t full = a.n / G;
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  // a whole warp iterates together so flag_warp stays convergent
  for (uint64_t base = uint64_t(blockIdx.x) * blockDim.x + (threadIdx.x & ~31u); base < full; base += stride) {
    const uint64_t v = base + (threadIdx.x & 31);
    uint32_t bits = k.status;
    if (v < full && !bits) {
      float w[G], m[G], var[G];
      adamw_vector<G>(a, sbooks, k, expert, v, G, w, m, var, &bits);
      bool certified;
      const uint32_t idx = state == 0 ? enc_vector<G>(w, eb, &certified)
                          : state == 1 ? enc_vector<G>(m, eb, &certified)
                                       : enc_vector<G>(var, eb, &certified);
      atomicAdd(&hist[idx], 1u);
    }
    flag_warp(status, bits);
  }
  __syncthreads();
  if (threadIdx.x < 16 && hist[threadIdx.x]) atomicAdd(out + threadIdx.x, hist[threadIdx.x]);
}

// decode -> AdamW -> encode of W', M', V' with their new books, one vector
// per thread, and a count of weight values whose decoded value changed.
template <int G>
__global__ void __launch_bounds__(kThreads) k_adamw_encode(AdamwBatch a, const float* __restrict__ new_books,
                                                           uint32_t* __restrict__ out_codes,
                                                           uint32_t* __restrict__ changed,
                                                           uint32_t* __restrict__ status) {
  __shared__ float sbooks[4 * 16 * G];
  __shared__ EncBook<G> eb[3];
  const uint32_t e = blockIdx.y;
  for (int i = threadIdx.x; i < 64 * G; i += blockDim.x) sbooks[i] = a.books[uint64_t(e) * 64 * G + i];
  for (int s = 0; s < 3; ++s) enc_book_setup<G>(eb[s], new_books + (uint64_t(e) * 3 + s) * 16 * G);
  const AdamwCoefs k = load_coefs(a.coefs + 7 * e);
  if (blockIdx.x == 0 && threadIdx.x == 0 && (eb[0].bad || eb[1].bad || eb[2].bad)) atomicOr(status, kNonfinite);
  const uint64_t vectors = (uint64_t(a.n) + G - 1) / G;
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warps = uint64_t(gridDim.x) * (blockDim.x / 32);
  uint32_t changes = 0;
  for (uint64_t base = (uint64_t(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32) * 32; base < vectors;
       base += warps * 32) {
    const uint64_t v = base + lane;
    uint32_t idx[3] = {0, 0, 0}, bits = k.status;
    if (v < vectors && !bits) {
      const int valid = int(min(uint64_t(G), uint64_t(a.n) - v * G));
      float w[G], m[G], var[G];
      adamw_vector<G>(a, sbooks, k, e, v, valid, w, m, var, &bits);
      bool certified;
      if (valid == G) {
        idx[0] = enc_vector<G>(w, eb[0], &certified);
        idx[1] = enc_vector<G>(m, eb[1], &certified);
        idx[2] = enc_vector<G>(var, eb[2], &certified);
      } else {
        idx[0] = enc_exact<G>(w, valid, 0xffffu, eb[0].rows);
        idx[1] = enc_exact<G>(m, valid, 0xffffu, eb[1].rows);
        idx[2] = enc_exact<G>(var, valid, 0xffffu, eb[2].rows);
      }
      // vq.py:402: decoded new weight against decoded old weight, value by value
      const uint32_t old = code_at(a.codes + uint64_t(e) * 4 * a.words, v);
      for (int j = 0; j < valid; ++j)
        changes += eb[0].rows[idx[0] * G + j] != sbooks[old * G + j];
    }
#pragma unroll
    for (int s = 0; s < 3; ++s) {
      const uint32_t word_bits = pack_nibbles(idx[s]);
      const uint64_t word = (base >> 3) + (lane >> 3);
      if ((lane & 7) == 0 && word < a.words) out_codes[(uint64_t(e) * 3 + s) * a.words + word] = word_bits;
    }
    flag_warp(status, bits);
  }
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

template <template <int> class F, typename... Args>
cudaError_t by_group(uint32_t g, Args&&... args) {
  switch (g) {
    case 8: return F<8>::run(args...);
    case 16: return F<16>::run(args...);
    default: return F<32>::run(args...);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int G>
struct RunDecode {
  static cudaError_t run(const uint32_t* codes, const float* book, float* out, uint64_t n, uint32_t* status,
                         cudaStream_t s) {
    if (aligned16(out)) {
      k_decode<G><<<grid_for(n / 4 + 1), kThreads, 0, s>>>(codes, book, out, n, status);
    } else {
      k_decode_scalar<G><<<grid_for(n), kThreads, 0, s>>>(codes, book, out, n, status);
    }
    return cudaGetLastError();
  }
};

template <int G>
struct RunEncode {
  static cudaError_t run(const float* x, uint64_t n, const float* book, uint32_t* codes, uint32_t* status,
                         cudaStream_t s) {
    const uint64_t vectors = (n + G - 1) / G;
    k_encode<G><<<grid_for(vectors, 4), kThreads, 0, s>>>(x, n, book, codes, status, aligned16(x) ? 1 : 0);
    return cudaGetLastError();
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

template <int G, int MC>
cudaError_t launch_dense_lut_mc(const float* X, const uint32_t* codes, const float* books, float* Y, uint32_t M,
                                uint32_t N, uint32_t K, uint32_t batch, uint64_t words, uint32_t* status,
                                cudaStream_t s) {
  const uint32_t T = K / G;
  // table budget: MC x TC x 16 floats <= 128 KiB; code stages 2 x 256 rows
  // x (TC/2 + 16) bytes <= 96 KiB; TC a multiple of 32
  const uint32_t by_table = (128u * 1024u / (MC * 64u)) / 32u * 32u;
  const uint32_t by_stage = ((96u * 1024u / (2u * kThreads)) - 16u) * 2u / 32u * 32u;
  uint32_t tc = std::min<uint32_t>(T, std::min(by_table, by_stage));
  tc = std::max<uint32_t>(tc, 32u);
  const size_t smem = size_t(MC) * tc * 64 + 2 * size_t(kThreads) * lut_row_pitch(tc);
  // rows per block: enough blocks to fill the GPU, many rows to amortise the table
  const uint64_t want_blocks = uint64_t(sm_count()) * 4;
  uint64_t rows = (uint64_t(N) * batch + want_blocks - 1) / want_blocks;
  rows = std::min<uint64_t>(std::max<uint64_t>(rows, kThreads), 8192);
  rows = (rows + kThreads - 1) / kThreads * kThreads;
  dim3 grid(uint32_t((N + rows - 1) / rows), batch);
  cudaError_t err = cudaFuncSetAttribute(k_dense_lut<G, MC>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (err != cudaSuccess) return err;
  k_dense_lut<G, MC><<<grid, kThreads, smem, s>>>(X, codes, books, Y, M, N, K, uint32_t(rows), tc, words, status);
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
    if (nt && K % G == 0 && (K / G) % 32 == 0 && aligned16(codes) && (words * 4) % 16 == 0) {
      if (M == 1) return launch_dense_lut_mc<G, 1>(X, codes, books, Y, M, N, K, p.batch, words, status, s);
      if (M == 2) return launch_dense_lut_mc<G, 2>(X, codes, books, Y, M, N, K, p.batch, words, status, s);
      if (M <= 4) return launch_dense_lut_mc<G, 4>(X, codes, books, Y, M, N, K, p.batch, words, status, s);
      return launch_dense_lut_mc<G, 8>(X, codes, books, Y, M, N, K, p.batch, words, status, s);
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
      dim3 grid((N + 255) / 256, (M + 63) / 64);
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
    } else if (p.op == Op::AdamwUsage) {
      cudaError_t err = cudaMemsetAsync(ptr[5], 0, 16 * sizeof(uint32_t), s);
      if (err != cudaSuccess) return err;
      k_adamw_usage<G><<<grid_for(p.m / G, 4), kThreads, 0, s>>>(a, p.aux1, p.aux0, static_cast<const float*>(ptr[3]),
                                                                 static_cast<uint32_t*>(ptr[5]), status);
    } else {
      cudaError_t err = cudaMemsetAsync(ptr[6], 0, size_t(p.batch) * sizeof(uint32_t), s);
      if (err != cudaSuccess) return err;
      const uint32_t per = std::max<uint32_t>(1, grid_for(vectors * p.batch, 4) / p.batch);
      dim3 grid(std::min<uint32_t>(per, uint32_t((vectors + kThreads - 1) / kThreads)), p.batch);
      k_adamw_encode<G><<<grid, kThreads, 0, s>>>(a, static_cast<const float*>(ptr[3]),
                                                   static_cast<uint32_t*>(ptr[5]), static_cast<uint32_t*>(ptr[6]),
                                                   status);
    }
    return cudaGetLastError();
  }
};

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
    default:
      return cudaErrorInvalidValue;
  }
}

const char* kernel_manifest() {
  return "vq4-b200/1 sm_100a: k_decode k_decode_scalar k_encode k_matmul_exact k_adamw k_dense_lut "
         "k_coded_lut k_gemm_generic k_adamw_sample k_adamw_usage k_adamw_encode";
}

}  // namespace ack
