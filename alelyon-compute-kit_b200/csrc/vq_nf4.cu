// The NF4 comparator on the GPU: bitsandbytes' NF4 with double quantisation
// read in its stored form, as the reference kit defines it
// (src/alelyon_compute_kit/_kit/kernels/nf4_decode.comp, nf4_gemv.comp):
//
//   k_nf4_decode<STORAGE>  nf4-decode/v1: one thread per packed word of 8
//                          values, scale = fl(map[q] * absmax2), absmax =
//                          fl(scale + offset), value = fl(code[index] *
//                          absmax), written as FP32 or rounded to bf16 / fp16
//                          (nf4_decode.comp:108-158)
//   k_nf4_gemv<E, P, R>    nf4-gemv/v1: C = A . W^T for groups of at most R
//                          rows, A and the decoded weight 16-bit (E: bf16 or
//                          fp16). The law's 64 partial sums of a column (lane
//                          l: words l, l + 64, ... in order, each word's 8
//                          values in order) are held P to a thread by a team
//                          of 64 / P threads, then the law's tree s = 32 .. 1
//                          runs across the team (shuffles; shared memory for
//                          the step between a 64-thread team's two warps) and
//                          within threads (nf4_gemv.comp:203-266). A thread
//                          keeps the 16 weights of its current absmax (each
//                          rounded to 16 bits and widened) in shared memory,
//                          rebuilt only when the absmax changes, so a value
//                          costs one table read, one multiply and one add.
//
// Every FP32 operation is a separately rounded __fmul_rn / __fadd_rn, so the
// words are the law's wherever it defines them (products and partial sums
// zero or normal), NaN payloads aside.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "vq_common.cuh"
#include "vq_kernels.hpp"

namespace ack {
namespace {

constexpr uint32_t kNanBits = 0x7FC00000u;

__device__ __forceinline__ bool dev_aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// FP32 -> bf16 bits, round to nearest even, NaN kept quiet (nf4_decode.comp:72-79).
__device__ __forceinline__ uint32_t to_bf16(float x) {
  const uint32_t b = __float_as_uint(x);
  if ((b & 0x7F800000u) == 0x7F800000u && (b & 0x007FFFFFu) != 0u) return (b >> 16) | 0x0040u;
  return (b + 0x7FFFu + ((b >> 16) & 1u)) >> 16;
}

// FP32 -> fp16 bits by the kit's integer routine: round to nearest even,
// subnormals kept, NaN -> sign | 0x7E00 (nf4_decode.comp:83-103).
__device__ __forceinline__ uint32_t to_f16(float x) {
  const uint32_t w = __float_as_uint(x);
  const uint32_t sign = (w >> 16) & 0x8000u, e = (w >> 23) & 0xFFu, m = w & 0x7FFFFFu;
  if (e == 0xFFu) return sign | (m != 0u ? 0x7E00u : 0x7C00u);
  const int he = int(e) - 112;
  if (he >= 31) return sign | 0x7C00u;
  if (he <= 0) {
    if (he < -10) return sign;
    const uint32_t mf = m | 0x800000u, shift = uint32_t(14 - he);
    uint32_t q = mf >> shift;
    const uint32_t rem = mf & ((1u << shift) - 1u), half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q += 1u;
    return sign | q;
  }
  uint32_t h = (uint32_t(he) << 10) | (m >> 13);
  const uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
  return sign | h;
}

template <int E>
__device__ __forceinline__ uint32_t to16(float x) {
  return E == 0 ? to_bf16(x) : to_f16(x);
}

// 16-bit word -> FP32, exact (the hardware conversion for fp16).
template <int E>
__device__ __forceinline__ float widen16(uint32_t h) {
  return E == 0 ? __uint_as_float(h << 16) : __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

// The member holding source value s: the last start at or below it (the low
// words of the int64 starts, ascending from 0).
__device__ __forceinline__ uint32_t member_of(const uint32_t* __restrict__ starts, uint32_t members, uint32_t s) {
  uint32_t lo = 0, hi = members;
  while (hi - lo > 1u) {
    const uint32_t mid = (lo + hi) / 2u;
    if (__ldg(starts + 2u * mid) <= s) lo = mid;
    else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ float block_absmax(const Nf4Source& src, const float* map, uint32_t s, float offset) {
  const uint32_t blk = s >> 6;
  const uint32_t q = (__ldg(src.absmax_q + (blk >> 2)) >> (8u * (blk & 3u))) & 0xFFu;
  return __fadd_rn(__fmul_rn(map[q], __ldg(src.absmax2 + (blk >> 8))), offset);
}

template <int STORAGE>
__global__ void __launch_bounds__(256) k_nf4_decode(Nf4Source src, const uint32_t* __restrict__ ids, void* out,
                                                    uint32_t n, uint32_t words, uint32_t selected,
                                                    uint32_t member_values) {
  __shared__ float tab[272];
  for (uint32_t i = threadIdx.x; i < 272u; i += blockDim.x) tab[i] = src.tables[i];
  __syncthreads();
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t w = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; w < words; w += stride) {
    const uint32_t i0 = uint32_t(w) * 8u;
    uint32_t m, s0;
    bool bad = false;
    if (selected == 0u) {
      m = member_of(src.starts, src.members, i0);
      s0 = i0;
    } else {
      const uint32_t j = i0 / member_values;
      m = ids[2u * j];
      bad = ids[2u * j + 1u] != 0u || m >= src.members;  // a negative or too-large int64 id
      s0 = (bad ? 0u : src.starts[2u * m]) + (i0 - j * member_values);
    }
    const uint32_t count = min(8u, n - i0);
    float v[8];
    if (bad || s0 >= src.src_limit || count > src.src_limit - s0) {
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = __uint_as_float(kNanBits);
    } else {
      const uint32_t s = src.src_base + s0;
      const uint32_t word = __ldg(src.packed + (s >> 3));
      const float absmax = block_absmax(src, tab + 16, s, src.offsets[m]);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t byte = (word >> (8 * (k >> 1))) & 0xFFu;
        v[k] = __fmul_rn(tab[(k & 1) ? (byte & 0xFu) : (byte >> 4)], absmax);
      }
    }
    if constexpr (STORAGE == 0) {
      float* o = static_cast<float*>(out) + i0;
      if (count == 8u && dev_aligned16(o)) {
        reinterpret_cast<float4*>(o)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(o)[1] = make_float4(v[4], v[5], v[6], v[7]);
      } else {
        for (uint32_t k = 0; k < count; ++k) o[k] = v[k];
      }
    } else {
      uint16_t* o = static_cast<uint16_t*>(out) + i0;
      uint32_t h[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) h[k] = STORAGE == 1 ? to_bf16(v[k]) : to_f16(v[k]);
      if (count == 8u && dev_aligned16(o)) {
        *reinterpret_cast<uint4*>(o) =
            make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
      } else {
        for (uint32_t k = 0; k < count; ++k) o[k] = static_cast<uint16_t>(h[k]);
      }
    }
  }
}

template <int E, int P, int R>
__global__ void __launch_bounds__(256) k_nf4_gemv(Nf4Gemv g) {
  constexpr int T = 64 / P;          // threads of a team (one column of one group)
  constexpr int kTeams = 256 / T;    // teams of a block
  __shared__ float code_s[16], map_s[256];
  __shared__ float wtab[16][256];    // each thread's rounded weights of its current absmax
  __shared__ float cross[T == 64 ? R : 1][T == 64 ? 256 : 1];  // the tree's step between a team's warps
  const uint32_t tid = threadIdx.x, q = tid % T;
  for (uint32_t i = tid; i < 272u; i += 256u) {
    if (i < 16u) code_s[i] = g.src.tables[i];
    else map_s[i - 16u] = g.src.tables[i];
  }
  __syncthreads();
  const uint64_t total = uint64_t(g.groups) * g.n;
  const uint32_t words = g.k / 8u;
  // block-uniform loop (the 64-thread teams meet at __syncthreads)
  for (uint64_t t0 = uint64_t(blockIdx.x) * kTeams; t0 < total; t0 += uint64_t(gridDim.x) * kTeams) {
    const uint64_t team = t0 + tid / T;
    const uint32_t z = uint32_t(team / g.n), col = uint32_t(team % g.n);
    uint32_t row_start = 0, m_rows = 0, w_base = 0;
    bool ok = team < total;
    if (ok) {
      row_start = g.table[3u * z];
      m_rows = g.table[3u * z + 1u];
      w_base = g.table[3u * z + 2u];
      // the shader's group guards (nf4_gemv.comp:209-210)
      ok = !(m_rows == 0u || m_rows > uint32_t(R) || row_start + m_rows < row_start || row_start + m_rows > g.rows ||
             (w_base & 7u) != 0u || w_base > g.src.src_limit || g.n * g.k > g.src.src_limit - w_base);
    }
    float acc[P][R];
#pragma unroll
    for (int r = 0; r < P; ++r)
#pragma unroll
      for (int m = 0; m < R; ++m) acc[r][m] = 0.f;
    if (ok) {
      const uint32_t col_base = w_base + col * g.k;
      const uint32_t first = member_of(g.src.starts, g.src.members, col_base);
      const bool one = first == member_of(g.src.starts, g.src.members, col_base + g.k - 1u);
      const float col_off = __ldg(g.src.offsets + first);
      uint32_t key = 0xFFFFFFFFu;  // the bits of the absmax wtab holds (none yet)
      bool have = false;
      uint32_t cur_blk = 0xFFFFFFFFu;
      float absmax = 0.f;
      for (uint32_t base = 0; base < words; base += 64u) {
        // this thread's run of P consecutive words: one coalesced vector load
        // when it is whole and 16-byte aligned
        const uint32_t j0 = base + uint32_t(P) * q;
        const uint32_t s0 = g.src.src_base + col_base + 8u * j0;
        const uint32_t* wp = g.src.packed + (s0 >> 3);
        uint32_t pw[P];
        if constexpr (P >= 4) {
          if (j0 + P <= words && (reinterpret_cast<uintptr_t>(wp) & 15u) == 0) {
#pragma unroll
            for (int v = 0; v < P / 4; ++v) {
              const uint4 u = __ldg(reinterpret_cast<const uint4*>(wp) + v);
              pw[4 * v] = u.x;
              pw[4 * v + 1] = u.y;
              pw[4 * v + 2] = u.z;
              pw[4 * v + 3] = u.w;
            }
          } else {
#pragma unroll
            for (int r = 0; r < P; ++r) pw[r] = j0 + uint32_t(r) < words ? __ldg(wp + r) : 0u;
          }
        } else {
          pw[0] = j0 < words ? __ldg(wp) : 0u;
        }
#pragma unroll
        for (int r = 0; r < P; ++r) {
          const uint32_t j = j0 + uint32_t(r);
          if (j < words) {
            const uint32_t s = s0 + 8u * uint32_t(r);
            // the absmax only changes with its 64-value block (or, in a column
            // that straddles members, with the member)
            if (!one || (s >> 6) != cur_blk) {
              absmax = block_absmax(g.src, map_s, s,
                                    one ? col_off
                                        : __ldg(g.src.offsets + member_of(g.src.starts, g.src.members,
                                                                          col_base + 8u * j)));
              cur_blk = s >> 6;
              if (!have || __float_as_uint(absmax) != key) {
#pragma unroll
                for (int e = 0; e < 16; ++e) wtab[e][tid] = widen16<E>(to16<E>(__fmul_rn(code_s[e], absmax)));
                key = __float_as_uint(absmax);
                have = true;
              }
            }
            const uint32_t word = pw[r];
            float w[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const uint32_t byte = (word >> (8 * (e >> 1))) & 0xFFu;
              w[e] = wtab[(e & 1) ? (byte & 0xFu) : (byte >> 4)][tid];
            }
#pragma unroll
            for (int m = 0; m < R; ++m) {
              if (uint32_t(m) < m_rows) {
                const uint4 av = __ldg(g.A + ((uint64_t(row_start + uint32_t(m)) * g.lda + 8u * j) >> 3));
                const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  const float x = widen16<E>((aw[e >> 1] >> (16 * (e & 1))) & 0xFFFFu);
                  acc[r][m] = __fadd_rn(acc[r][m], __fmul_rn(x, w[e]));
                }
              }
            }
          }
        }
      }
    }
    // the law's tree: partial l = P q + r; steps s >= P pair threads q and
    // q + s / P, steps s < P pair registers r and r + s
    if constexpr (T == 64) {
      if (q >= 32u)
#pragma unroll
        for (int m = 0; m < R; ++m) cross[m][tid] = acc[0][m];
      __syncthreads();
      if (q < 32u)
#pragma unroll
        for (int m = 0; m < R; ++m) acc[0][m] = __fadd_rn(acc[0][m], cross[m][tid + 32u]);
      __syncthreads();  // `cross` is the next team's
#pragma unroll
      for (int d = 16; d >= 1; d >>= 1)
#pragma unroll
        for (int m = 0; m < R; ++m) acc[0][m] = __fadd_rn(acc[0][m], __shfl_down_sync(0xffffffffu, acc[0][m], d));
    } else {
#pragma unroll
      for (int s = 32; s >= P; s >>= 1)
#pragma unroll
        for (int r = 0; r < P; ++r)
#pragma unroll
          for (int m = 0; m < R; ++m)
            acc[r][m] = __fadd_rn(acc[r][m], __shfl_down_sync(0xffffffffu, acc[r][m], s / P, T));
#pragma unroll
      for (int s = P / 2; s >= 1; s >>= 1)
#pragma unroll
        for (int r = 0; r < s; ++r)
#pragma unroll
          for (int m = 0; m < R; ++m) acc[r][m] = __fadd_rn(acc[r][m], acc[r + s][m]);
    }
    if (ok && q == 0u)
#pragma unroll
      for (int m = 0; m < R; ++m)
        if (uint32_t(m) < m_rows) g.C[uint64_t(row_start + uint32_t(m)) * g.n + col] = acc[0][m];
  }
}

template <int E, int P, int R>
cudaError_t gemv_variant(const Nf4Gemv& g, cudaStream_t s) {
  constexpr int kTeams = 256 / (64 / P);
  const uint64_t total = uint64_t(g.groups) * g.n;
  const uint64_t blocks = (total + kTeams - 1) / kTeams;
  const uint32_t grid = uint32_t(std::min<uint64_t>(blocks, uint64_t(sm_count()) * 8));
  k_nf4_gemv<E, P, R><<<grid, 256, 0, s>>>(g);
  return cudaGetLastError();
}

}  // namespace

cudaError_t nf4_decode(const Nf4Source& src, const uint32_t* ids, void* out, uint32_t n, uint32_t selected,
                       uint32_t member_values, uint32_t storage, cudaStream_t s) {
  const uint32_t words = (n + 7u) / 8u;
  const uint32_t grid = uint32_t(std::min<uint64_t>((uint64_t(words) + 255) / 256, uint64_t(sm_count()) * 16));
  switch (storage) {
    case 0: k_nf4_decode<0><<<grid, 256, 0, s>>>(src, ids, out, n, words, selected, member_values); break;
    case 1: k_nf4_decode<1><<<grid, 256, 0, s>>>(src, ids, out, n, words, selected, member_values); break;
    default: k_nf4_decode<2><<<grid, 256, 0, s>>>(src, ids, out, n, words, selected, member_values);
  }
  return cudaGetLastError();
}

cudaError_t nf4_gemv(const Nf4Gemv& g, uint32_t max_rows, uint32_t elem, cudaStream_t s) {
  if (!aligned16(g.A)) return cudaErrorMisalignedAddress;  // A is read as 16-byte words
  const int module = max_rows <= 1 ? 0 : (max_rows <= 4 ? 1 : 2);
  if (elem == 0) {
    if (module == 0) return gemv_variant<0, 8, 1>(g, s);
    if (module == 1) return gemv_variant<0, 4, 4>(g, s);
    return gemv_variant<0, 1, 16>(g, s);
  }
  if (module == 0) return gemv_variant<1, 8, 1>(g, s);
  if (module == 1) return gemv_variant<1, 4, 4>(g, s);
  return gemv_variant<1, 1, 16>(g, s);
}

}  // namespace ack
