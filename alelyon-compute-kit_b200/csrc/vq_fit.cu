// fit_codebook on the device (ops 24, 25): Lloyd iterations with the
// certified search, books staged in shared memory.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "vq_common.cuh"

namespace ack {
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

cudaError_t run_adamw_fit_impl(const Plan& p, void* const* ptr, cudaStream_t s) {
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

cudaError_t run_fit_values_impl(const Plan& p, void* const* ptr, cudaStream_t s) {
  if (p.group == 8) return run_fit_values_group<8>(p, ptr, s);
  if (p.group == 16) return run_fit_values_group<16>(p, ptr, s);
  return run_fit_values_group<32>(p, ptr, s);
}

}  // namespace

cudaError_t launch_adamw_fit(const Plan& p, void* const* ptr, cudaStream_t s) {
  if (!aligned16(ptr[3])) return cudaErrorMisalignedAddress;  // sample rows are read in 16-byte quads
  return run_adamw_fit_impl(p, ptr, s);
}

cudaError_t launch_fit_values(const Plan& p, void* const* ptr, cudaStream_t s) {
  if (!aligned16(ptr[4])) return cudaErrorMisalignedAddress;  // the gathered sample is read in quads
  return run_fit_values_impl(p, ptr, s);
}

}  // namespace ack
