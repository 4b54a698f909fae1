// Device-side building blocks shared by the vq4 kernels: code access, status
// flags, constant-bank codebook slots and the certified nearest-entry search.
// Included by vq_kernels.cu only (it defines the constant-bank array).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ack {

constexpr uint32_t kNonfinite = 1u;   // vq4.comp:5-8 status bits
constexpr uint32_t kLayout = 2u;
constexpr uint32_t kOptimizer = 4u;

// Index of vector `v` in a packed image: nibble v%8 of word v/8, little-endian.
__device__ __forceinline__ uint32_t code_at(const uint32_t* __restrict__ codes, uint64_t v) {
  return (__ldg(codes + (v >> 3)) >> (4u * uint32_t(v & 7u))) & 15u;
}

__device__ __forceinline__ bool finite32(float x) {
  return (__float_as_uint(x) & 0x7f800000u) != 0x7f800000u;
}

// OR `bits` into the status word once per warp. Every lane of the warp that
// is active must call it.
__device__ __forceinline__ void flag_warp(uint32_t* status, uint32_t bits) {
  const uint32_t mask = __activemask();
  const uint32_t all = __reduce_or_sync(mask, bits);
  if (all && (threadIdx.x & 31) == (__ffs(mask) - 1)) atomicOr(status, all);
}

// Codebooks of in-flight encode launches live in the constant bank. The
// launcher copies the caller's book into one of kBookSlots slots on the
// launch stream (stream-ordered, device to device) and picks the kernel
// instance compiled for that slot, so every book value the 16 x G filter
// multiplies by is a compile-time constant-bank operand: a warp-wide
// broadcast from the constant cache, with no shared-memory traffic. A slot
// holds up to three books of group 32 (the fused AdamW pass re-encodes W, M
// and V with three books).
constexpr int kBookSlots = 8;
constexpr int kSlotFloats = 3 * 16 * 32;
__constant__ float4 c_books[kBookSlots][kSlotFloats / 4];

// Book B (0..2) of slot SLOT, row-major 16 x G, read in 16-byte quads: one
// constant-bank load feeds four FMAs (scalar constant loads with computed
// offsets would saturate the address-divergence unit instead).
template <int G, int SLOT, int B>
struct CBook {
  // components 4q..4q+3 of entry e
  static __device__ __forceinline__ float4 quad(int e, int q) { return c_books[SLOT][(B * 16 * G + e * G) / 4 + q]; }
  static __device__ __forceinline__ float at(int e, int j) {
    const float4 t = quad(e, j >> 2);
    const int r = j & 3;
    return r == 0 ? t.x : (r == 1 ? t.y : (r == 2 ? t.z : t.w));
  }
};

// Facts about a codebook the search needs, computed once per block:
//   q      fl32(||c_e||^2), the square norm summed in float64 then rounded
//   cmax2  max_e ||c_e||^2 rounded up
//   uniq   bit e set when row e differs from every lower row; a duplicate
//          row can never win because ties keep the lowest index
//   bad    the book holds a NaN or an infinity
struct alignas(16) BookMeta {
  float q[16];
  float cmax2;
  uint32_t uniq;
  uint32_t bad;
};

// The BookMeta of each slot's books, written once per launch by
// k_book_meta right after the slot is filled (stream-ordered before the
// kernels that read it).
__device__ BookMeta g_meta[kBookSlots][3];

// Compute `m` with the first warp of the block (the other threads return
// at once); no barrier.
template <int G, class Book>
__device__ void meta_compute(BookMeta& m) {
  if (threadIdx.x < 32) {
    const int e = threadIdx.x & 15;
    double s = 0.0;
    bool bad = false;
    for (int j = 0; j < G; ++j) {
      const float c = Book::at(e, j);
      bad |= !finite32(c);
      s = __dadd_rn(s, __dmul_rn(double(c), double(c)));
    }
    bool uniq = true;
    for (int f = 0; f < e; ++f) {
      bool same = true;
      for (int j = 0; j < G; ++j) same &= Book::at(f, j) == Book::at(e, j);
      if (same) uniq = false;
    }
    float up = __double2float_ru(s);
    for (int o = 8; o; o >>= 1) up = fmaxf(up, __shfl_xor_sync(0xffffffffu, up, o));
    const uint32_t u = __ballot_sync(0xffffffffu, uniq) & 0xffffu;
    const uint32_t b = __ballot_sync(0xffffffffu, bad) & 0xffffu;
    if (threadIdx.x < 16) m.q[e] = __double2float_rn(s);
    if (threadIdx.x == 0) {
      m.cmax2 = up;
      m.uniq = u;
      m.bad = b != 0;
    }
  }
}

// Copy slot SLOT's meta of book B into shared memory; all threads call it,
// it ends with a barrier.
template <int SLOT, int B>
__device__ __forceinline__ void meta_load(BookMeta& m) {
  constexpr int kWords = sizeof(BookMeta) / 4;
  if (threadIdx.x < kWords)
    reinterpret_cast<uint32_t*>(&m)[threadIdx.x] = reinterpret_cast<const uint32_t*>(&g_meta[SLOT][B])[threadIdx.x];
  __syncthreads();
}

// Exact nearest entry among the set bits of `cand`, computed the way the
// reference CPU encoder computes it (vq.py:167-174): float64 distances
// accumulated in component order, d += (v_j - b_j)^2 with each operation
// rounded on its own, over the first `valid` components; the lowest index
// wins a tie; a NaN distance wins at its first occurrence (np.argmin).
template <int G, class Book>
__device__ __noinline__ uint32_t enc_exact_mem(const float* x, int valid, uint32_t cand);

// Inline wrapper: the exact pass is rare, so it lives out of line and the
// hot path's register budget stays the filter's.
template <int G, class Book>
__device__ __forceinline__ uint32_t enc_exact(const float (&x)[G], int valid, uint32_t cand) {
  return enc_exact_mem<G, Book>(x, valid, cand);
}

template <int G, class Book>
__device__ __noinline__ uint32_t enc_exact_mem(const float* x, int valid, uint32_t cand) {
  double best = 0.0;
  int chosen = -1;
  bool nan_seen = false;
  for (int e = 0; e < 16; ++e) {
    if (!((cand >> e) & 1u)) continue;
    double d = 0.0;
    for (int j = 0; j < valid; ++j) {
      const double t = __dsub_rn(double(x[j]), double(Book::at(e, j)));
      d = __dadd_rn(d, __dmul_rn(t, t));
    }
    if (nan_seen) continue;
    if (d != d) {
      chosen = e;
      nan_seen = true;
    } else if (chosen < 0 || d < best) {
      best = d;
      chosen = e;
    }
  }
  return chosen < 0 ? 0u : uint32_t(chosen);
}

// Certified nearest entry of one complete vector.
//
// Filter: f_e = ||c_e||^2 - 2 x.c_e in FP32 (16 fused multiply-adds per
// component, the book values constant-bank operands). |f_e - G_e| <= eps
// with G_e the exact value of the same expression and
// eps = (G + 8) 2^-23 (||x||^2 + max ||c||^2): twice the forward-error bound
// of the FMA chain, the rounded norms and the final FMA, plus an absolute
// floor for subnormal products. Any entry whose f_e lies within 2 eps of the
// minimum could be the float64 winner (the float64 distances differ from the
// exact ones by far less than eps); when that candidate set holds more than
// one distinct row, or anything is not finite, the exact float64 pass decides
// among the candidates. The result is always the reference encoder's choice.
template <int G, class Book>
__device__ __forceinline__ uint32_t enc_vector(const float (&x)[G], const BookMeta& m, bool* certified) {
  float acc[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) acc[e] = 0.f;
  float nx2 = 0.f;
#pragma unroll
  for (int q = 0; q < G / 4; ++q) {
    const float x0 = x[4 * q], x1 = x[4 * q + 1], x2 = x[4 * q + 2], x3 = x[4 * q + 3];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float4 c = Book::quad(e, q);  // components in order: the same sums as one by one
      acc[e] = fmaf(x3, c.w, fmaf(x2, c.z, fmaf(x1, c.y, fmaf(x0, c.x, acc[e]))));
    }
    nx2 = fmaf(x3, x3, fmaf(x2, x2, fmaf(x1, x1, fmaf(x0, x0, nx2))));
  }
  float f[16];
  const float4* q4 = reinterpret_cast<const float4*>(m.q);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 q = q4[i];
    f[4 * i + 0] = fmaf(-2.f, acc[4 * i + 0], q.x);
    f[4 * i + 1] = fmaf(-2.f, acc[4 * i + 1], q.y);
    f[4 * i + 2] = fmaf(-2.f, acc[4 * i + 2], q.z);
    f[4 * i + 3] = fmaf(-2.f, acc[4 * i + 3], q.w);
  }
  float fb = f[0];
  uint32_t best = 0;
#pragma unroll
  for (int e = 1; e < 16; ++e)
    if (f[e] < fb) {
      fb = f[e];
      best = uint32_t(e);
    }
  constexpr float kappa = float(G + 8) * (1.0f / 8388608.0f);
  const float eps = fmaf(kappa, nx2 + m.cmax2, 1e-37f);
  const float thr = fmaf(2.f, eps, fb);
  uint32_t cand = 0;
#pragma unroll
  for (int e = 0; e < 16; ++e) cand |= uint32_t(f[e] <= thr) << e;
  cand &= m.uniq;
  const bool clean = finite32(thr) && finite32(fb) && !m.bad;
  if (clean && cand == (1u << best)) {
    *certified = false;
    return best;
  }
  *certified = true;
  return enc_exact<G, Book>(x, G, clean ? cand : 0xffffu);
}

// OR together the nibbles of the 8 lanes that share a word and return the
// packed word (valid in every lane). All 32 lanes must call it.
__device__ __forceinline__ uint32_t pack_nibbles(uint32_t idx) {
  uint32_t w = idx << (4u * (threadIdx.x & 7u));
  w |= __shfl_xor_sync(0xffffffffu, w, 1);
  w |= __shfl_xor_sync(0xffffffffu, w, 2);
  w |= __shfl_xor_sync(0xffffffffu, w, 4);
  return w;
}

// The shader's AdamW for one value (vq4.comp:98-115), every operation
// rounded on its own. Returns status bits; on a nonzero return from the
// input checks the outputs are not meaningful (the shader writes nothing).
struct AdamwCoefs {
  float lr, beta1, beta2, eps, decay, c1, c2;
  uint32_t status;  // nonzero: coefficients refused (vq4.comp:92-97)
};

__device__ __forceinline__ AdamwCoefs load_coefs(const float* __restrict__ c) {
  AdamwCoefs k;
  k.lr = c[0];
  k.beta1 = c[1];
  k.beta2 = c[2];
  k.eps = c[3];
  k.decay = c[4];
  k.c1 = c[5];
  k.c2 = c[6];
  k.status = 0;
  const float all[7] = {k.lr, k.beta1, k.beta2, k.eps, k.decay, k.c1, k.c2};
  for (int j = 0; j < 7; ++j)
    if (!finite32(all[j])) k.status = kNonfinite;
  if (!k.status && (k.lr < 0.f || k.beta1 < 0.f || k.beta1 >= 1.f || k.beta2 < 0.f || k.beta2 >= 1.f ||
                    k.eps <= 0.f || k.decay < 0.f || k.c1 <= 0.f || k.c1 > 1.f || k.c2 <= 0.f || k.c2 > 1.f))
    k.status = kOptimizer;
  return k;
}

// Returns 0, or the status bits of a refused input (then the outputs are
// unspecified), or kNonfinite with outputs written for a nonfinite result.
__device__ __forceinline__ uint32_t adamw_value(const AdamwCoefs& k, float w, float m, float v, float g,
                                                float* nw, float* nm, float* nv, bool* skip) {
  *skip = false;
  if (!finite32(w) || !finite32(m) || !finite32(v) || !finite32(g)) {
    *skip = true;
    return kNonfinite;
  }
  if (v < 0.f) {
    *skip = true;
    return kOptimizer;
  }
  const float next_m = __fadd_rn(__fmul_rn(k.beta1, m), __fmul_rn(__fsub_rn(1.f, k.beta1), g));
  const float next_v = __fadd_rn(__fmul_rn(k.beta2, v), __fmul_rn(__fsub_rn(1.f, k.beta2), __fmul_rn(g, g)));
  const float cm = __fdiv_rn(next_m, k.c1);
  const float cv = __fdiv_rn(next_v, k.c2);
  const float den = __fadd_rn(__fsqrt_rn(cv), k.eps);
  const float decayed = __fmul_rn(w, __fsub_rn(1.f, __fmul_rn(k.lr, k.decay)));
  const float next_w = __fsub_rn(decayed, __fdiv_rn(__fmul_rn(k.lr, cm), den));
  *nw = next_w;
  *nm = next_m;
  *nv = next_v;
  const bool ok = finite32(next_m) && finite32(next_v) && finite32(cm) && finite32(cv) && finite32(den) &&
                  finite32(decayed) && finite32(next_w);
  return ok ? 0u : kNonfinite;
}

}  // namespace ack
