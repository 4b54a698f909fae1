// Device-side building blocks shared by the vq4 kernels: code access, status
// flags, constant-bank codebook slots and the certified nearest-entry search.
// The constant-bank array and CBook exist only where ACK_VQ_CONSTANT_BOOKS is
// defined (vq_codec.cu), so exactly one unit owns the array.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ack {

constexpr uint32_t kNonfinite = 1u;   // vq4.comp:5-8 status bits
constexpr uint32_t kLayout = 2u;
constexpr uint32_t kOptimizer = 4u;
constexpr uint32_t kStalled = 8u;     // a bounded pipeline wait ran out (no reference counterpart)

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
// launcher stages the caller's book into one of kBookSlots slots on the
// launch stream and picks the kernel instance compiled for that slot, so
// every book value the 16 x G filter multiplies by is a compile-time
// constant-bank operand: a warp-wide broadcast from the constant cache, with
// no shared-memory traffic. A slot holds up to three books of group 32 (the
// fused AdamW pass re-encodes W, M and V with three books) and, after them,
// each book's BookMeta.
//
// Within a slot a book is stored pair-interleaved: value j of entry e at
// float ((e / 2) * G + j) * 2 + e % 2, so the 16-byte quad (p, h) holds
// (c_2p[2h], c_2p+1[2h], c_2p[2h+1], c_2p+1[2h+1]): two entry pairs that one
// packed two-lane FMA each consumes.
constexpr int kBookSlots = 8;
constexpr int kSlotBookFloats = 3 * 16 * 32;
constexpr int kMetaFloats = 32;  // one BookMeta (19 words used), per book
constexpr int kSlotFloats = kSlotBookFloats + 3 * kMetaFloats;
template <int G>
__host__ __device__ constexpr int book_pos(int e, int j) { return ((e >> 1) * G + j) * 2 + (e & 1); }

#ifdef ACK_VQ_CONSTANT_BOOKS
__constant__ float4 c_books[kBookSlots][kSlotFloats / 4];


// Book B (0..2) of slot SLOT and its BookMeta, which the staging kernel
// stores after the books (float kSlotBookFloats + B * kMetaFloats).
template <int G, int SLOT, int B>
struct CBook {
  // entries 2p, 2p+1 at components 2h, 2h+1
  static __device__ __forceinline__ float4 quad(int p, int h) { return c_books[SLOT][(B * 16 * G + p * 2 * G) / 4 + h]; }
  static __device__ __forceinline__ float at(int e, int j) {
    return reinterpret_cast<const float*>(c_books[SLOT])[B * 16 * G + book_pos<G>(e, j)];
  }
  // quad i of the BookMeta (compile-time i: an immediate constant operand)
  static __device__ __forceinline__ float4 metaq(int i) {
    return c_books[SLOT][(kSlotBookFloats + B * kMetaFloats) / 4 + i];
  }
  // (q_2p, q_2p+1)
  static __device__ __forceinline__ float2 qpair(int p) {
    const float4 t = metaq(p >> 1);
    return (p & 1) ? make_float2(t.z, t.w) : make_float2(t.x, t.y);
  }
  static __device__ __forceinline__ float cmax2() { return metaq(4).x; }
  static __device__ __forceinline__ uint32_t uniq() { return __float_as_uint(metaq(4).y); }
  static __device__ __forceinline__ bool bad() { return __float_as_uint(metaq(4).z) != 0; }
};
#endif  // ACK_VQ_CONSTANT_BOOKS

// Facts about a codebook the search needs, computed once per launch by the
// staging kernel and stored in the slot beside the book:
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
static_assert(sizeof(BookMeta) <= kMetaFloats * 4, "BookMeta fits its slot region");

// Compute `m` for the row-major 16 x G book `book` with one warp (lanes
// 0..31 must all call it); no barrier.
template <int G>
__device__ void meta_compute(const float* __restrict__ book, BookMeta& m) {
  const int lane = threadIdx.x & 31;
  const int e = lane & 15;
  double s = 0.0;
  bool bad = false;
  for (int j = 0; j < G; ++j) {
    const float c = book[e * G + j];
    bad |= !finite32(c);
    s = __dadd_rn(s, __dmul_rn(double(c), double(c)));
  }
  bool uniq = true;
  for (int f = 0; f < e; ++f) {
    bool same = true;
    for (int j = 0; j < G; ++j) same &= book[f * G + j] == book[e * G + j];
    if (same) uniq = false;
  }
  float up = __double2float_ru(s);
  for (int o = 8; o; o >>= 1) up = fmaxf(up, __shfl_xor_sync(0xffffffffu, up, o));
  const uint32_t u = __ballot_sync(0xffffffffu, uniq) & 0xffffu;
  const uint32_t b = __ballot_sync(0xffffffffu, bad) & 0xffffu;
  if (lane < 16) m.q[e] = __double2float_rn(s);
  if (lane == 0) {
    m.cmax2 = up;
    m.uniq = u;
    m.bad = b != 0;
  }
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
// component as 8 two-lane packed FMAs, the book values constant-bank
// operands; ||x||^2 as two interleaved partial sums). |f_e - G_e| <= eps
// with G_e the exact value of the same expression and
// eps = (G + 8) 2^-23 (||x||^2 + max ||c||^2): twice the forward-error bound
// of the FMA chain, the rounded norms and the final FMA, plus an absolute
// floor for subnormal products. The float64 winner w (the reference
// encoder's choice) has f_w <= min_e f_e + 2 eps, so it lies in the
// candidate set {e : f_e <= min f + 2 eps} (duplicate rows removed: a
// duplicate of a lower row never wins a tie). A set of one entry is that
// winner; otherwise, or when anything is not finite, the exact float64 pass
// decides among the candidates.
//
// `src`, when not null, is where x lives in memory: the rare exact pass then
// reads the vector from there, so the values need not stay in registers
// after the filter.
// MEM: `src` is never null, so the register copy of x is never needed by the
// exact pass and stays out of local memory.
template <int G, class Book, bool MEM = false>
__device__ __forceinline__ uint32_t enc_vector(const float (&x)[G], bool* certified, const float* src = nullptr) {
  // acc[p] = (x.c_2p, x.c_2p+1): one packed FMA per component and entry pair,
  // each lane rounded like fmaf, components in order
  float2 acc[8];
#pragma unroll
  for (int p = 0; p < 8; ++p) acc[p] = make_float2(0.f, 0.f);
  float2 n2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int h = 0; h < G / 2; ++h) {
    const float x0 = x[2 * h], x1 = x[2 * h + 1];
    const float2 xx0 = make_float2(x0, x0), xx1 = make_float2(x1, x1);
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      const float4 c = Book::quad(p, h);
      acc[p] = __ffma2_rn(xx1, make_float2(c.z, c.w), __ffma2_rn(xx0, make_float2(c.x, c.y), acc[p]));
    }
    n2 = __ffma2_rn(make_float2(x0, x1), make_float2(x0, x1), n2);
  }
  const float nx2 = n2.x + n2.y;
  float f[16];
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    const float2 t = __ffma2_rn(make_float2(-2.f, -2.f), acc[p], Book::qpair(p));
    f[2 * p] = t.x;
    f[2 * p + 1] = t.y;
  }
  // the minimum as a tree (a NaN f_e is skipped here and caught below)
  float lo[8];
#pragma unroll
  for (int p = 0; p < 8; ++p) lo[p] = fminf(f[2 * p], f[2 * p + 1]);
#pragma unroll
  for (int w = 4; w; w >>= 1)
#pragma unroll
    for (int p = 0; p < w; ++p) lo[p] = fminf(lo[p], lo[p + w]);
  const float fb = lo[0];
  constexpr float kappa = float(G + 8) * (1.0f / 8388608.0f);
  const float eps = fmaf(kappa, nx2 + Book::cmax2(), 1e-37f);
  const float thr = fmaf(2.f, eps, fb);
  // f_e <= thr as the sign of thr - f_e (exact for a rounded difference; a
  // zero difference is +0, since thr = fb + 2 eps with eps > 0 is never -0),
  // gathered by funnel shifts: bit e of `over` is set
  // iff f_e > thr. A NaN f_e leaves `clean` false, where the mask is unused.
  uint32_t over_lo = 0, over_hi = 0;
#pragma unroll
  for (int p = 3; p >= 0; --p) {
    const float2 d = __ffma2_rn(make_float2(f[2 * p], f[2 * p + 1]), make_float2(-1.f, -1.f), make_float2(thr, thr));
    over_lo = __funnelshift_l(__float_as_uint(d.y), over_lo, 1);
    over_lo = __funnelshift_l(__float_as_uint(d.x), over_lo, 1);
    const float2 u =
        __ffma2_rn(make_float2(f[2 * p + 8], f[2 * p + 9]), make_float2(-1.f, -1.f), make_float2(thr, thr));
    over_hi = __funnelshift_l(__float_as_uint(u.y), over_hi, 1);
    over_hi = __funnelshift_l(__float_as_uint(u.x), over_hi, 1);
  }
  const uint32_t cand = ~((over_hi << 8) | over_lo) & Book::uniq();
  const bool clean = finite32(thr) && finite32(fb) && !Book::bad();
  if (clean && cand != 0u && (cand & (cand - 1u)) == 0u) {
    *certified = false;
    return uint32_t(__ffs(cand) - 1);
  }
  *certified = true;
  if (MEM || src) return enc_exact_mem<G, Book>(src, G, clean ? cand : 0xffffu);
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
