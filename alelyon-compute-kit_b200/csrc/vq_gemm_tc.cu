// Dense activations times coded weights on the tensor cores (op 16, flag 8):
// Y[e] = X[e] * decode(W[e])^T, W stored N x K with groups of G along K.
//
// Formulation. With T = K / G groups per row and P[m][t][i] = x[m, tG:tG+G]
// . c_i (the projection of each activation segment on each of the 16
// codebook entries),
//     Y[m][n] = sum_t P[m][t][idx(n, t)] = sum_{t,i} OneHot[n][(t,i)] P[m][(t,i)],
// a GEMM with K' = 16 T. The one-hot operand is exact in bf16; P is split
// into bf16 hi + lo halves (P - hi rounded again), which together carry 16
// mantissa bits, and both halves ride in one MMA as the N dimension:
// B = [P_hi ; P_lo] (2 Mp rows). The accumulators hold sum hi and sum lo in
// FP32; the epilogue adds them. Every product in the MMA is exact (1 x bf16),
// so the error is the FP32 accumulation plus ~2^-17 |P| per term.
//
//   k_dense_tc_prep   P for every (expert, row m, group t, entry i): bf16 hi
//                     and lo into the caller's workspace, K'-contiguous rows
//                     [e][n' < 2 Mp][k' = 16 t + i] (rows m >= M are zero)
//   k_dense_tc        persistent, one CTA per SM over (expert, 128-row tile)
//                     work items. Warp 0: TMA loads of B chunks (2 Mp x 64
//                     k', SWIZZLE_128B) into an SB-stage ring. Warp 1 lane 0:
//                     tcgen05.mma.kind::f16 with A in tensor memory (M 128,
//                     N = 2 Mp, K 16; four per 64-wide K' chunk). Warps 4-7:
//                     each thread owns one W row (TMEM lane), builds the
//                     one-hot words of 4 groups from its codes and stores
//                     them with tcgen05.st into an SA-stage TMEM ring (one
//                     mbarrier arrival per warp per chunk). Warps
//                     8-11: epilogue, tcgen05.ld of the finished accumulator
//                     (ND buffers), hi + lo, coalesced stores of Y.
//
// The A operand never touches shared memory: the one-hot words go from
// registers to tensor memory, and the tensor core reads them from there.
// Shared memory carries only B. Every mbarrier wait is bounded: one that runs
// out sets kStalled, and the block waits (bounded) for its own TMA loads and
// MMAs in flight before TMEM is released.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "vq_common.cuh"
#include "vq_tc.cuh"

namespace ack {
namespace {

using tc::mb_arrive;
using tc::mb_expect;
using tc::mb_init;
using tc::mb_wait;
using tc::smem_u32;

constexpr int kTcRows = 128;      // W rows per work item (the MMA's M)
constexpr int kChunk = 64;        // K' per chunk: one 128-byte bf16 row of B
constexpr int kSA = 8;            // A stages in tensor memory (32 columns each)
constexpr int kBatch = 4;         // chunks the builders store between waits for their TMEM stores
constexpr int kTcThreads = 384;   // 12 warps

template <int NP>
struct TcCfg {
  static constexpr int ND = NP <= 128 ? 2 : 1;                      // accumulator buffers
  static constexpr uint32_t kStage = uint32_t(NP) * 128u;           // bytes of one B chunk
  static constexpr int SB = std::max(2, std::min(8, int(98304u / kStage)));
  static constexpr uint32_t kColsUsed = uint32_t(kSA) * 32u + uint32_t(ND) * NP;
  static constexpr uint32_t kCols = kColsUsed <= 32 ? 32u : kColsUsed <= 64 ? 64u : kColsUsed <= 128 ? 128u
                                  : kColsUsed <= 256 ? 256u : 512u;
  // at least 116 KB, so that one CTA holds an SM (grids are one CTA per SM)
  static constexpr size_t kSmem = std::max<size_t>(1024 + size_t(SB) * kStage, 116u * 1024u);
  // D: FP32, A and B bf16, both K-major, N = NP, M = 128
  static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(NP >> 3) << 17) |
                                     (uint32_t(128 >> 4) << 24);
};

// P of one (expert, row m < Mp, group t): 16 entries, bf16 hi into row m and
// lo into row Mp + m of the expert's block. Rows m >= mc are written as zeros.
template <int G>
__global__ void __launch_bounds__(256) k_dense_tc_prep(const float* __restrict__ X, const float* __restrict__ books,
                                                        __nv_bfloat16* __restrict__ P, uint32_t M, uint32_t m0,
                                                        uint32_t mc, uint32_t mp, uint32_t K,
                                                        uint32_t* __restrict__ status) {
  __shared__ float sb[16 * G];
  const uint32_t e = blockIdx.y;
  for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) sb[i] = books[uint64_t(e) * 16 * G + i];
  __syncthreads();
  if (blockIdx.x == 0 && m0 == 0) {
    uint32_t bits = 0;
    for (int i = threadIdx.x; i < 16 * G; i += blockDim.x) bits |= finite32(sb[i]) ? 0u : kNonfinite;
    flag_warp(status, bits);
  }
  const uint32_t T = K / G;
  const uint64_t items = uint64_t(mp) * T;
  const uint64_t kp = uint64_t(16) * T;                       // K' of one row of P
  __nv_bfloat16* pe = P + uint64_t(e) * 2 * mp * kp;
  for (uint64_t it = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; it < items;
       it += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t m = uint32_t(it / T), t = uint32_t(it % T);
    uint32_t hi[8], lo[8];
    if (m < mc) {
      const float4* xs = reinterpret_cast<const float4*>(X + (uint64_t(e) * M + m0 + m) * K + uint64_t(t) * G);
      float x[G];
#pragma unroll
      for (int q = 0; q < G / 4; ++q) {
        const float4 v = __ldg(xs + q);
        x[4 * q] = v.x;
        x[4 * q + 1] = v.y;
        x[4 * q + 2] = v.z;
        x[4 * q + 3] = v.w;
      }
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        float p0 = 0.f, p1 = 0.f;
#pragma unroll
        for (int j = 0; j < G; ++j) {
          p0 = fmaf(x[j], sb[i * G + j], p0);
          p1 = fmaf(x[j], sb[(i + 1) * G + j], p1);
        }
        const __nv_bfloat16 h0 = __float2bfloat16_rn(p0), h1 = __float2bfloat16_rn(p1);
        const __nv_bfloat16 l0 = __float2bfloat16_rn(p0 - __bfloat162float(h0));
        const __nv_bfloat16 l1 = __float2bfloat16_rn(p1 - __bfloat162float(h1));
        hi[i / 2] = uint32_t(__bfloat16_as_ushort(h0)) | (uint32_t(__bfloat16_as_ushort(h1)) << 16);
        lo[i / 2] = uint32_t(__bfloat16_as_ushort(l0)) | (uint32_t(__bfloat16_as_ushort(l1)) << 16);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) hi[i] = lo[i] = 0u;
    }
    uint4* dh = reinterpret_cast<uint4*>(pe + uint64_t(m) * kp + uint64_t(t) * 16);
    uint4* dl = reinterpret_cast<uint4*>(pe + uint64_t(mp + m) * kp + uint64_t(t) * 16);
    dh[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    dh[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
    dl[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    dl[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
  }
}

// The eight 32-bit words of the bf16 one-hot vector of entry `e` (1.0 at
// element e of 16).
__device__ __forceinline__ void one_hot8(uint32_t e, uint32_t* w) {
  const uint32_t v = (e & 1u) ? 0x3F800000u : 0x00003F80u;
  const uint32_t h = e >> 1;
#pragma unroll
  for (uint32_t j = 0; j < 8; ++j) w[j] = (h == j) ? v : 0u;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

struct TcArgs {
  const uint32_t* codes;   // canonical images, E x (N x T/8 words)
  float* Y;                // (E, M, N)
  uint32_t M, m0, mc, mp;  // rows of X/Y, this chunk's first row and row count, padded rows of P
  uint32_t N, T, E;
  uint32_t* status;
};

template <int NP>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_dense_tc(const __grid_constant__ CUtensorMap pmap, TcArgs a) {
  using C = TcCfg<NP>;
  constexpr int SB = C::SB, ND = C::ND;
  extern __shared__ unsigned char tc_smem[];
  unsigned char* ring = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem) + 1023) &
                                                         ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_b[SB], free_b[SB], full_a[kSA], free_a[kSA], full_d[ND], free_d[ND];
  __shared__ uint32_t tmem_base;
  const uint32_t tid = threadIdx.x, warp = tid / 32, lane = tid & 31;
  const uint32_t tiles_per_expert = (a.N + kTcRows - 1) / kTcRows;
  const uint64_t units = uint64_t(a.E) * tiles_per_expert;
  const uint32_t mine = units > blockIdx.x ? uint32_t((units - blockIdx.x + gridDim.x - 1) / gridDim.x) : 0u;
  const uint32_t CH = a.T / 4;  // K' chunks per work item (4 groups each)

  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(C::kCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int s = 0; s < SB; ++s) {
      mb_init(&full_b[s], 1);
      mb_init(&free_b[s], 1);
    }
    // the builders and the epilogue arrive once per warp (four warps each)
    for (int s = 0; s < kSA; ++s) {
      mb_init(&full_a[s], 4);
      mb_init(&free_a[s], 1);
    }
    for (int b = 0; b < ND; ++b) {
      mb_init(&full_d[b], 1);
      mb_init(&free_d[b], 4);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  const uint32_t a_col = 0, d_col = uint32_t(kSA) * 32u;
  bool ok = true;

  if (warp == 0) {
    // producer: one TMA load of B (2 Mp rows x 64 k') per chunk
    if (lane == 0) {
      uint64_t issued = 0;
      for (uint32_t it = 0; it < mine && ok; ++it) {
        const uint64_t u = blockIdx.x + uint64_t(it) * gridDim.x;
        const int32_t row = int32_t((u / tiles_per_expert) * uint64_t(2 * a.mp));
        for (uint32_t c = 0; c < CH; ++c) {
          const uint64_t q = uint64_t(it) * CH + c;
          const uint32_t s = uint32_t(q % SB);
          if (q >= uint64_t(SB) && !(ok = mb_wait(&free_b[s], uint32_t((q / SB) - 1) & 1u))) break;
          mb_expect(&full_b[s], C::kStage);
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
              "[%4];" ::"r"(smem_u32(ring + s * C::kStage)),
              "l"(&pmap), "r"(int32_t(c * kChunk)), "r"(row), "r"(smem_u32(&full_b[s]))
              : "memory");
          ++issued;
        }
      }
      if (!ok) atomicOr(a.status, kStalled);
      // the loads in flight land before the block may exit
      for (uint64_t q = issued > uint64_t(SB) ? issued - SB : 0; q < issued; ++q)
        if (!mb_wait(&full_b[q % SB], uint32_t(q / SB) & 1u)) atomicOr(a.status, kStalled);
    }
  } else if (warp == 1) {
    // MMA issuer
    if (lane == 0) {
      uint64_t committed = 0;
      for (uint32_t it = 0; it < mine && ok; ++it) {
        const uint32_t db = it % ND;
        if (it >= uint32_t(ND) && !(ok = mb_wait(&free_d[db], ((it / ND) - 1) & 1u))) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + d_col + db * NP;
        for (uint32_t c = 0; c < CH; ++c) {
          const uint64_t q = uint64_t(it) * CH + c;
          const uint32_t s = uint32_t(q % SB), sa = uint32_t(q % kSA);
          if (!(ok = mb_wait(&full_b[s], uint32_t(q / SB) & 1u))) break;
          if (!(ok = mb_wait(&full_a[sa], uint32_t(q / kSA) & 1u))) break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t b_addr = smem_u32(ring + s * C::kStage);
#pragma unroll
          for (uint32_t i = 0; i < 4; ++i)
            asm volatile(
                "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::
                    "r"(d), "r"(tmem + a_col + sa * 32u + 8u * i), "l"(tc::Swz<32>::desc(b_addr + 32u * i)),
                "r"(C::kIdesc), "r"(uint32_t(c | i))
                : "memory");
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                           smem_u32(&free_b[s]))
                       : "memory");
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                           smem_u32(&free_a[sa]))
                       : "memory");
          ++committed;
        }
        if (!ok) break;
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&full_d[db]))
                     : "memory");
      }
      if (!ok) atomicOr(a.status, kStalled);
      // every committed MMA completes before TMEM is released: chunk q was
      // issued only after its A slot's previous phase completed, so free_a's
      // parity names the last commit's phase unambiguously
      if (committed) {
        const uint64_t q = committed - 1;
        if (!mb_wait(&free_a[q % kSA], uint32_t(q / kSA) & 1u)) atomicOr(a.status, kStalled);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // one-hot builders: thread r owns W row r of the item (TMEM lane r). A
    // row's codes arrive 128 bytes (8 uint4, 64 chunks) at a time, all eight
    // loads in flight at once, with the next segment's line prefetched into
    // L1; each chunk's words are built before its slot is awaited; TMEM
    // stores are awaited once per batch of kBatch chunks.
    const uint32_t r = tid - 128, lane_base = (warp & 3u) * 32u;
    const uint64_t expert_words = uint64_t(a.N) * (a.T / 8);
    const uint32_t nu = a.T / 32;  // uint4 of codes per row
    auto row_src = [&](uint32_t it2, bool* valid) {
      const uint64_t u = blockIdx.x + uint64_t(it2) * gridDim.x;
      const uint64_t e = u / tiles_per_expert;
      const uint32_t n = uint32_t(u % tiles_per_expert) * kTcRows + r;
      *valid = n < a.N;
      return reinterpret_cast<const uint4*>(a.codes + e * expert_words + uint64_t(*valid ? n : 0) * (a.T / 8));
    };
    uint64_t q = 0;  // chunks built so far
    for (uint32_t it = 0; it < mine && ok; ++it) {
      bool valid;
      const uint4* src = row_src(it, &valid);
      for (uint32_t seg = 0; seg < nu && ok; seg += 8) {
        uint4 sv[8];
#pragma unroll
        for (uint32_t i = 0; i < 8; ++i)
          sv[i] = (valid && seg + i < nu) ? __ldg(src + seg + i) : make_uint4(0, 0, 0, 0);
        {  // the next segment's line (this row, or the next item's row) into L1
          bool nvalid = valid;
          const uint4* nsrc = seg + 8 < nu ? src + seg + 8 : (it + 1 < mine ? row_src(it + 1, &nvalid) : nullptr);
          if (nsrc && nvalid) asm volatile("prefetch.global.L1 [%0];" ::"l"(nsrc));
        }
#pragma unroll
        for (uint32_t i = 0; i < 8; ++i) {
          if (seg + i >= nu || !ok) break;
          const uint4 cur = sv[i];
#pragma unroll 1
          for (uint32_t half = 0; half < 2 && ok; ++half) {  // two batches of kBatch chunks
#pragma unroll
            for (uint32_t b = 0; b < kBatch; ++b) {
              const uint32_t cc = half * kBatch + b;
              const uint32_t word = half ? (b < 2 ? cur.z : cur.w) : (b < 2 ? cur.x : cur.y);
              const uint32_t bits16 = word >> (16u * (cc & 1u));
              uint32_t w[32];
#pragma unroll
              for (int g = 0; g < 4; ++g) one_hot8((bits16 >> (4 * g)) & 15u, w + 8 * g);
              const uint64_t qc = q + b;
              const uint32_t sa = uint32_t(qc % kSA);
              if (qc >= uint64_t(kSA)) {
                // warp-uniform: tcgen05.st is .sync.aligned
                const uint32_t got = lane == 0 ? uint32_t(mb_wait(&free_a[sa], uint32_t((qc / kSA) - 1) & 1u)) : 0u;
                if (!(ok = __shfl_sync(0xffffffffu, got, 0) != 0u)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");  // the MMAs reading it are done
              }
              tmem_st32(tmem + (lane_base << 16) + a_col + sa * 32u, w);
            }
            if (!ok) break;
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0)  // one arrival per warp and chunk
              for (uint32_t b = 0; b < kBatch; ++b) mb_arrive(&full_a[uint32_t((q + b) % kSA)]);
            q += kBatch;
          }
        }
      }
    }
    // on the stall path a batch may have stores in flight: they land before TMEM is released
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    if (!ok) atomicOr(a.status, kStalled);
  } else if (warp >= 8) {
    // epilogue: thread r reads TMEM lane r (W row r), hi + lo, stores Y
    const uint32_t r = tid - 256, lane_base = (warp & 3u) * 32u;
    uint32_t bits = 0;
    for (uint32_t it = 0; it < mine && ok; ++it) {
      const uint32_t db = it % ND;
      if (!(ok = __all_sync(0xffffffffu, mb_wait(&full_d[db], (it / ND) & 1u)))) break;  // warp-uniform
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint64_t u = blockIdx.x + uint64_t(it) * gridDim.x;
      const uint64_t e = u / tiles_per_expert;
      const uint32_t n = uint32_t(u % tiles_per_expert) * kTcRows + r;
      const uint32_t base = tmem + (lane_base << 16) + d_col + db * NP;
      float* y = a.Y + (e * a.M + a.m0) * a.N + n;
      for (uint32_t mb = 0; mb < a.mp; mb += 16) {
        uint32_t hi[16], lo[16];
        tmem_ld16(base + mb, hi);
        tmem_ld16(base + a.mp + mb, lo);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (n < a.N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const uint32_t m = mb + j;
            if (m < a.mc) {
              const float v = __uint_as_float(hi[j]) + __uint_as_float(lo[j]);
              bits |= finite32(v) ? 0u : kNonfinite;
              y[uint64_t(m) * a.N] = v;
            }
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mb_arrive(&free_d[db]);
    }
    if (!ok) atomicOr(a.status, kStalled);
    flag_warp(a.status, bits);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 2) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kCols));
}

// The tensor map of the P workspace: rows of K' bf16, boxes of 2 Mp rows x
// 64 elements (128 bytes), 128-byte swizzle (the UMMA K-major layout).
bool p_tensor_map(const void* ws, uint64_t kp, uint64_t rows, uint32_t box_rows, CUtensorMap* map) {
  const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return false;
  const cuuint64_t dims[2] = {cuuint64_t(kp), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(kp) * 2};
  const cuuint32_t box[2] = {cuuint32_t(kChunk), box_rows};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ws), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NP>
cudaError_t launch_tc_np(const CUtensorMap& map, const TcArgs& a, cudaStream_t s) {
  using C = TcCfg<NP>;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(k_dense_tc<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(C::kSmem));
  });
  if (attr != cudaSuccess) return attr;
  const uint64_t units = uint64_t(a.E) * ((a.N + kTcRows - 1) / kTcRows);
  const uint32_t grid = uint32_t(std::min<uint64_t>(units, uint64_t(sm_count())));
  k_dense_tc<NP><<<grid, kTcThreads, C::kSmem, s>>>(map, a);
  return cudaGetLastError();
}

template <int G>
cudaError_t dense_tc_group(const float* X, const uint32_t* codes, const float* books, float* Y, uint32_t M,
                           uint32_t N, uint32_t K, uint32_t E, void* ws, uint32_t* status, cudaStream_t s) {
  const uint32_t T = K / G;
  const uint64_t kp = uint64_t(16) * T;
  for (uint32_t m0 = 0; m0 < M; m0 += kDenseTcMaxRows) {
    const uint32_t mc = std::min<uint32_t>(kDenseTcMaxRows, M - m0);
    const uint32_t mp = dense_tc_padded_rows(mc);
    const uint64_t items = uint64_t(mp) * T;
    const dim3 pgrid(uint32_t(std::min<uint64_t>((items + 255) / 256, 1024)), E);
    k_dense_tc_prep<G><<<pgrid, 256, 0, s>>>(X, books, static_cast<__nv_bfloat16*>(ws), M, m0, mc, mp, K, status);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    CUtensorMap map;
    if (!p_tensor_map(ws, kp, uint64_t(E) * 2 * mp, 2 * mp, &map)) return cudaErrorInvalidValue;
    TcArgs a{codes, Y, M, m0, mc, mp, N, T, E, status};
    switch (mp) {
      case 8: err = launch_tc_np<16>(map, a, s); break;
      case 16: err = launch_tc_np<32>(map, a, s); break;
      case 24: err = launch_tc_np<48>(map, a, s); break;
      case 32: err = launch_tc_np<64>(map, a, s); break;
      case 40: err = launch_tc_np<80>(map, a, s); break;
      case 48: err = launch_tc_np<96>(map, a, s); break;
      case 56: err = launch_tc_np<112>(map, a, s); break;
      case 64: err = launch_tc_np<128>(map, a, s); break;
      case 80: err = launch_tc_np<160>(map, a, s); break;
      case 96: err = launch_tc_np<192>(map, a, s); break;
      case 112: err = launch_tc_np<224>(map, a, s); break;
      default: err = launch_tc_np<256>(map, a, s); break;
    }
    if (err != cudaSuccess) return err;
  }
  return cudaSuccess;
}

}  // namespace

cudaError_t launch_dense_tc(const Plan& p, void* const* ptr, cudaStream_t s) {
  const float* X = static_cast<const float*>(ptr[0]);
  const uint32_t* codes = static_cast<const uint32_t*>(ptr[1]);
  const float* books = static_cast<const float*>(ptr[2]);
  void* ws = ptr[4];
  float* Y = static_cast<float*>(ptr[5]);
  uint32_t* status = static_cast<uint32_t*>(ptr[7]);
  if (!aligned16(X) || !aligned16(codes) || !aligned16(ws)) return cudaErrorMisalignedAddress;
  const uint32_t M = uint32_t(p.m), N = uint32_t(p.n), K = uint32_t(p.k);
  switch (p.group) {
    case 8: return dense_tc_group<8>(X, codes, books, Y, M, N, K, p.batch, ws, status, s);
    case 16: return dense_tc_group<16>(X, codes, books, Y, M, N, K, p.batch, ws, status, s);
    default: return dense_tc_group<32>(X, codes, books, Y, M, N, K, p.batch, ws, status, s);
  }
}

}  // namespace ack
