// Dense activations times coded weights on the tensor cores (op 16, flag 8):
// Y[e] = X[e] * decode(W[e])^T, W stored N x K with groups of G along K.
//
// Formulation. With T = K / G groups per row and P[m][t][i] = x[m, tG:tG+G]
// . c_i (the projection of each activation segment on each of the 16
// codebook entries),
//     Y[m][n] = sum_t P[m][t][idx(n, t)] = sum_{t,i} P[m][(t,i)] OneHot[n][(t,i)],
// a GEMM with K' = 16 T. The one-hot operand is exact in bf16; P is split
// into bf16 hi + lo halves (P - hi rounded again), which together carry 16
// mantissa bits. Every product in the MMA is exact (bf16 x 1), so the error
// is the FP32 accumulation plus ~2^-17 |P| per term.
//
// Operand roles. One tcgen05.mma of M = 128 costs about the same whatever its
// N (measured ~150 cycles for K = 16 with N from 32 to 256): the 128-row A
// slab sets the price. So the operand with few rows, P, is A (M = 128: 64
// rows of X, hi and lo interleaved), and the codes are B with N = 256 W rows
// per instruction. The one-hot B goes through shared memory (an MMA reads B
// only from there).
//
//   k_dense_tc_prep   P of every (expert, 64-row tile of X, group, entry):
//                     row 2m = bf16(P[m]), row 2m + 1 = bf16(P[m] - hi), in
//                     the caller's workspace [e][tile][128][K'] (rows of X
//                     beyond M are zero)
//   k_dense_tc        persistent, one CTA per SM over (expert, 256-row tile
//                     of W, 64-row tile of X) items. Warp 0: TMA loads of A
//                     chunks (128 rows x 64 k', 128-byte swizzle). Warps 4-11
//                     (thread = W row): the row's one-hot entries of 4 groups
//                     per chunk in the B stage (same swizzle), kept up to date
//                     by clearing the 4 entries set there last time and
//                     setting the 4 new ones. Warp 1 lane 0: four
//                     tcgen05.mma.kind::f16 per chunk (M 128, N 256, K 16),
//                     accumulators in TMEM (two buffers of 256 columns).
//                     Warps 12-15: tcgen05.ld of the finished accumulator,
//                     hi + lo by a lane-pair shuffle, Y rows stored as
//                     128-byte runs.
//
// Every mbarrier wait is bounded: one that runs out sets kStalled, and the
// block waits (bounded) for its own TMA loads and MMAs in flight before TMEM
// is released. Barrier arrivals are one per warp.
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

constexpr int kWRows = 256;        // W rows per item (the MMA's N)
constexpr int kPRows = 128;        // P rows per item (the MMA's M): 64 rows of X, hi and lo
constexpr int kXRows = 64;         // rows of X per item
constexpr int kChunk = 64;         // K' per chunk: one 128-byte bf16 row of each operand
constexpr int kStages = 4;         // stages of A (TMA) and B (one-hot), filled and released together
constexpr int kBuilderWarps = 8;   // one W row per thread
constexpr int kTcThreads = 512;    // 16 warps: 0 TMA, 1 MMA, 2 TMEM, 3 idle, 4-11 builders, 12-15 epilogue
constexpr uint32_t kAStage = kPRows * 128u;   // 16 KB
constexpr uint32_t kBStage = kWRows * 128u;   // 32 KB
constexpr uint32_t kCols = 512;               // two 256-column accumulators
constexpr size_t kTcSmem = 1024 + size_t(kStages) * (kAStage + kBStage);
// D FP32, A and B bf16, both K-major, N = 256, M = 128
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(kWRows >> 3) << 17) |
                            (uint32_t(kPRows >> 4) << 24);

// P of one (expert, X tile, row m < 64, group t): 16 entries, hi into row 2m,
// lo into row 2m + 1. Rows of X at or beyond mc are written as zeros.
template <int G>
__global__ void __launch_bounds__(256) k_dense_tc_prep(const float* __restrict__ X, const float* __restrict__ books,
                                                        __nv_bfloat16* __restrict__ P, uint32_t M, uint32_t m0,
                                                        uint32_t mc, uint32_t tiles, uint32_t K,
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
  const uint64_t kp = uint64_t(16) * T;                       // K' of one row of P
  const uint64_t items = uint64_t(tiles) * kXRows * T;
  __nv_bfloat16* pe = P + uint64_t(e) * tiles * kPRows * kp;
  for (uint64_t it = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; it < items;
       it += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t m = uint32_t(it / T), t = uint32_t(it % T);   // m: row within this pass (tile * 64 + row)
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
    // rows 2 (m % 64) and 2 (m % 64) + 1 of X tile m / 64
    const uint64_t row = uint64_t(m / kXRows) * kPRows + 2u * (m % kXRows);
    uint4* dh = reinterpret_cast<uint4*>(pe + row * kp + uint64_t(t) * 16);
    uint4* dl = reinterpret_cast<uint4*>(pe + (row + 1) * kp + uint64_t(t) * 16);
    dh[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    dh[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
    dl[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    dl[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
  }
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

struct TcArgs {
  const uint32_t* codes;   // canonical images, E x (N x T/8 words)
  float* Y;                // (E, M, N)
  uint32_t M, m0, mc;      // rows of X/Y, this pass's first row and row count
  uint32_t xtiles;         // 64-row tiles of X in this pass
  uint32_t N, T, E;
  uint32_t* status;
  uint32_t vec;            // rows of Y start 16-byte aligned (N % 4 == 0): float4 stores
};

__global__ void __launch_bounds__(kTcThreads, 1) k_dense_tc(const __grid_constant__ CUtensorMap pmap, TcArgs a) {
  extern __shared__ unsigned char tc_smem[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem) + 1023) &
                                                         ~uintptr_t(1023));
  unsigned char* ring_a = base;
  unsigned char* ring_b = base + kStages * kAStage;
  // full[s]: stage s holds its chunk (the TMA bytes and every builder warp's
  // entries); empty[s]: the MMAs that read it are done (one commit)
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], full_d[2], free_d[2];
  __shared__ uint32_t tmem_base;
  const uint32_t tid = threadIdx.x, warp = tid / 32, lane = tid & 31;
  const uint32_t wtiles = (a.N + kWRows - 1) / kWRows;
  const uint64_t per_expert = uint64_t(wtiles) * a.xtiles;
  const uint64_t units = uint64_t(a.E) * per_expert;
  const uint32_t mine = units > blockIdx.x ? uint32_t((units - blockIdx.x + gridDim.x - 1) / gridDim.x) : 0u;
  const uint32_t CH = a.T / 4;  // K' chunks per item (4 groups each)
  // item u -> (expert, W tile, X tile); the X tiles of one W tile are adjacent
  auto item = [&](uint32_t it, uint64_t* e, uint32_t* wt, uint32_t* xt) {
    const uint64_t u = blockIdx.x + uint64_t(it) * gridDim.x;
    *e = u / per_expert;
    const uint64_t r = u % per_expert;
    *wt = uint32_t(r / a.xtiles);
    *xt = uint32_t(r % a.xtiles);
  };

  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(kCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mb_init(&full[s], 1 + kBuilderWarps);
      mb_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mb_init(&full_d[b], 1);
      mb_init(&free_d[b], 4);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  bool ok = true;

  if (warp == 0) {
    // producer: one TMA load of A (128 rows of P x 64 k') per chunk
    if (lane == 0) {
      uint64_t issued = 0;
      for (uint32_t it = 0; it < mine && ok; ++it) {
        uint64_t e;
        uint32_t wt, xt;
        item(it, &e, &wt, &xt);
        const int32_t row = int32_t((e * a.xtiles + xt) * kPRows);
        for (uint32_t c = 0; c < CH; ++c) {
          const uint64_t q = uint64_t(it) * CH + c;
          const uint32_t s = uint32_t(q % kStages);
          if (q >= uint64_t(kStages) && !(ok = mb_wait(&empty[s], uint32_t((q / kStages) - 1) & 1u))) break;
          mb_expect(&full[s], kAStage);
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
              "[%4];" ::"r"(smem_u32(ring_a + s * kAStage)),
              "l"(&pmap), "r"(int32_t(c * kChunk)), "r"(row), "r"(smem_u32(&full[s]))
              : "memory");
          ++issued;
        }
      }
      if (!ok) atomicOr(a.status, kStalled);
      // the loads in flight land before the block may exit (after a stall,
      // a stage whose builders gave up is waited out to the bound)
      for (uint64_t q = issued > uint64_t(kStages) ? issued - kStages : 0; q < issued; ++q)
        if (!mb_wait(&full[q % kStages], uint32_t(q / kStages) & 1u)) atomicOr(a.status, kStalled);
    }
  } else if (warp == 1) {
    // MMA issuer
    if (lane == 0) {
      uint64_t committed = 0;
      for (uint32_t it = 0; it < mine && ok; ++it) {
        const uint32_t db = it & 1u;
        if (it >= 2u && !(ok = mb_wait(&free_d[db], ((it / 2) - 1) & 1u))) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + db * uint32_t(kWRows);
        for (uint32_t c = 0; c < CH; ++c) {
          const uint64_t q = uint64_t(it) * CH + c;
          const uint32_t st = uint32_t(q % kStages);
          if (!(ok = mb_wait(&full[st], uint32_t(q / kStages) & 1u))) break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t aa = smem_u32(ring_a + st * kAStage), ba = smem_u32(ring_b + st * kBStage);
#pragma unroll
          for (uint32_t i = 0; i < 4; ++i)
            asm volatile(
                "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::
                    "r"(d), "l"(tc::Swz<32>::desc(aa + 32u * i)), "l"(tc::Swz<32>::desc(ba + 32u * i)),
                "r"(kIdesc), "r"(uint32_t(c | i))
                : "memory");
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                           smem_u32(&empty[st]))
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
      // issued only after its stage's previous phase completed, so empty's
      // parity names the last commit's phase unambiguously
      if (committed) {
        const uint64_t q = committed - 1;
        if (!mb_wait(&empty[q % kStages], uint32_t(q / kStages) & 1u)) atomicOr(a.status, kStalled);
      }
    }
  } else if (warp >= 4 && warp < 4 + kBuilderWarps) {
    // one-hot builders: thread r owns W row r of the item. A row's codes
    // arrive 128 bytes (8 uint4, 64 chunks) at a time, all eight loads in
    // flight at once, the next segment's line prefetched into L1.
    //
    // The B stages start zeroed, and a stage's row differs from what it held
    // kStages chunks earlier in at most 8 bf16 entries: per chunk the thread
    // clears the 4 entries it set there last time and sets the 4 new ones.
    // Every 128-bit code word is 8 chunks, so q % kStages = cc % kStages below.
    static_assert(8 % kStages == 0, "the chunk loop's stage index is cc % kStages");
    const uint32_t r = tid - 128;
    const uint64_t expert_words = uint64_t(a.N) * (a.T / 8);
    const uint32_t nu = a.T / 32;  // uint4 of codes per row
    auto row_src = [&](uint32_t it2, bool* valid) {
      uint64_t e;
      uint32_t wt, xt;
      item(it2, &e, &wt, &xt);
      const uint32_t n = wt * kWRows + r;
      *valid = n < a.N;
      return reinterpret_cast<const uint4*>(a.codes + e * expert_words + uint64_t(*valid ? n : 0) * (a.T / 8));
    };
    // this thread's row in a B stage: 16-byte unit j at r * 128 + ((j ^ (r & 7)) << 4);
    // entry e of group g (of the chunk's 4) is bf16 element 16 g + e, in unit 2 g + e / 8
    const uint32_t row_off = r * 128u, sw = r & 7u;
    auto entry = [&](uint32_t g, uint32_t e) {
      return row_off + (((2u * g + (e >> 3)) ^ sw) << 4) + ((e & 7u) << 1);
    };
#pragma unroll
    for (uint32_t s = 0; s < uint32_t(kStages); ++s)
#pragma unroll
      for (uint32_t j = 0; j < 8; ++j)
        *reinterpret_cast<uint4*>(ring_b + s * kBStage + row_off + j * 16u) = make_uint4(0, 0, 0, 0);
    // the entries set in each stage (offsets within the stage, < 32 KB: two per word)
    uint32_t prev[kStages][2];
#pragma unroll
    for (uint32_t s = 0; s < uint32_t(kStages); ++s)
#pragma unroll
      for (uint32_t h = 0; h < 2; ++h) prev[s][h] = entry(2 * h, 0) | (entry(2 * h + 1, 0) << 16);
    uint64_t q = 0;
    for (uint32_t it = 0; it < mine && ok; ++it) {
      bool valid;
      const uint4* src = row_src(it, &valid);
      for (uint32_t seg = 0; seg < nu && ok; seg += 8) {
        uint4 sv[8];
#pragma unroll
        for (uint32_t i = 0; i < 8; ++i)
          sv[i] = (valid && seg + i < nu) ? __ldg(src + seg + i) : make_uint4(0, 0, 0, 0);
        {
          bool nvalid = valid;
          const uint4* nsrc = seg + 8 < nu ? src + seg + 8 : (it + 1 < mine ? row_src(it + 1, &nvalid) : nullptr);
          if (nsrc && nvalid) asm volatile("prefetch.global.L1 [%0];" ::"l"(nsrc));
        }
#pragma unroll
        for (uint32_t i = 0; i < 8; ++i) {
          if (seg + i >= nu || !ok) break;
          const uint4 cur = sv[i];
#pragma unroll
          for (uint32_t cc = 0; cc < 8; ++cc) {
            const uint32_t word = cc < 4 ? (cc < 2 ? cur.x : cur.y) : (cc < 6 ? cur.z : cur.w);
            const uint32_t bits16 = word >> (16u * (cc & 1u));
            const uint32_t sb = cc % uint32_t(kStages);
            if (q >= uint64_t(kStages)) {
              const uint32_t got = lane == 0 ? uint32_t(mb_wait(&empty[sb], uint32_t((q / kStages) - 1) & 1u)) : 0u;
              if (!(ok = __shfl_sync(0xffffffffu, got, 0) != 0u)) break;
            }
            unsigned char* stage = ring_b + sb * kBStage;
#pragma unroll
            for (uint32_t h = 0; h < 2; ++h) {
              const uint32_t a0 = entry(2 * h, (bits16 >> (8u * h)) & 15u);
              const uint32_t a1 = entry(2 * h + 1, (bits16 >> (8u * h + 4u)) & 15u);
              *reinterpret_cast<uint16_t*>(stage + (prev[sb][h] & 0xFFFFu)) = 0;
              *reinterpret_cast<uint16_t*>(stage + (prev[sb][h] >> 16)) = 0;
              *reinterpret_cast<uint16_t*>(stage + a0) = 0x3F80u;  // bf16 1.0
              *reinterpret_cast<uint16_t*>(stage + a1) = 0x3F80u;
              prev[sb][h] = a0 | (a1 << 16);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor core
            __syncwarp();
            if (lane == 0) mb_arrive(&full[sb]);
            ++q;
          }
        }
      }
    }
    if (!ok) atomicOr(a.status, kStalled);
  } else if (warp >= 4 + kBuilderWarps) {
    // epilogue: thread p reads TMEM lane p (P row p: X row p / 2, hi or lo),
    // adds its pair partner's value, and even lanes store Y rows
    const uint32_t lane_base = (warp & 3u) * 32u, p = lane_base + lane;
    uint32_t bits = 0;
    for (uint32_t it = 0; it < mine && ok; ++it) {
      const uint32_t db = it & 1u;
      const uint32_t got = lane == 0 ? uint32_t(mb_wait(&full_d[db], (it / 2) & 1u)) : 0u;
      if (!(ok = __shfl_sync(0xffffffffu, got, 0) != 0u)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      uint64_t e;
      uint32_t wt, xt;
      item(it, &e, &wt, &xt);
      const uint32_t m = xt * kXRows + p / 2;   // row within this pass
      const bool store = (p & 1u) == 0 && m < a.mc;
      float* yrow = a.Y + (e * a.M + a.m0 + m) * a.N + wt * kWRows;
      const uint32_t nvalid = min(uint32_t(kWRows), a.N - wt * kWRows);
      for (uint32_t cb = 0; cb < uint32_t(kWRows); cb += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + (lane_base << 16) + db * uint32_t(kWRows) + cb, v);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        float y[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float own = __uint_as_float(v[j]);
          y[j] = own + __shfl_xor_sync(0xffffffffu, own, 1);   // hi + lo
        }
        if (store && cb < nvalid) {
          if (a.vec && cb + 32 <= nvalid) {
            float4* dst = reinterpret_cast<float4*>(yrow + cb);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              dst[j] = make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
              bits |= (finite32(y[4 * j]) && finite32(y[4 * j + 1]) && finite32(y[4 * j + 2]) &&
                       finite32(y[4 * j + 3])) ? 0u : kNonfinite;
            }
          } else {
#pragma unroll
            for (uint32_t j = 0; j < 32; ++j)
              if (cb + j < nvalid) {
                yrow[cb + j] = y[j];
                bits |= finite32(y[j]) ? 0u : kNonfinite;
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
  if (warp == 2) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
}

// The tensor map of the P workspace: rows of K' bf16, boxes of 128 rows x
// 64 elements (128 bytes), 128-byte swizzle (the UMMA K-major layout).
bool p_tensor_map(const void* ws, uint64_t kp, uint64_t rows, CUtensorMap* map) {
  const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return false;
  const cuuint64_t dims[2] = {cuuint64_t(kp), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(kp) * 2};
  const cuuint32_t box[2] = {cuuint32_t(kChunk), cuuint32_t(kPRows)};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ws), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int G>
cudaError_t dense_tc_group(const float* X, const uint32_t* codes, const float* books, float* Y, uint32_t M,
                           uint32_t N, uint32_t K, uint32_t E, void* ws, uint32_t* status, cudaStream_t s) {
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(k_dense_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kTcSmem));
  });
  if (attr != cudaSuccess) return attr;
  const uint32_t T = K / G;
  const uint64_t kp = uint64_t(16) * T;
  for (uint32_t m0 = 0; m0 < M; m0 += kDenseTcMaxRows) {
    const uint32_t mc = std::min<uint32_t>(kDenseTcMaxRows, M - m0);
    const uint32_t xtiles = (mc + kXRows - 1) / kXRows;
    const uint64_t items = uint64_t(xtiles) * kXRows * T;
    const dim3 pgrid(uint32_t(std::min<uint64_t>((items + 255) / 256, 1024)), E);
    k_dense_tc_prep<G><<<pgrid, 256, 0, s>>>(X, books, static_cast<__nv_bfloat16*>(ws), M, m0, mc, xtiles, K,
                                              status);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    CUtensorMap map;
    if (!p_tensor_map(ws, kp, uint64_t(E) * xtiles * kPRows, &map)) return cudaErrorInvalidValue;
    TcArgs a{codes, Y, M, m0, mc, xtiles, N, T, E, status, N % 4 == 0 ? 1u : 0u};
    const uint64_t units = uint64_t(E) * ((N + kWRows - 1) / kWRows) * xtiles;
    const uint32_t grid = uint32_t(std::min<uint64_t>(units, uint64_t(sm_count())));
    k_dense_tc<<<grid, kTcThreads, kTcSmem, s>>>(map, a);
    err = cudaGetLastError();
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
  if (!aligned16(X) || !aligned16(codes) || !aligned16(ws) || !aligned16(Y))
    return cudaErrorMisalignedAddress;  // 16-byte loads of X and codes, 16-byte stores of Y rows
  const uint32_t M = uint32_t(p.m), N = uint32_t(p.n), K = uint32_t(p.k);
  switch (p.group) {
    case 8: return dense_tc_group<8>(X, codes, books, Y, M, N, K, p.batch, ws, status, s);
    case 16: return dense_tc_group<16>(X, codes, books, Y, M, N, K, p.batch, ws, status, s);
    default: return dense_tc_group<32>(X, codes, books, Y, M, N, K, p.batch, ws, status, s);
  }
}

}  // namespace ack
