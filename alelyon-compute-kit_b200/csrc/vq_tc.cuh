// tcgen05 / TMA / mbarrier primitives for sm_100a kernels (inline PTX):
// shared-memory addresses, tf32 rounding, the UMMA K-major swizzle and
// shared-memory matrix descriptors, instruction descriptors, and mbarrier
// operations whose waits are bounded.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ack {
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
// 16 consecutive TMEM columns of this warp's 32 lanes into r[0..15]
// (tcgen05.ld 32x32b.x16; the values are valid after tcgen05.wait::ld).
__device__ __forceinline__ void tmem_ld16(uint32_t* r, uint32_t taddr) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

constexpr uint32_t kPolls = 1u << 22;       // the normal bound of a wait
constexpr uint32_t kTestPolls = 1u << 10;   // pipeline waits under a host-injected stall test

// Wait for the phase of parity `parity` to complete; false after `polls`
// polls (each suspends for a hardware-chosen interval), never an endless
// spin. A non-suspending probe first: a phase that completed earlier (the
// common case for a stage filled ahead) returns without entering the
// suspend path.
__device__ __forceinline__ bool mb_wait(uint64_t* b, uint32_t parity, uint32_t polls = kPolls) {
  uint32_t done;
  asm volatile("{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(done)
               : "r"(smem_u32(b)), "r"(parity)
               : "memory");
  if (done) return true;
  for (uint32_t it = 0; it < polls; ++it) {
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

}  // namespace tc
}  // namespace ack
