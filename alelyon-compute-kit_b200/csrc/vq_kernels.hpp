// Launcher of the vq4 kernels: one admitted plan, its operand device
// pointers (slot order of the plan's schema), the stream to enqueue on.
#pragma once

#include <cuda_runtime.h>

#include "vq_plan.hpp"

namespace ack {

// Enqueue the plan's kernels on `stream` (the current device). The plan must
// have passed admission; pointers are device addresses in slot order.
cudaError_t launch(const Plan& plan, void* const* ptr, cudaStream_t stream);

// Books one ack_vq_encode_noalloc call may encode with (its static scratch).
constexpr uint32_t kStaticEncodeBooks = 64;

// Encode `batch` tensors of `n` values (x: batch x n floats, books: batch x
// 16 x group, codes: batch x words(n) u32) using only the library's static
// scratch; the caller has validated the arguments.
cudaError_t encode_noalloc(const float* x, uint64_t n, uint32_t batch, const float* books, uint32_t group,
                           uint32_t* codes, uint32_t* status, cudaStream_t stream);

// Test only (ack_inject_fault kind 2): arm a stall test for the next
// tensor-core encode launch in this process (1: its producer issues no load;
// 2: its consumers take no accumulator). Defined in vq_codec.cu.
void set_encode_stall_test(uint32_t mode);

// ---- NF4 comparator (vq_nf4.cu): nf4-decode/v1 and nf4-gemv/v1 ----
// The stored source: packed indices (two a byte, the first value in the high
// nibble), one absmax index byte a block of 64 values, one FP32 absmax2 a
// nested block of 256 blocks, the 16 code values then the 256 map values,
// int64 member starts (read as their low words) and one FP32 offset a member.
struct Nf4Source {
  const uint32_t* packed;
  const uint32_t* absmax_q;
  const float* absmax2;
  const float* tables;
  const uint32_t* starts;
  const float* offsets;
  uint32_t members, src_base, src_limit;
};
struct Nf4Gemv {
  const uint4* A;          // rows x lda 16-bit words, read 8 at a time
  float* C;                // rows x n
  const uint32_t* table;   // groups x (first row, rows, weight base)
  uint32_t n, k, lda, rows, groups;
  Nf4Source src;
};
cudaError_t nf4_decode(const Nf4Source& src, const uint32_t* ids, void* out, uint32_t n, uint32_t selected,
                       uint32_t member_values, uint32_t storage, cudaStream_t stream);
cudaError_t nf4_gemv(const Nf4Gemv& g, uint32_t max_rows, uint32_t elem, cudaStream_t stream);

// ---- Y shards written straight into peers' memory (vq_products.cu, vq_peer.cu) ----
// Up to 7 other ranks' output slots (CUDA IPC mappings over NVLink); the
// product writes each output to its own Y and to every peer slot at the same
// offset, then fences at system scope before its blocks exit.
constexpr uint32_t kMaxPeers = 7;
struct PeerY {
  float* dst[kMaxPeers];
  uint32_t n;
};
// The byte-pair GEMV (op 16, M = 1, W stored N x K, canonical) with peer
// stores; cudaErrorNotSupported for a plan the byte-pair kernel does not take.
cudaError_t dense_peers(const Plan& p, void* const* ptr, const PeerY& peers, cudaStream_t stream);
// Publish `epoch` into slot `rank` of every rank's flag array (release, system
// scope), after the stream's earlier work.
cudaError_t peer_signal(uint32_t* const* flags, uint32_t world, uint32_t rank, uint32_t epoch, cudaStream_t stream);
// Wait (bounded: `polls` polls a flag) until every rank's flag here has
// reached `epoch`; a wait that runs out sets the stalled status bit.
cudaError_t peer_wait(const uint32_t* flags, uint32_t world, uint32_t epoch, uint32_t* status, uint32_t polls,
                      cudaStream_t stream);

}  // namespace ack
