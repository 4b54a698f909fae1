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

}  // namespace ack
