// Launcher of the vq4 kernels: one admitted plan, its operand device
// pointers (slot order of the plan's schema), the stream to enqueue on.
#pragma once

#include <cuda_runtime.h>

#include "vq_plan.hpp"

namespace ack {

// Enqueue the plan's kernels on `stream` (the current device). The plan must
// have passed admission; pointers are device addresses in slot order.
cudaError_t launch(const Plan& plan, void* const* ptr, cudaStream_t stream);

}  // namespace ack
