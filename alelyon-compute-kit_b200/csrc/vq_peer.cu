// Step flags between ranks whose products write straight into each other's
// memory (CUDA IPC mappings over NVLink; no multicast object is involved):
//
//   k_peer_signal  after the stream's product: a system-scope fence, then a
//                  release store of the step's epoch into this rank's slot of
//                  every rank's flag array
//   k_peer_wait    one thread per sender: acquire loads of this rank's flags
//                  until each has reached the epoch, bounded (the poll count
//                  is the caller's, each poll backs off ~100 ns); a wait that
//                  runs out sets the stalled status bit and returns
//
// Epochs only grow, so a flag that has moved past the epoch (a sender already
// a step ahead) also completes the wait.
#include <cuda_runtime.h>

#include <cstdint>

#include "vq_common.cuh"
#include "vq_kernels.hpp"

namespace ack {
namespace {

struct FlagPtrs {
  uint32_t* p[kMaxPeers + 1];
};

__global__ void k_peer_signal(FlagPtrs f, uint32_t world, uint32_t rank, uint32_t epoch) {
  __threadfence_system();
  const uint32_t i = threadIdx.x;
  if (i < world) asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f.p[i] + rank), "r"(epoch) : "memory");
}

__global__ void k_peer_wait(const uint32_t* __restrict__ flags, uint32_t world, uint32_t epoch,
                            uint32_t* __restrict__ status, uint32_t polls) {
  const uint32_t i = threadIdx.x;
  if (i >= world) return;
  for (uint32_t it = 0; it < polls; ++it) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + i) : "memory");
    if (int32_t(v - epoch) >= 0) return;
    __nanosleep(100);
  }
  atomicOr(status, kStalled);
}

}  // namespace

cudaError_t peer_signal(uint32_t* const* flags, uint32_t world, uint32_t rank, uint32_t epoch, cudaStream_t s) {
  if (world == 0 || world > kMaxPeers + 1 || rank >= world) return cudaErrorInvalidValue;
  FlagPtrs f{};
  for (uint32_t i = 0; i < world; ++i) f.p[i] = flags[i];
  k_peer_signal<<<1, 32, 0, s>>>(f, world, rank, epoch);
  return cudaGetLastError();
}

cudaError_t peer_wait(const uint32_t* flags, uint32_t world, uint32_t epoch, uint32_t* status, uint32_t polls,
                      cudaStream_t s) {
  if (world == 0 || world > kMaxPeers + 1) return cudaErrorInvalidValue;
  k_peer_wait<<<1, 32, 0, s>>>(flags, world, epoch, status, polls);
  return cudaGetLastError();
}

}  // namespace ack
