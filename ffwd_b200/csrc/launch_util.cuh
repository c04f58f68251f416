// Host helpers for kernel launches.
#pragma once

#include <atomic>
#include <cstdint>
#include <cuda_runtime.h>

namespace fb {

// Raise a kernel's dynamic shared-memory limit once per device (the attribute
// call costs far more than a launch, so it stays off the per-launch path).
// One flag word per kernel (the kernel itself is the template argument).
template <auto Kern>
cudaError_t set_smem_once(int bytes) {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

}  // namespace fb
