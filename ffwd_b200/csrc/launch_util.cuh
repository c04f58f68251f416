// Host helpers for kernel launches.
#pragma once

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <utility>
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

// Launch with programmatic stream serialization (the kernel must call
// griddep_wait before touching global data, see ptx.cuh), so the launch and
// set-up of kernel k + 1 overlap the tail of kernel k.  FFWD_B200_PDL=0 makes
// it a normal launch (A/B comparisons).
inline bool pdl_enabled() {
    static const bool on = [] {
        const char *e = getenv("FFWD_B200_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace fb
