// launch_util.cuh -- per-device kernel set-up shared by the launch units.
//
// The dynamic shared-memory opt-in (cudaFuncAttributeMaxDynamicSharedMemorySize)
// is a per-device attribute of a kernel, and a persistent kernel's grid is its
// occupancy times the device's SM count; both are established on the first
// launch on each device and cached per (kernel, device).  The shared-memory
// carveout is left to the driver: forcing the maximum shrinks L1, which holds
// the in-flight global loads these streaming kernels depend on (measured
// 11% slower for FWHT rows of 1024-4096 on B200).
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <utility>

namespace cubf {

constexpr int kMaxDevices = 64;

struct KernelSetup {
    std::atomic<int> grid_cap[kMaxDevices];  // 0: not set up on that device yet
};

// `setup` must have static storage duration (zero-initialised).  On success
// *grid_cap = resident CTAs per SM x SMs of the current device.  A kernel
// whose residency is set by its shared memory (tensor-core tiles) passes
// `max_carveout` to ask for the largest shared-memory carveout; without it the
// occupancy the driver grants such a kernel can be a single CTA per SM.
template <typename Kernel>
cudaError_t setup_kernel(KernelSetup& setup, Kernel kernel, int threads, int smem_bytes, int* grid_cap,
                         bool max_carveout = false) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    int cap = setup.grid_cap[dev].load(std::memory_order_acquire);
    if (cap == 0) {
        if (smem_bytes > 48 * 1024) {
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
            if (e != cudaSuccess) return e;
        }
        if (max_carveout) {
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     cudaSharedmemCarveoutMaxShared);
            if (e != cudaSuccess) return e;
        }
        int per_sm = 0, sms = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem_bytes);
        if (e != cudaSuccess) return e;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        if (per_sm <= 0) return cudaErrorInvalidConfiguration;
        cap = per_sm * sms;
        setup.grid_cap[dev].store(cap, std::memory_order_release);
    }
    *grid_cap = cap;
    return cudaSuccess;
}

// Launch as a programmatic dependent of the kernel before it on the stream
// (cudaLaunchAttributeProgrammaticStreamSerialization): the kernel's CTAs
// may be scheduled while that kernel finishes, and must call pdl_begin()
// (common.cuh) before touching global memory.  Between back-to-back kernels
// of this library -- the passes of one execution, and successive executions
// -- that hides the launch latency and the CTA ramp behind the previous
// kernel's tail.
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kernel)(KArgs...), unsigned grid, unsigned threads, std::size_t smem,
                             cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace cubf
