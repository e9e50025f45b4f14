// Kernel launches with programmatic dependent launch (PDL).
//
// Every kernel of this library is launched with cudaLaunchAttributeProgrammaticStreamSerialization, so the next
// kernel on a stream (or the next node of a captured CUDA graph) is scheduled while the previous one drains: its CTAs
// take SMs as the previous grid's CTAs leave and run their prologue (barrier init, tensor-map prefetch) before the
// previous grid has finished. The rule that keeps this exact: every kernel executes grid_dep_wait() -- which returns
// once all prerequisite grids have completed and their memory is visible -- before its first access to global memory
// and before it allocates tensor memory (a CTA that waits holds no TMEM, so no chain of launches can deadlock on TMEM).
// griddepcontrol.wait is a no-op in a grid launched without the attribute, so a kernel behaves the same either way.
// grid_dep_launch() lets the next grid start launching once every CTA of this one has executed it (or exited); where
// it is placed affects only overlap, never results. MKB_PDL=0 in the environment launches without the attribute.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <utility>

namespace mkb {

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Whether launches carry the PDL attribute (read once from MKB_PDL; default on).
bool pdl_enabled();

// kernel<<<grid, block, smem, st>>>(args...) with the PDL attribute when enabled. The arguments are converted to the
// kernel's parameter types as in a <<<>>> launch.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same launch as clusters of two CTAs along x (a kernel written for CTA pairs without __cluster_dims__).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k_pairs(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                  Args&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Raises a kernel's dynamic shared-memory limit to `bytes` on the current device. cudaFuncSetAttribute acts on the
// calling thread's current device only, so a launch site keeps one bit per device in `done` (devices 0..63) and a
// process that launches on several devices sets the limit on each of them; threads that race both set it, which is
// harmless. Devices beyond 63 set it on every call.
template <typename... KArgs>
inline cudaError_t smem_limit_once(std::atomic<uint64_t>& done, void (*kernel)(KArgs...), int bytes)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return e;
    const uint64_t bit = dev >= 0 && dev < 64 ? uint64_t(1) << dev : 0;
    if (bit && (done.load(std::memory_order_acquire) & bit))
        return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && bit)
        done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

}  // namespace mkb
