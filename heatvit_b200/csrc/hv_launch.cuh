// hv_launch.cuh — kernel launches with programmatic dependent launch (PDL).
//
// Kernels of the inference pipeline are launched with
// cudaLaunchAttributeProgrammaticStreamSerialization.  Each of them executes
// griddep_wait() before its first access to memory that an earlier kernel of
// the stream writes or reads, and griddep_launch() right after it.  The next
// kernel's CTAs may then be scheduled on SMs that the current kernel's tail
// frees, run their prologue (weights into shared memory, TMEM allocation,
// barrier set-up), and block in their own griddep_wait() until this grid has
// completed and its writes are visible.
#pragma once
#include <cuda_runtime.h>
#include <utility>

namespace hv {

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace hv
