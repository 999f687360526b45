// Programmatic dependent launch for the small kernels of a decode step.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace nb200 {

// kernel<<<grid, block, smem, st>>>(args...) that may begin while the previous
// kernel in the stream drains (programmatic stream serialisation).  Every
// kernel launched this way executes griddepcontrol.wait before it reads or
// writes memory that earlier kernels use, and then griddepcontrol
// .launch_dependents so that its own successor can be scheduled.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args &&...args) {
    cudaLaunchConfig_t cfg{};
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

// The kernel side: wait for the previous grid, then release the next one.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace nb200
