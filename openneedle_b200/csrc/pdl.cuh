// Programmatic dependent launch for the small kernels of a decode step.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace nb200 {

// kernel<<<grid, block, smem, st>>>(args...) that may begin while the previous
// kernel in the stream drains (programmatic stream serialisation).  Every
// kernel launched this way executes griddepcontrol.wait before it reads or
// writes memory that earlier kernels use.  The kernels do not trigger their
// successors early (griddepcontrol.launch_dependents): on the decode step a
// successor released at the start of its predecessor occupies SM slots while
// it waits and was measured slower (2.34 ms per config-5 step) than leaving
// the release to the predecessor's exit (2.21 ms) or not using programmatic
// launches at all (2.25 ms).
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

// The kernel side: wait until the previous grid has finished and its memory
// operations are visible.
__device__ __forceinline__ void pdl_enter() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

}  // namespace nb200
