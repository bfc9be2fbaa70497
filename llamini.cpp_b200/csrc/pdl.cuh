// pdl.cuh -- Programmatic Dependent Launch between the kernels of a step.
//
// Every kernel of the token loop is launched with programmatic stream
// serialisation: it may start while its predecessor is still running, issues
// the loads that do not depend on the predecessor (weights, older KV-cache
// entries), and only then waits for the predecessor's results. Each kernel
// waits (pdl_wait) before it touches anything a predecessor writes and before
// it exits, so completion stays ordered along the chain. Before the wait a
// kernel only reads data that no kernel of the chain writes.
#pragma once

#include <cuda_runtime.h>
#include <utility>

namespace lm {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" :::); }

bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace lm
