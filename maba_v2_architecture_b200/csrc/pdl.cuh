// Programmatic dependent launch for the decode chain.
//
// A kernel launched with launch_pdl() may start once every CTA of the previous
// kernel on the stream has started (griddep_launch_dependents() at the top of a
// kernel lets its successor start that early).  It must call griddep_wait()
// before it reads anything an earlier kernel wrote (or writes anything an
// earlier kernel reads); what it does before the wait -- weight loads, index
// arithmetic -- overlaps the predecessor's tail.  Both instructions are no-ops
// in a kernel launched without the attribute.
#pragma once
#include "common.cuh"

namespace maba {

__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
    if (e != cudaSuccess)
        return set_error(MABA_ERR_CUDA, "launch: %s (%s)", cudaGetErrorName(e), cudaGetErrorString(e));
    return MABA_OK;
}

}  // namespace maba
