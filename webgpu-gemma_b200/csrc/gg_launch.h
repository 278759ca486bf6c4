// gg_launch.h -- kernel launches with programmatic dependent launch (PDL).
//
// The batched paths (prefill chunks, batched decode, gg_linear) are chains of short kernels on
// one stream. Launched with programmatic stream serialization, a kernel may become resident
// while its predecessor finishes: it runs what does not depend on earlier kernels (barrier
// set-up, TMEM allocation, streaming its weights into registers) and then waits in pdl_wait()
// (griddepcontrol.wait) until the predecessor has completed and its writes are visible. Every
// kernel launched this way calls pdl_wait() before it reads or writes any buffer another kernel
// of the chain touches.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace gg {

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = at;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, kernel, std::forward<Args>(args)...);
}

}  // namespace gg
