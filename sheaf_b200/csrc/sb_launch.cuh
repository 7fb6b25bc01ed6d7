// Programmatic dependent launch (PDL) for the kernels of a step.
//
// A kernel launched with `launch_pdl` may be scheduled while the kernel
// before it on the stream is still running: its launch and prologue overlap
// that kernel's tail. Every kernel launched this way calls `pdl_wait()`
// before its first global-memory access, read or write, and before it can
// return; the wait ends when the preceding kernel has completed and its
// writes are visible (it is a no-op for an ordinary launch). Because each
// kernel waits for its predecessor before finishing, completion of the
// predecessor implies completion of everything before it.
//
// `pdl_trigger()` lets the next kernel be scheduled. Kernels that allocate
// tensor memory trigger only after their allocation and allocate only after
// their wait, so a successor resident on the same SM can never hold columns
// a predecessor still has to allocate.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace sb {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Kernel families that may launch programmatically: bit 0 GEMMs, 1 row-wise
// kernels, 2 attention, 3 optimizer and sampling. The default mask is 5
// (GEMMs and attention): those kernels fit at most one or two CTAs per SM,
// so an early launch cannot crowd their CTAs onto the SMs that happen to be
// free first. The row-wise and optimizer kernels split their rows statically
// over the blocks; placed early onto a partly busy GPU, several blocks land
// on one SM and the kernel measured slower (nanoGPT step: 2.62 ms with mask
// 5, 2.76 ms with every family). SHEAF_B200_PDL overrides the mask.
int pdl_mask();
#ifndef SB_PDL_FAMILY
#define SB_PDL_FAMILY 0
#endif

// Launches `k` on `s` with programmatic stream serialisation allowed.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (pdl_mask() >> SB_PDL_FAMILY) & 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

}  // namespace sb
