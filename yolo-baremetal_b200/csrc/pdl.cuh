// Programmatic dependent launch: every kernel of a forward plan is launched
// with programmatic stream serialisation, so it may start (prologue: shared
// memory, barriers, tensor memory, constant weights) while its predecessor in
// the stream is still finishing.  pdl_wait() blocks until the predecessor
// grid has completed and its writes are visible; every kernel calls it before
// its first access to activation memory (reads, and writes that a
// predecessor might still read).  Persistent kernels, whose CTAs are all
// resident, call pdl_trigger() at their start so that their successor can
// launch into the SMs they leave free; a dependent only launches once every
// CTA of its predecessor has triggered or exited, so it never takes resources
// a not-yet-started predecessor CTA needs.  Without the launch attribute
// (or after a non-kernel predecessor) both instructions are no-ops.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <utility>

namespace yb {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
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
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Raises a kernel's dynamic shared memory limit to `bytes` on the current
// device, once per device (`done` holds one bit per device ordinal), so that
// one process driving several GPUs sets it on each of them.
template <typename... KArgs>
cudaError_t smem_attr_once(void (*kernel)(KArgs...), int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit && (done.load() & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit);
  return e;
}

}  // namespace yb
