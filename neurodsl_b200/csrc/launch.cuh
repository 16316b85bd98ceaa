// launch.cuh — kernel launches with cluster and programmatic-dependent-launch
// attributes, and the device side of programmatic dependent launch (PDL).
//
// PDL lets a kernel's CTAs start while the previous kernel of the stream is
// still running.  A PDL-capable kernel here follows one rule:
//   1. before pdl_wait() it reads only operands that no unfinished kernel can
//      be writing — the constant ones (weights, LayerNorm parameters, and in
//      decode attention the cached keys/values below the appended position);
//      it writes nothing;
//   2. pdl_wait() returns once the previous kernel has finished and its memory
//      is visible; only then does it read activations and write outputs;
//   3. it calls pdl_trigger() after pdl_wait(), so at most one kernel runs
//      ahead of the one that is working: every kernel before that one has
//      finished.
// Launched without the attribute both instructions are no-ops, so the same
// kernels serve both modes.  The mode is per host thread (set_pdl_enabled),
// off by default; callers turn it on where the rule's constant operands
// really are constant, e.g. the decode steps of a model whose weights and
// earlier cache entries no kernel of the step writes.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace nd {

bool pdl_enabled();
void set_pdl_enabled(bool on);

// Upper bound on the SMs a persistent kernel (the large-M GEMM, prefill
// attention) occupies, for launches from the calling host thread; 0 = all.
// Leaves SMs free for kernels on other streams, e.g. a collective that
// overlaps the compute.
int sm_limit();
void set_sm_limit(int n);
// The current device's SM count (cached per device).
int current_sm_count();
// The device's SM count under the calling thread's limit.
inline int limited_sms(int sms) {
  const int lim = sm_limit();
  return lim > 0 && lim < sms ? lim : sms;
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launch `kernel` with an optional 1-D cluster of `cluster_x` CTAs along x
// (gridDim.x must be a multiple of it) and, when `pdl_capable` and the mode is
// on, the programmatic stream serialization attribute.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t stream, int cluster_x, bool pdl_capable, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(cluster_x);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl_capable && pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = n ? attr : nullptr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace nd
