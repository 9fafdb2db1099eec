// Kernel launch with programmatic dependent launch (PDL) allowed.  A kernel
// launched this way may start while the previous kernel in the stream is still
// running; it must execute griddepcontrol.wait (bwn::pdl_wait) before touching
// anything the previous kernel writes.  Every bwn kernel triggers its own
// dependents at entry (bwn::pdl_trigger), which takes effect once all of its
// CTAs have started, so an early dependent never starves it of SMs.
// Set BWN_PDL=0 to launch normally (A/B measurement).
#pragma once
#include <cuda_runtime.h>

#include <cstdlib>
#include <utility>

#include "common/host.h"

namespace bwn {

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("BWN_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  BWN_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

}  // namespace bwn
