// Completion signal of a producer grid to every rank of a symmetric-memory
// group (used by the fused collective kernels and the MoE combine).
#pragma once
#include "common/host.h"
#include "common/sm100.cuh"

namespace bwn {

// Each CTA (one thread, after a CTA barrier) orders its stores before a ticket;
// the last CTA publishes the new epoch to every rank's flag array (one system
// fence, then relaxed stores).
__device__ __forceinline__ void signal_done(const CommSignal& sig) {
  __threadfence();
  const int t = atomicAdd(sig.done_ticket, 1);
  if (t == (int)gridDim.x - 1) {
    *sig.done_ticket = 0;
    fence_acq_rel_sys();
    const unsigned e = (unsigned)(*sig.epoch) + 1u;
    *sig.epoch = (int)e;
    for (int r = 0; r < sig.world; ++r) st_relaxed_sys_u32(sig.peer_flags[r] + sig.rank, e);
  }
}

}  // namespace bwn
