// Work-unit scheduling shared by the grouped expert GEMMs (bf16 in
// csrc/kernels/moe.cu, fp8 weights in csrc/kernels/moe_w8.cu).
#pragma once
#include "kernels/moe.h"

namespace bwn {

constexpr int kGMaxGroups = kMoeDecodeMaxGroups;  // local experts + a shared-expert group

// Work units are compacted over the groups' actual row counts (cached in
// shared memory at kernel start): unit u -> group e by binary search over the
// per-group unit prefix, so empty groups and empty row tiles cost nothing.
struct GUnits {
  int pref[kGMaxGroups + 1];  // units before group e
  int cnt[kGMaxGroups];
  int off[kGMaxGroups];
};

__device__ __forceinline__ bool gunit(const GroupedArgs& a, const GUnits& g, int u, int& e, int& tm, int& tn, int& n0,
                                      int& nrows, int BN) {
  int lo = 0, hi = a.groups;  // largest e with pref[e] <= u
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (g.pref[mid] <= u) lo = mid; else hi = mid;
  }
  e = lo;
  const int rem = u - g.pref[e];
  tm = rem % a.tiles_m;
  tn = rem / a.tiles_m;
  const int cnt = g.cnt[e];
  n0 = g.off[e] + tn * BN;
  nrows = min(BN, cnt - tn * BN);
  return nrows > 0;
}

// Fill the unit table from the device row counts: every thread of the block
// calls it; the caller synchronizes before reading ``pref``.
__device__ __forceinline__ void gunits_fill(const GroupedArgs& a, GUnits& gu, int BN) {
  for (int e = threadIdx.x; e < a.groups; e += blockDim.x) {
    const int c = min(a.counts[e], a.max_tiles_n * BN);
    gu.cnt[e] = c;
    gu.off[e] = a.offsets[e];
    gu.pref[e + 1] = a.tiles_m * ((c + BN - 1) / BN);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    gu.pref[0] = 0;
    for (int e = 0; e < a.groups; ++e) gu.pref[e + 1] += gu.pref[e];
  }
}

}  // namespace bwn
