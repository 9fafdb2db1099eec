// Expert-parallel MoE all-to-all over NVLink peer memory: dispatch of routed
// token rows to the ranks that own their experts, and return of the expert
// outputs to the ranks that own the tokens.  The reference does expert
// parallelism as masked-dense compute followed by an all-reduce
// (contrib/qwen3.6-35b-a3b/static_decode_35b.py:811-821, 1183); here the rows
// themselves move, written straight into the owner's receive buffer with
// peer stores, so each rank computes only the (token, expert) pairs it owns.
//
// Per MoE layer, on every rank (W ranks, E_l local experts each):
//   ep_count_kernel   count this rank's pairs per (destination, local expert),
//                     all-gather the count blocks into every rank's table
//                     (peer stores + flag A), wait for all blocks, derive the
//                     receive counts / offsets of the local experts
//   ep_send_kernel    each (token, slot) pair: a warp copies the token row into
//                     the owner's expert-major receive buffer at
//                     offset(dst, e) + an atomic slot, plus its (src, token,
//                     slot) tag; the last CTA publishes flag B
//   ep_wait_kernel    wait until every source has published (flag B or C)
//   (grouped tcgen05 GEMMs run on the receive buffer: gate/up+SwiGLU, down)
//   ep_return_kernel  each received row goes back to its source's combine
//                     buffer at [token][slot] (peer stores); flag C
//   (the source's moe_combine then takes the router-weighted sum of its slots)
// All waits are bounded (status bit on timeout).  Buffers are reused across
// layers without extra barriers: a rank can only write a peer's buffer for the
// next layer after that peer has passed the flag that follows its last read.
#include "comm/ep.h"
#include "common/host.h"
#include "common/launch.cuh"
#include "common/sm100.cuh"

namespace bwn {

namespace {

__device__ __forceinline__ bool wait_lane(const unsigned* flags, int world, unsigned epoch, int* status,
                                          uint64_t limit_ns) {
  const int r = threadIdx.x;
  if (r >= world) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while ((int)(ld_acquire_sys(flags + r) - epoch) < 0) {
    if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > limit_ns) {
      set_status(status, kStatusPeerTimeout);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void publish(const EpArgs& a, int flag_off, int* epoch) {
  fence_acq_rel_sys();
  const unsigned e = (unsigned)(*epoch) + 1u;
  *epoch = (int)e;
  for (int r = 0; r < a.world; ++r) st_relaxed_sys_u32(a.peer_flags[r] + flag_off + a.rank, e);
}

// last CTA of the grid publishes (after every CTA's stores)
__device__ __forceinline__ void grid_publish(const EpArgs& a, int* ticket, int flag_off, int* epoch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int t = atomicAdd(ticket, 1);
    if (t == (int)gridDim.x - 1) {
      *ticket = 0;
      publish(a, flag_off, epoch);
    }
  }
}

}  // namespace

__global__ void __launch_bounds__(256) ep_count_kernel(EpArgs a) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ int s_cnt[];  // [W * E_l]
  const int W = a.world, El = a.e_local, n = a.T * a.k;
  for (int i = threadIdx.x; i < W * El; i += blockDim.x) s_cnt[i] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < n; p += blockDim.x) {
    const int e = a.ids[p];
    if (e >= 0 && e < W * El) atomicAdd(&s_cnt[e], 1);  // global id = dst * E_l + local expert
  }
  __syncthreads();
  // all-gather: this rank's block [W][E_l] into table[rank] of every rank
  for (int r = 0; r < W; ++r) {
    int* dst = a.peer_table[r] + (long)a.rank * W * El;
    for (int i = threadIdx.x; i < W * El; i += blockDim.x)
      asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(dst + i), "r"(s_cnt[i]) : "memory");
  }
  for (int i = threadIdx.x; i < W * El; i += blockDim.x) a.send_ctr[i] = 0;  // slots for ep_send_kernel
  __syncthreads();
  if (threadIdx.x == 0) publish(a, kEpFlagA, a.epoch_a);
  __syncthreads();
  const bool ok = __syncthreads_and(wait_lane(a.flags + kEpFlagA, W, (unsigned)(*a.epoch_a), a.status, a.limit_ns));
  if (threadIdx.x == 0) a.ok[0] = ok ? 1 : 0;
  if (!ok) {  // a rank never published its counts: receive nothing, send nothing
    for (int e = threadIdx.x; e <= El; e += blockDim.x) {
      if (e < El) a.recv_counts[e] = 0;
      a.recv_offsets[e] = 0;
    }
    return;
  }
  // receive counts / offsets of this rank's experts (expert-major rows):
  // per-expert sums in parallel, then one scan out of shared memory
  int* s_rc = s_cnt;  // reuse: [E_l]
  for (int e = threadIdx.x; e < El; e += blockDim.x) {
    int c = 0;
    for (int s = 0; s < W; ++s) c += __ldcg(a.table + ((long)s * W + a.rank) * El + e);
    s_rc[e] = c;
    a.recv_counts[e] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < El; ++e) {
      a.recv_offsets[e] = acc;
      acc += s_rc[e];
    }
    a.recv_offsets[El] = acc;
  }
}

__global__ void __launch_bounds__(256) ep_send_kernel(EpArgs a) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ int s_off[];  // [W * E_l] base offset of this rank's rows in (dst, e); then [W * E_l] totals
  if (!a.ok[0]) return;  // the count exchange timed out: no peer stores
  const int W = a.world, El = a.e_local, H = a.H;
  int* s_tot = s_off + W * El;
  for (int i = threadIdx.x; i < W * El; i += blockDim.x) {
    const int dst = i / El, e = i % El;
    int tot = 0, mine = 0;
    for (int s = 0; s < W; ++s) {
      const int c = __ldcg(a.table + ((long)s * W + dst) * El + e);
      tot += c;
      if (s < a.rank) mine += c;
    }
    s_tot[i] = tot;
    s_off[i] = mine;
  }
  __syncthreads();
  if (threadIdx.x < W) {  // exclusive scan over the destination's experts
    int acc = 0;
    for (int e = 0; e < El; ++e) {
      const int i = threadIdx.x * El + e;
      s_off[i] += acc;
      acc += s_tot[i];
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int n = a.T * a.k;
  for (int p = blockIdx.x * nw + warp; p < n; p += gridDim.x * nw) {
    const int eg = a.ids[p];
    if (eg < 0 || eg >= W * El) continue;
    const int dst = eg / El, e = eg % El;
    int idx = 0;
    if (lane == 0) idx = s_off[dst * El + e] + atomicAdd(&a.send_ctr[dst * El + e], 1);
    idx = __shfl_sync(0xffffffffu, idx, 0);
    if (idx >= a.max_recv) {
      if (lane == 0) set_status(a.status, kStatusBounds);
      continue;
    }
    const int t = p / a.k, j = p % a.k;
    const uint4* src = reinterpret_cast<const uint4*>(a.x + (long)t * a.ldx);
    uint4* dstp = reinterpret_cast<uint4*>(a.peer_recv_x[dst] + (long)idx * H);
    for (int c = lane; c < H / 8; c += 32) dstp[c] = src[c];
    if (lane == 0) {
      const int4 tag = make_int4(a.rank, t, j, 0);
      *reinterpret_cast<int4*>(a.peer_recv_tag[dst] + (long)idx * 4) = tag;
    }
  }
  grid_publish(a, a.ticket_b, kEpFlagB, a.epoch_b);
}

__global__ void __launch_bounds__(64) ep_wait_kernel(EpArgs a, int flag_off, const int* epoch, int which) {
  pdl_trigger();
  pdl_wait();
  const bool ok = __syncthreads_and(wait_lane(a.flags + flag_off, a.world, (unsigned)(*epoch), a.status, a.limit_ns));
  if (threadIdx.x == 0) a.ok[1 + which] = ok ? 1 : 0;
}

__global__ void __launch_bounds__(256) ep_return_kernel(EpArgs a) {
  pdl_trigger();
  pdl_wait();
  if (!a.ok[1]) return;  // rows did not all arrive: return nothing
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int rows = a.recv_offsets[a.e_local];
  const int H = a.H;
  for (int r = blockIdx.x * nw + warp; r < rows && r < a.max_recv; r += gridDim.x * nw) {
    const int4 tag = __ldcg(reinterpret_cast<const int4*>(a.recv_tag + (long)r * 4));
    const int src = tag.x, t = tag.y, j = tag.z;
    if (src < 0 || src >= a.world || t < 0 || t >= a.T_max || j < 0 || j >= a.k) {
      if (lane == 0) set_status(a.status, kStatusBounds);
      continue;
    }
    const uint4* s = reinterpret_cast<const uint4*>(a.y + (long)r * a.ldy);  // local GEMM output
    uint4* d = reinterpret_cast<uint4*>(a.peer_comb[src] + ((long)t * a.k + j) * H);
    for (int c = lane; c < H / 8; c += 32) d[c] = s[c];
  }
  grid_publish(a, a.ticket_c, kEpFlagC, a.epoch_c);
}

void ep_count(const EpArgs& a, cudaStream_t st) {
  BWN_CHECK(a.world >= 1 && a.world <= kEpMaxRanks, "ep: 1..%d ranks", kEpMaxRanks);
  BWN_CHECK(a.H % 8 == 0, "ep: hidden must be a multiple of 8");
  const size_t smem = sizeof(int) * a.world * a.e_local;
  launch_k(ep_count_kernel, dim3(1), dim3(256), smem, st, a);
}

void ep_send(const EpArgs& a, cudaStream_t st) {
  const size_t smem = 2 * sizeof(int) * a.world * a.e_local;
  const int pairs = a.T * a.k;
  int grid = std::min((pairs + 7) / 8, num_sms());
  if (grid < 1) grid = 1;
  launch_k(ep_send_kernel, dim3(grid), dim3(256), smem, st, a);
}

void ep_wait(const EpArgs& a, int which, cudaStream_t st) {
  const int off = which == 0 ? kEpFlagB : kEpFlagC;
  launch_k(ep_wait_kernel, dim3(1), dim3(64), 0, st, a, off, which == 0 ? (const int*)a.epoch_b : (const int*)a.epoch_c,
           which);
}

void ep_return(const EpArgs& a, cudaStream_t st) {
  const int grid = std::max(1, std::min(a.max_recv / 8 + 1, num_sms()));
  launch_k(ep_return_kernel, dim3(grid), dim3(256), 0, st, a);
}

}  // namespace bwn
