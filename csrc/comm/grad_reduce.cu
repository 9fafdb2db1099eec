// Data-parallel gradient all-reduce fused with the cast and the 1/world scale,
// through NVLink multicast (NVLS).  The reference leaves gradient reduction to
// DTensor / FSDP collectives (contrib/esm2/train_esm.py:216-226,
// contrib/esm2/train_esm_fsdp.py:111-117).  Per gradient bucket:
//
//   grad_pack_kernel    fp32 grads * (1/world) -> bf16 into this rank's slot of
//                       the symmetric bucket buffer; the last CTA publishes
//                       flag 1 to every rank
//   grad_wait_kernel    one CTA waits for every rank's flag 1
//   grad_rs_ag_kernel   this rank's 1/world slice is read as the sum of all
//                       ranks' copies with multimem.ld_reduce (fp32
//                       accumulation in the switch) and written back to every
//                       rank's copy with one multimem.st (reduce-scatter +
//                       all-gather in one pass); the last CTA publishes flag 2
//   grad_wait_kernel    (flag 2), then grad_unpack_kernel: bf16 -> fp32 grads
//
// Each rank's NVLink port carries bucket/world bytes in and out per phase
// instead of the (world-1)/world * 2 of a ring.  The launches run on a side
// stream as buckets fill during backward.  All waits are bounded.
#include "comm/grad_reduce.h"
#include "common/host.h"
#include "common/launch.cuh"
#include "common/sm100.cuh"

namespace bwn {

namespace {

// true when every rank's flag reached `epoch` within the limit
__device__ __forceinline__ bool wait_all(const unsigned* flags, int world, unsigned epoch, int* status,
                                         uint64_t limit_ns) {
  const int r = threadIdx.x;
  bool ok = true;
  if (r < world) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while ((int)(ld_acquire_sys(flags + r) - epoch) < 0) {
      if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > limit_ns) {
        set_status(status, kStatusPeerTimeout);
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok);
}

__device__ __forceinline__ void grid_signal(const GradBucketArgs& a, int* ticket, int flag_slot) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int t = atomicAdd(ticket, 1);
    if (t == (int)gridDim.x - 1) {
      *ticket = 0;
      fence_acq_rel_sys();
      for (int r = 0; r < a.world; ++r) st_relaxed_sys_u32(a.peer_flags[r] + flag_slot + a.rank, a.epoch);
    }
  }
}

}  // namespace

__global__ void __launch_bounds__(256) grad_pack_kernel(GradBucketArgs a) {
  pdl_trigger();
  pdl_wait();
  const long n8 = a.n / 8;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    const float4 x0 = reinterpret_cast<const float4*>(a.grad)[2 * i];
    const float4 x1 = reinterpret_cast<const float4*>(a.grad)[2 * i + 1];
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
    o2[0] = __floats2bfloat162_rn(x0.x * a.scale, x0.y * a.scale);
    o2[1] = __floats2bfloat162_rn(x0.z * a.scale, x0.w * a.scale);
    o2[2] = __floats2bfloat162_rn(x1.x * a.scale, x1.y * a.scale);
    o2[3] = __floats2bfloat162_rn(x1.z * a.scale, x1.w * a.scale);
    reinterpret_cast<uint4*>(a.local)[i] = o;
  }
  grid_signal(a, a.ticket, 0);
}

// One CTA waits for a phase of every rank and records the outcome in
// ticket[1]; the kernels that follow are launched without programmatic
// overlap, so no CTA of theirs holds an SM while the peers are still behind
// (backward keeps running on the main stream), and after a timeout they touch
// no peer memory.
__global__ void __launch_bounds__(32) grad_wait_kernel(GradBucketArgs a, int slot) {
  const bool ok = wait_all(a.flags + slot, a.world, a.epoch, a.status, a.limit_ns);
  if (threadIdx.x == 0) a.ticket[1] = ok ? 1 : 0;
}

__global__ void __launch_bounds__(256) grad_rs_ag_kernel(GradBucketArgs a) {
  if (!a.ticket[1]) return;
  const long slice = a.n / a.world;  // multiple of 8
  const long base = (long)a.rank * slice;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < slice / 8; i += (long)gridDim.x * blockDim.x) {
    float v[8];
    mc_ld_reduce_bf16x8(a.mc + base + i * 8, v);
    mc_st_bf16x8(a.mc + base + i * 8, v);
  }
  grid_signal(a, a.ticket, kGradFlagSlots);
}

__global__ void __launch_bounds__(256) grad_unpack_kernel(GradBucketArgs a) {
  if (!a.ticket[1]) return;
  const long n8 = a.n / 8;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(a.local) + i);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
    float4 o0, o1;
    float2 f;
    f = __bfloat1622float2(h[0]); o0.x = f.x; o0.y = f.y;
    f = __bfloat1622float2(h[1]); o0.z = f.x; o0.w = f.y;
    f = __bfloat1622float2(h[2]); o1.x = f.x; o1.y = f.y;
    f = __bfloat1622float2(h[3]); o1.z = f.x; o1.w = f.y;
    reinterpret_cast<float4*>(a.grad)[2 * i] = o0;
    reinterpret_cast<float4*>(a.grad)[2 * i + 1] = o1;
  }
}

static int grid_for(long n8) {
  const long g = (n8 + 255) / 256;
  return (int)std::max<long>(1, std::min<long>(g, 4L * num_sms()));
}

void grad_bucket_reduce(const GradBucketArgs& a, cudaStream_t st) {
  BWN_CHECK(a.world >= 1 && a.world <= 8, "grad reduce: 1..8 ranks");
  BWN_CHECK(a.n % (8L * a.world) == 0, "grad reduce: bucket length must be a multiple of 8 * world");
  launch_k(grad_pack_kernel, dim3(grid_for(a.n / 8)), dim3(256), 0, st, a);
  grad_wait_kernel<<<1, 32, 0, st>>>(a, 0);
  grad_rs_ag_kernel<<<grid_for(a.n / 8 / a.world), 256, 0, st>>>(a);
  BWN_CUDA_CHECK(cudaGetLastError());
}

void grad_bucket_unpack(const GradBucketArgs& a, cudaStream_t st) {
  grad_wait_kernel<<<1, 32, 0, st>>>(a, kGradFlagSlots);
  grad_unpack_kernel<<<grid_for(a.n / 8), 256, 0, st>>>(a);
  BWN_CUDA_CHECK(cudaGetLastError());
}

}  // namespace bwn
