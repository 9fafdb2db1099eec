// Prefill op registrations (torch.ops.bwn.deltanet_prefill / gqa_prefill).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdlib>
#include <mutex>
#include <tuple>

#include "common/host.h"
#include "kernels/deepseek.h"
#include "kernels/launch.h"
#include "kernels/moe.h"
#include "kernels/prefill.h"
#include "ops_ext.h"

namespace bwn {
using at::Tensor;

static inline const __nv_bfloat16* cbf(const Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }
static inline __nv_bfloat16* mbf(const Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }

// qkv/z/a/b are [B, S, *] views of one projection output: inner stride 1, a
// common row stride between tokens (stride(1)), and stride(0) == S*stride(1).
static long row_stride(const Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() == 3 && t.stride(2) == 1, "bwn: ", name, " must be [B, S, *] with inner stride 1");
  TORCH_CHECK(t.size(0) == 1 || t.stride(0) == t.size(1) * t.stride(1), "bwn: ", name, " rows must be uniform");
  return t.stride(1);
}

// Optional int32 device tensor holding the chunk's start position in element 0.
static const int* start_ptr(const c10::optional<Tensor>& start_t, const Tensor& like) {
  if (!start_t.has_value()) return nullptr;
  TORCH_CHECK(start_t->scalar_type() == at::kInt && start_t->numel() >= 1 && start_t->device() == like.device(),
              "bwn: start_t must be an int32 tensor on the activations' device");
  return start_t->data_ptr<int>();
}

Tensor deltanet_prefill_op(const Tensor& qkv, const Tensor& z, const Tensor& a, const Tensor& b, Tensor conv_ring,
                           Tensor state, int64_t start, const Tensor& valid_len, const Tensor& conv_w,
                           const Tensor& A_log, const Tensor& dt_bias, const Tensor& norm_w, int64_t k_heads,
                           double eps, const c10::optional<Tensor>& start_t) {
  check_bf16(qkv, "qkv");
  check_bf16(z, "z");
  check_bf16(a, "a");
  check_bf16(b, "b");
  check_bf16(conv_ring, "conv_ring");
  check_f32(conv_w, "conv_w");
  TORCH_CHECK(valid_len.scalar_type() == at::kInt && valid_len.is_contiguous(), "valid_len int32");
  TORCH_CHECK(state.is_contiguous() && state.size(2) == 128 && state.size(3) == 128, "state [B,VH,128,128]");
  const c10::cuda::CUDAGuard guard(qkv.device());
  const int B = (int)qkv.size(0), S = (int)qkv.size(1), VH = (int)state.size(1);
  const int S_pad = ((S + 63) / 64) * 64;
  auto opt = qkv.options();
  auto qn = at::empty({B, k_heads, S_pad, 128}, opt);
  auto kn = at::empty({B, k_heads, S_pad, 128}, opt);
  auto vn = at::empty({B, VH, S_pad, 128}, opt);
  auto g = at::empty({B, VH, S_pad}, opt.dtype(at::kFloat));
  auto be = at::empty({B, VH, S_pad}, opt.dtype(at::kFloat));
  auto out = at::empty({B, S, VH * 128}, opt);
  DnPrefillArgs p{};
  p.qkv = cbf(qkv);
  p.qkv_row = row_stride(qkv, "qkv");
  p.z = cbf(z);
  p.z_row = row_stride(z, "z");
  p.a = cbf(a);
  p.b = cbf(b);
  p.ab_row = row_stride(a, "a");
  TORCH_CHECK(row_stride(b, "b") == p.ab_row, "a and b share a row stride");
  TORCH_CHECK(conv_ring.dim() == 3 && (conv_ring.size(1) == 4 || conv_ring.size(1) == 8) && conv_ring.is_contiguous(),
              "conv_ring [B, 4 or 8, C]");
  p.conv_ring = mbf(conv_ring);
  p.ring_slots = (int)conv_ring.size(1);
  p.state = state.data_ptr();
  p.state_bf16 = state.scalar_type() == at::kBFloat16;
  p.valid_len = valid_len.data_ptr<int>();
  p.conv_w = conv_w.data_ptr<float>();
  p.A_log = A_log.data_ptr<float>();
  p.dt_bias = dt_bias.data_ptr<float>();
  p.norm_w = norm_w.data_ptr<float>();
  p.q_out = mbf(qn);
  p.k_out = mbf(kn);
  p.v_out = mbf(vn);
  p.g_out = g.data_ptr<float>();
  p.beta_out = be.data_ptr<float>();
  p.out = mbf(out);
  p.out_row = out.stride(1);
  p.batch = B;
  p.S = S;
  p.status = status_dev_ptr();
  p.S_pad = S_pad;
  p.start = (int)start;
  p.start_dev = start_ptr(start_t, qkv);
  p.k_heads = (int)k_heads;
  p.v_heads = VH;
  p.l2_eps = 1e-6f;
  p.norm_eps = (float)eps;
  if (S > 0) deltanet_prefill(p, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

Tensor gqa_prefill_op(const Tensor& qg, const Tensor& k, const Tensor& v, const Tensor& q_norm_w,
                      const Tensor& k_norm_w, const Tensor& cos, const Tensor& sin, Tensor k_cache, Tensor v_cache,
                      int64_t start, double eps, const c10::optional<Tensor>& start_t) {
  check_bf16(qg, "qg");
  check_bf16(k, "k");
  check_bf16(v, "v");
  check_bf16(k_cache, "k_cache");
  TORCH_CHECK(qg.dim() == 4 && qg.size(3) == 512 && qg.stride(3) == 1 && qg.stride(2) == 512, "qg [B,S,QH,512]");
  TORCH_CHECK(k.dim() == 4 && k.size(3) == 256 && k.stride(3) == 1 && k.stride(2) == 256, "k [B,S,KVH,256]");
  TORCH_CHECK(v.stride(1) == k.stride(1) && v.stride(2) == 256, "v shares k's layout");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.size(3) == 256, "caches contiguous");
  const c10::cuda::CUDAGuard guard(qg.device());
  const int B = (int)qg.size(0), S = (int)qg.size(1), QH = (int)qg.size(2), KVH = (int)k.size(2);
  TORCH_CHECK(qg.size(0) == 1 || qg.stride(0) == S * qg.stride(1), "qg rows uniform");
  // with a device start the bound is checked by the kernel (status word)
  TORCH_CHECK(start_t.has_value() || start + S <= k_cache.size(2), "gqa_prefill: chunk exceeds the cache");
  const int S_pad = ((S + 127) / 128) * 128;
  auto q_rot = at::empty({B, QH, S_pad, 256}, qg.options());
  auto out = at::empty({B, S, QH * 256}, qg.options());
  GqaPrefillArgs p{};
  p.qg = cbf(qg);
  p.qg_row = qg.stride(1);
  p.k = cbf(k);
  p.v = cbf(v);
  p.kv_row = k.stride(1);
  p.q_norm_w = q_norm_w.data_ptr<float>();
  p.k_norm_w = k_norm_w.data_ptr<float>();
  p.cos = cos.data_ptr<float>();
  p.sin = sin.data_ptr<float>();
  p.k_cache = mbf(k_cache);
  p.v_cache = mbf(v_cache);
  p.q_rot = mbf(q_rot);
  p.out = mbf(out);
  p.out_row = out.stride(1);
  p.status = status_dev_ptr();
  p.batch = B;
  p.S = S;
  p.S_pad = S_pad;
  p.start = (int)start;
  p.start_dev = start_ptr(start_t, qg);
  p.q_heads = QH;
  p.kv_heads = KVH;
  p.s_max = (int)k_cache.size(2);
  p.rope_dim = (int)cos.size(1);
  p.eps = (float)eps;
  p.scale = 1.f / 16.f;  // 1/sqrt(256)
  if (S > 0) gqa_prefill(p, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

// ---------------------------------------------------------------------------
// MoE
// ---------------------------------------------------------------------------
std::tuple<Tensor, Tensor> moe_topk_op(const Tensor& logits, int64_t k, bool renorm, const c10::optional<Tensor>& bias,
                                       int64_t mode, double route_scale) {
  check_f32(logits, "logits");
  TORCH_CHECK(logits.dim() == 2 && logits.is_contiguous(), "logits [T, E] contiguous");
  const c10::cuda::CUDAGuard guard(logits.device());
  const int T = (int)logits.size(0), E = (int)logits.size(1);
  auto w = at::empty({T, k}, logits.options());
  auto ids = at::empty({T, k}, logits.options().dtype(at::kInt));
  MoeTopkArgs a{};
  a.logits = logits.data_ptr<float>();
  a.bias = bias.has_value() ? bias->data_ptr<float>() : nullptr;
  a.T = T;
  a.E = E;
  a.k = (int)k;
  a.renorm = renorm;
  a.deepseek = mode != 0;
  a.sqrt_softplus = mode == 1;
  a.route_scale = (float)route_scale;
  a.w = w.data_ptr<float>();
  a.ids = ids.data_ptr<int>();
  moe_topk(a, at::cuda::getCurrentCUDAStream().stream());
  return {w, ids};
}

// Routed experts of this rank: pack -> grouped gate/up (SwiGLU) -> grouped down
// -> weighted combine (+ gated shared expert).  Returns this rank's partial [T, H].
Tensor moe_experts_op(const Tensor& x, const Tensor& w, const Tensor& ids, const Tensor& gate_up, const Tensor& down,
                      int64_t e0, const c10::optional<Tensor>& shared_y, const c10::optional<Tensor>& shared_gate,
                      double swiglu_limit) {
  check_bf16(x, "x");
  check_bf16(gate_up, "gate_up");
  check_bf16(down, "down");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x [T, H]");
  TORCH_CHECK(gate_up.is_contiguous() && down.is_contiguous(), "expert weights contiguous");
  const c10::cuda::CUDAGuard guard(x.device());
  const int T = (int)x.size(0), H = (int)x.size(1), k = (int)ids.size(1);
  const int El = (int)gate_up.size(0), I2 = (int)gate_up.size(1), I = I2 / 2;
  TORCH_CHECK(down.size(0) == El && down.size(1) == H && down.size(2) == I, "down [E, H, I]");
  auto opt = x.options();
  auto iopt = opt.dtype(at::kInt);
  const int n = T * k;
  auto counts = at::empty({El}, iopt);
  auto offsets = at::empty({El + 1}, iopt);
  auto pos_of = at::empty({n}, iopt);
  auto row_src = at::empty({std::max(n, 1)}, iopt);
  auto xp = at::empty({std::max(n, 1), H}, opt);
  auto y1 = at::empty({std::max(n, 1), I}, opt);
  auto y2 = at::empty({std::max(n, 1), H}, opt);
  auto out = at::empty({T, H}, opt);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  MoeRouteArgs r{};
  r.ids = ids.data_ptr<int>();
  r.T = T;
  r.k = k;
  r.e0 = (int)e0;
  r.E_local = El;
  r.counts = counts.data_ptr<int>();
  r.offsets = offsets.data_ptr<int>();
  r.pos_of = pos_of.data_ptr<int>();
  r.row_src = row_src.data_ptr<int>();
  r.x = cbf(x);
  r.ldx = x.stride(0);
  r.H = H;
  r.x_perm = mbf(xp);
  moe_route(r, st);
  GroupedProblem g{};
  g.W = gate_up.data_ptr();
  g.X = xp.data_ptr();
  g.rows_total = n;
  g.counts = r.counts;
  g.offsets = r.offsets;
  g.groups = El;
  g.N = I2;
  g.K = H;
  g.max_rows_per_group = T;
  g.swiglu = true;
  g.swiglu_limit = (float)swiglu_limit;
  g.out = mbf(y1);
  g.ldo = I;
  g.status = status_dev_ptr();
  grouped_gemm(g, st);
  g.W = down.data_ptr();
  g.X = y1.data_ptr();
  g.N = H;
  g.K = I;
  g.swiglu = false;
  g.swiglu_limit = 0.f;
  g.out = mbf(y2);
  g.ldo = H;
  grouped_gemm(g, st);
  MoeCombineArgs c{};
  c.y = cbf(y2);
  c.w = w.data_ptr<float>();
  c.pos_of = r.pos_of;
  c.T = T;
  c.k = k;
  c.H = H;
  if (shared_y.has_value()) {
    c.shared_y = cbf(*shared_y);
    c.ld_shared = shared_y->stride(0);
    c.shared_gate = shared_gate.has_value() ? shared_gate->data_ptr<float>() : nullptr;
  }
  c.out = mbf(out);
  c.ldo = out.stride(0);
  moe_combine(c, st);
  return out;
}

// Routed experts with block-scaled E4M3FN weights (scales per 16 rows x 128
// columns, csrc/kernels/moe.h): the same pack -> gate/up (SwiGLU) -> down ->
// combine pipeline as moe_experts, the two GEMMs on the fp8 grouped kernel.
Tensor moe_experts_w8_op(const Tensor& x, const Tensor& w, const Tensor& ids, const Tensor& gate_up8,
                         const Tensor& gate_up_s16, const Tensor& down8, const Tensor& down_s16, int64_t e0,
                         const c10::optional<Tensor>& shared_y, const c10::optional<Tensor>& shared_gate,
                         double swiglu_limit) {
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x [T, H]");
  TORCH_CHECK(gate_up8.is_cuda() && gate_up8.scalar_type() == at::kByte && gate_up8.is_contiguous() &&
                  gate_up8.dim() == 3, "gate_up8: uint8 [E, 2I, H] contiguous");
  TORCH_CHECK(down8.is_cuda() && down8.scalar_type() == at::kByte && down8.is_contiguous() && down8.dim() == 3,
              "down8: uint8 [E, H, I] contiguous");
  check_f32(gate_up_s16, "gate_up_scales16");
  check_f32(down_s16, "down_scales16");
  const c10::cuda::CUDAGuard guard(x.device());
  const int T = (int)x.size(0), H = (int)x.size(1), k = (int)ids.size(1);
  const int El = (int)gate_up8.size(0), I2 = (int)gate_up8.size(1), I = I2 / 2;
  TORCH_CHECK(gate_up8.size(2) == H && down8.size(0) == El && down8.size(1) == H && down8.size(2) == I,
              "expert shapes: gate_up8 [E, 2I, H], down8 [E, H, I]");
  TORCH_CHECK(gate_up_s16.is_contiguous() && gate_up_s16.numel() == (long)El * (I2 / 16) * ((H + 127) / 128),
              "gate_up_scales16 [E, 2I/16, ceil(H/128)]");
  TORCH_CHECK(down_s16.is_contiguous() && down_s16.numel() == (long)El * (H / 16) * ((I + 127) / 128),
              "down_scales16 [E, H/16, ceil(I/128)]");
  auto opt = x.options();
  auto iopt = opt.dtype(at::kInt);
  const int n = T * k;
  auto counts = at::empty({El}, iopt);
  auto offsets = at::empty({El + 1}, iopt);
  auto pos_of = at::empty({n}, iopt);
  auto row_src = at::empty({std::max(n, 1)}, iopt);
  auto xp = at::empty({std::max(n, 1), H}, opt);
  auto y1 = at::empty({std::max(n, 1), I}, opt);
  auto y2 = at::empty({std::max(n, 1), H}, opt);
  auto out = at::empty({T, H}, opt);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  MoeRouteArgs r{};
  r.ids = ids.data_ptr<int>();
  r.T = T;
  r.k = k;
  r.e0 = (int)e0;
  r.E_local = El;
  r.counts = counts.data_ptr<int>();
  r.offsets = offsets.data_ptr<int>();
  r.pos_of = pos_of.data_ptr<int>();
  r.row_src = row_src.data_ptr<int>();
  r.x = cbf(x);
  r.ldx = x.stride(0);
  r.H = H;
  r.x_perm = mbf(xp);
  moe_route(r, st);
  GroupedW8Problem g{};
  g.W = gate_up8.data_ptr<uint8_t>();
  g.scales16 = gate_up_s16.data_ptr<float>();
  g.X = xp.data_ptr();
  g.rows_total = n;
  g.counts = r.counts;
  g.offsets = r.offsets;
  g.groups = El;
  g.N = I2;
  g.K = H;
  g.max_rows_per_group = T;
  g.swiglu = true;
  g.swiglu_limit = (float)swiglu_limit;
  g.out = mbf(y1);
  g.ldo = I;
  g.status = status_dev_ptr();
  grouped_gemm_w8(g, st);
  g.W = down8.data_ptr<uint8_t>();
  g.scales16 = down_s16.data_ptr<float>();
  g.X = y1.data_ptr();
  g.N = H;
  g.K = I;
  g.swiglu = false;
  g.swiglu_limit = 0.f;
  g.out = mbf(y2);
  g.ldo = H;
  grouped_gemm_w8(g, st);
  MoeCombineArgs c{};
  c.y = cbf(y2);
  c.w = w.data_ptr<float>();
  c.pos_of = r.pos_of;
  c.T = T;
  c.k = k;
  c.H = H;
  if (shared_y.has_value()) {
    c.shared_y = cbf(*shared_y);
    c.ld_shared = shared_y->stride(0);
    c.shared_gate = shared_gate.has_value() ? shared_gate->data_ptr<float>() : nullptr;
  }
  c.out = mbf(out);
  c.ldo = out.stride(0);
  moe_combine(c, st);
  return out;
}

// ---------------------------------------------------------------------------
// Decode-sized MoE block (csrc/kernels/moe_decode.cu): fused routing and gather
// (+ the shared expert as one more group), the two grouped GEMMs (bf16, or fp8
// E4M3FN experts when gate_up is uint8), then one combine kernel.

// grid-barrier words of moe_route_fused, one pair per device, zeroed once
static unsigned* moe_barrier_for(const Tensor& like) {
  static std::mutex mu;
  static Tensor bars[64];
  const int dev = like.get_device();
  std::lock_guard<std::mutex> lk(mu);
  if (!bars[dev & 63].defined()) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(at::cuda::getCurrentCUDAStream(dev).stream(), &cs);
    TORCH_CHECK(cs == cudaStreamCaptureStatusNone,
                "bwn: moe_decode must run once eagerly before CUDA-graph capture");
    bars[dev & 63] = at::zeros({64}, like.options().dtype(at::kInt));
  }
  return reinterpret_cast<unsigned*>(bars[dev & 63].data_ptr<int>());
}

// Returns (y [rows, H], w [T, k], pos_of [T, k], pos_sh [T], sg [T]); rows
// T*k + T.  gate_up [G, 2I, H] / down [G, H, I] hold this rank's experts and,
// with shared_group, the shared expert as group G-1 (its rows: tokens [t_lo, t_hi)).
std::vector<Tensor> moe_decode_op(const Tensor& x, const Tensor& router, const Tensor& gate_up, const Tensor& down,
                                  const c10::optional<Tensor>& gate_up_s16, const c10::optional<Tensor>& down_s16,
                                  int64_t e0, int64_t E, int64_t k, bool renorm, bool has_sg, bool shared_group,
                                  int64_t t_lo, int64_t t_hi, double swiglu_limit) {
  check_bf16(x, "x");
  check_bf16(router, "router");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && router.is_contiguous(), "x [T, H] rows, router contiguous");
  const bool fp8 = gate_up.scalar_type() == at::kByte;
  if (!fp8) {
    check_bf16(gate_up, "gate_up");
    check_bf16(down, "down");
  } else {
    TORCH_CHECK(gate_up_s16.has_value() && down_s16.has_value(), "fp8 experts need their scales");
    check_f32(*gate_up_s16, "gate_up_scales16");
    check_f32(*down_s16, "down_scales16");
  }
  TORCH_CHECK(gate_up.is_contiguous() && down.is_contiguous() && gate_up.dim() == 3 && down.dim() == 3,
              "experts [G, 2I, H] / [G, H, I] contiguous");
  const c10::cuda::CUDAGuard guard(x.device());
  const int T = (int)x.size(0), H = (int)x.size(1);
  const int G = (int)gate_up.size(0), I2 = (int)gate_up.size(1), I = I2 / 2;
  const int El = G - (shared_group ? 1 : 0);
  TORCH_CHECK(gate_up.size(2) == H && down.size(0) == G && down.size(1) == H && down.size(2) == I,
              "expert shapes: gate_up [G, 2I, H], down [G, H, I]");
  TORCH_CHECK(router.size(0) == E + (has_sg ? 1 : 0) && router.size(1) == H, "router [E (+1), H]");
  auto opt = x.options();
  auto iopt = opt.dtype(at::kInt);
  auto fopt = opt.dtype(at::kFloat);
  const int rows = T * (int)k + T;
  auto logits = at::empty({T, router.size(0)}, fopt);
  auto w = at::empty({T, k}, fopt);
  auto ids = at::empty({T, k}, iopt);
  auto sg = at::empty({T}, fopt);
  auto counts = at::empty({G}, iopt);
  auto offsets = at::empty({G + 1}, iopt);
  auto pos_of = at::empty({T, k}, iopt);
  auto pos_sh = at::empty({T}, iopt);
  auto xp = at::empty({rows, H}, opt);
  auto y1 = at::empty({rows, I}, opt);
  auto y2 = at::empty({rows, H}, opt);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  MoeRouteFusedArgs r{};
  r.x = cbf(x);
  r.ldx = x.stride(0);
  r.router = cbf(router);
  r.T = T;
  r.H = H;
  r.E = (int)E;
  r.k = (int)k;
  r.renorm = renorm;
  r.has_sg = has_sg;
  r.e0 = (int)e0;
  r.E_local = El;
  r.shared_group = shared_group;
  r.t_lo = (int)t_lo;
  r.t_hi = (int)t_hi;
  r.logits = logits.data_ptr<float>();
  r.bar = moe_barrier_for(x);
  r.w = w.data_ptr<float>();
  r.ids = ids.data_ptr<int>();
  r.sg = sg.data_ptr<float>();
  r.counts = counts.data_ptr<int>();
  r.offsets = offsets.data_ptr<int>();
  r.pos_of = pos_of.data_ptr<int>();
  r.pos_sh = pos_sh.data_ptr<int>();
  r.x_perm = mbf(xp);
  r.status = status_dev_ptr();
  r.limit_ns = 1000000000ull;
  moe_route_fused(r, st);
  const int max_rows = std::max(T, 1);
  if (!fp8) {
    GroupedProblem g{};
    g.W = gate_up.data_ptr();
    g.X = xp.data_ptr();
    g.rows_total = rows;
    g.counts = r.counts;
    g.offsets = r.offsets;
    g.groups = G;
    g.N = I2;
    g.K = H;
    g.max_rows_per_group = max_rows;
    g.swiglu = true;
    g.swiglu_limit = (float)swiglu_limit;
    g.out = mbf(y1);
    g.ldo = I;
    g.status = status_dev_ptr();
    grouped_gemm(g, st);
    g.W = down.data_ptr();
    g.X = y1.data_ptr();
    g.N = H;
    g.K = I;
    g.swiglu = false;
    g.swiglu_limit = 0.f;
    g.out = mbf(y2);
    g.ldo = H;
    grouped_gemm(g, st);
  } else {
    GroupedW8Problem g{};
    g.W = gate_up.data_ptr<uint8_t>();
    g.scales16 = gate_up_s16->data_ptr<float>();
    g.X = xp.data_ptr();
    g.rows_total = rows;
    g.counts = r.counts;
    g.offsets = r.offsets;
    g.groups = G;
    g.N = I2;
    g.K = H;
    g.max_rows_per_group = max_rows;
    g.swiglu = true;
    g.swiglu_limit = (float)swiglu_limit;
    g.out = mbf(y1);
    g.ldo = I;
    g.status = status_dev_ptr();
    grouped_gemm_w8(g, st);
    g.W = down.data_ptr<uint8_t>();
    g.scales16 = down_s16->data_ptr<float>();
    g.X = y1.data_ptr();
    g.N = H;
    g.K = I;
    g.swiglu = false;
    g.swiglu_limit = 0.f;
    g.out = mbf(y2);
    g.ldo = H;
    grouped_gemm_w8(g, st);
  }
  return {y2, w, pos_of, pos_sh, sg};
}

MoeCombineExArgs combine_args(const Tensor& y, const Tensor& w, const Tensor& pos_of,
                              const c10::optional<Tensor>& pos_sh, const c10::optional<Tensor>& sg,
                              const c10::optional<Tensor>& shared_y, const c10::optional<Tensor>& shared_gate) {
  check_bf16(y, "y");
  check_f32(w, "w");
  TORCH_CHECK(y.is_contiguous() && w.is_contiguous() && pos_of.is_contiguous() && pos_of.scalar_type() == at::kInt,
              "moe combine: contiguous y, w, int32 pos_of");
  MoeCombineExArgs c{};
  c.y = cbf(y);
  c.w = w.data_ptr<float>();
  c.pos_of = pos_of.data_ptr<int>();
  c.T = (int)w.size(0);
  c.k = (int)w.size(1);
  c.H = (int)y.size(1);
  if (pos_sh.has_value()) {
    TORCH_CHECK(sg.has_value() && pos_sh->scalar_type() == at::kInt && pos_sh->numel() == c.T, "pos_sh [T] int32");
    c.pos_sh = pos_sh->data_ptr<int>();
    c.sg = sg->data_ptr<float>();
  }
  if (shared_y.has_value()) {
    check_bf16(*shared_y, "shared_y");
    TORCH_CHECK(shared_gate.has_value(), "shared_y needs shared_gate");
    c.shared_y = cbf(*shared_y);
    c.ld_shared = shared_y->stride(0);
    c.shared_gate = shared_gate->data_ptr<float>();
  }
  return c;
}

// mode 0: returns the partial [T, H]; mode 1: resid += partial, returns RMSNorm(resid) * (1 + norm_w)
Tensor moe_combine_ex_op(const Tensor& y, const Tensor& w, const Tensor& pos_of, const c10::optional<Tensor>& pos_sh,
                         const c10::optional<Tensor>& sg, const c10::optional<Tensor>& shared_y,
                         const c10::optional<Tensor>& shared_gate, int64_t mode, const c10::optional<Tensor>& resid,
                         const c10::optional<Tensor>& norm_w, double eps) {
  const c10::cuda::CUDAGuard guard(y.device());
  MoeCombineExArgs c = combine_args(y, w, pos_of, pos_sh, sg, shared_y, shared_gate);
  auto out = at::empty({c.T, c.H}, y.options());
  c.mode = (int)mode;
  c.out = mbf(out);
  c.ldo = out.stride(0);
  if (mode == kCombineAddNorm) {
    TORCH_CHECK(resid.has_value() && norm_w.has_value(), "add-norm needs resid and norm_w");
    check_bf16(*resid, "resid");
    check_f32(*norm_w, "norm_w");
    TORCH_CHECK(resid->stride(1) == 1 && resid->size(0) == c.T && resid->size(1) == c.H, "resid [T, H]");
    c.resid = mbf(*resid);
    c.ldr = resid->stride(0);
    c.norm_w = norm_w->data_ptr<float>();
    c.eps = (float)eps;
  } else {
    TORCH_CHECK(mode == kCombinePartial, "moe_combine_ex: mode 0 or 1 (the symmetric-slot mode is moe_combine_symm)");
  }
  moe_combine_ex(c, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

// ---------------------------------------------------------------------------
// DeepSeek V4
// ---------------------------------------------------------------------------
std::tuple<Tensor, Tensor, Tensor> hc_pre_op(const Tensor& x, const Tensor& fn, const Tensor& scale, const Tensor& base,
                                             int64_t iters, double eps, double norm_eps,
                                             const c10::optional<Tensor>& mix_in) {
  check_bf16(x, "x");
  check_f32(fn, "fn");
  TORCH_CHECK(x.dim() == 3 && x.is_contiguous(), "x [T, hc, dim] contiguous");
  const c10::cuda::CUDAGuard guard(x.device());
  const int T = (int)x.size(0), hc = (int)x.size(1), dim = (int)x.size(2), mix = (int)fn.size(0);
  auto y = at::empty({T, dim}, x.options());
  auto post = at::empty({T, hc}, x.options().dtype(at::kFloat));
  auto comb = at::empty({T, hc, hc}, x.options().dtype(at::kFloat));
  HcPreArgs a{};
  a.x = cbf(x);
  a.fn = fn.data_ptr<float>();
  a.scale = scale.data_ptr<float>();
  a.base = base.data_ptr<float>();
  a.tokens = T;
  a.hc = hc;
  a.dim = dim;
  a.mix_out = mix;
  a.sinkhorn_iters = (int)iters;
  a.eps = (float)eps;
  a.norm_eps = (float)norm_eps;
  a.y = mbf(y);
  a.post = post.data_ptr<float>();
  a.comb = comb.data_ptr<float>();
  if (mix_in.has_value()) {
    check_f32(*mix_in, "mix_in");
    TORCH_CHECK(mix_in->dim() == 2 && mix_in->size(0) == T && mix_in->size(1) >= mix && mix_in->stride(1) == 1,
                "hc_pre: mix_in [T, >= mix_out] rows");
    TORCH_CHECK(((long)hc * dim) % 8 == 0, "hc_pre: hc*dim multiple of 8");
    a.mix_in = mix_in->data_ptr<float>();
    a.ld_mix = (int)mix_in->stride(0);
  }
  hc_pre(a, at::cuda::getCurrentCUDAStream().stream());
  return {y, post, comb};
}

Tensor hc_post_op(const Tensor& x, const Tensor& resid, const Tensor& post, const Tensor& comb) {
  check_bf16(x, "x");
  check_bf16(resid, "resid");
  TORCH_CHECK(x.is_contiguous() && resid.is_contiguous() && post.is_contiguous() && comb.is_contiguous(), "contig");
  const c10::cuda::CUDAGuard guard(x.device());
  auto out = at::empty_like(resid);
  hc_post(cbf(x), cbf(resid), post.data_ptr<float>(), comb.data_ptr<float>(), (int)resid.size(0), (int)resid.size(1),
          (int)resid.size(2), mbf(out), at::cuda::getCurrentCUDAStream().stream());
  return out;
}

// BWN_MQA_TC=0 keeps prefill-sized MQA on the CUDA-core kernel (A/B measurement).
static bool mqa_tc_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("BWN_MQA_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

Tensor mqa_attn_op(const Tensor& q, const Tensor& kv, const Tensor& visible, int64_t q_per_seq, double scale,
                   int64_t splits) {
  check_bf16(q, "q");
  check_bf16(kv, "kv");
  TORCH_CHECK(q.dim() == 3 && q.is_contiguous(), "q [rows, H, D]");
  TORCH_CHECK(kv.dim() == 3 && kv.stride(2) == 1 && kv.stride(1) == kv.size(2), "kv [B, T, D]");
  TORCH_CHECK(visible.scalar_type() == at::kInt && visible.is_contiguous(), "visible int32");
  const c10::cuda::CUDAGuard guard(q.device());
  const int rows = (int)q.size(0), H = (int)q.size(1), D = (int)q.size(2);
  {
    // prefill-sized: the tcgen05 kernel (no splits, no partials)
    MqaArgs t{};
    t.q = cbf(q);
    t.kv = cbf(kv);
    t.kv_seq_stride = kv.stride(0);
    t.visible = visible.data_ptr<int>();
    t.rows = rows;
    t.q_per_seq = (int)q_per_seq;
    t.H = H;
    t.D = D;
    t.scale = (float)scale;
    const int kv_rows = (int)kv.size(1);
    if (splits <= 0 && (long)rows * H >= 1024 && mqa_tc_enabled() && mqa_prefill_tc_supported(t, kv_rows)) {
      auto out = at::empty_like(q);
      t.out = mbf(out);
      mqa_prefill_tc(t, kv_rows, (long)kv.size(0) * kv_rows, status_dev_ptr(), at::cuda::getCurrentCUDAStream().stream());
      return out;
    }
  }
  if (splits <= 0) splits = std::max<int64_t>(1, std::min<int64_t>(32, (2 * num_sms() + rows - 1) / std::max(rows, 1)));
  auto ws = at::empty({(long)rows * splits * H * (2 + D)}, q.options().dtype(at::kFloat));
  auto tickets = at::zeros({rows}, q.options().dtype(at::kInt));
  auto out = at::empty_like(q);
  MqaArgs a{};
  a.q = cbf(q);
  a.kv = cbf(kv);
  a.kv_seq_stride = kv.stride(0);
  a.visible = visible.data_ptr<int>();
  a.rows = rows;
  a.q_per_seq = (int)q_per_seq;
  a.H = H;
  a.D = D;
  a.splits = (int)splits;
  a.scale = (float)scale;
  a.workspace = ws.data_ptr<float>();
  a.tickets = tickets.data_ptr<int>();
  a.out = mbf(out);
  mqa_attn(a, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

// ESM-2 rotary embedding fused with the scale and the layout change around
// attention: to_heads: x [B*S, H*D] (rows b*S+s) -> out [B, H, S, D];
// otherwise x [B, H, S, D] -> out [B*S, H*D].  sign -1 applies the transposed
// rotation (the backward of the forward one).
Tensor rope_half_op(const Tensor& x, const Tensor& cos, const Tensor& sin, int64_t B, int64_t S, int64_t H,
                    bool to_heads, double sign, double scale) {
  check_bf16(x, "x");
  check_f32(cos, "cos");
  check_f32(sin, "sin");
  TORCH_CHECK(x.is_contiguous() && cos.is_contiguous() && sin.is_contiguous(), "rope_half: contiguous inputs");
  TORCH_CHECK(x.numel() % (B * S * H) == 0, "rope_half: shape");
  const int64_t D = x.numel() / (B * S * H);
  TORCH_CHECK(D % 4 == 0 && cos.size(0) >= S && cos.size(1) == D / 2 && sin.sizes() == cos.sizes(),
              "rope_half: tables [>= S, D/2], D multiple of 4");
  const c10::cuda::CUDAGuard guard(x.device());
  Tensor out = to_heads ? at::empty({B, H, S, D}, x.options()) : at::empty({B * S, H * D}, x.options());
  RopeHalfArgs a{};
  a.in = cbf(x);
  a.out = mbf(out);
  const long tok_b = S * H * D, tok_s = H * D, tok_h = D;   // [B, S, H, D]
  const long hd_b = H * S * D, hd_s = D, hd_h = S * D;      // [B, H, S, D]
  if (to_heads) {
    a.in_b = tok_b; a.in_s = tok_s; a.in_h = tok_h;
    a.out_b = hd_b; a.out_s = hd_s; a.out_h = hd_h;
  } else {
    a.in_b = hd_b; a.in_s = hd_s; a.in_h = hd_h;
    a.out_b = tok_b; a.out_s = tok_s; a.out_h = tok_h;
  }
  a.cos = cos.data_ptr<float>();
  a.sin = sin.data_ptr<float>();
  a.B = (int)B;
  a.S = (int)S;
  a.H = (int)H;
  a.D = (int)D;
  a.sign = (float)sign;
  a.scale = (float)scale;
  rope_half(a, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

void rope_interleaved_op(Tensor x, const Tensor& cos, const Tensor& sin, const Tensor& pos) {
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() == 3 && x.is_contiguous(), "x [rows, H, D] contiguous");
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.is_contiguous(), "pos int32");
  const c10::cuda::CUDAGuard guard(x.device());
  rope_interleaved(mbf(x), (int)x.size(0), (int)x.size(1), (int)x.size(2), (int)cos.size(1), cos.data_ptr<float>(),
                   sin.data_ptr<float>(), pos.data_ptr<int>(), at::cuda::getCurrentCUDAStream().stream());
}

// Speculative verify of n_tok tokens per sequence with deferred commit.
// qkv/z/a/b: [B*n_tok, *] row views of one projection output.
Tensor deltanet_verify_op(const Tensor& qkv, const Tensor& z, const Tensor& a, const Tensor& b, Tensor stash_qkv,
                          Tensor stash_ab, const Tensor& vstep, Tensor conv_ring, Tensor state,
                          const Tensor& positions, const Tensor& pending, const Tensor& conv_w, const Tensor& A_log,
                          const Tensor& dt_bias, const Tensor& norm_w, int64_t k_heads, int64_t n_tok, double eps) {
  for (const Tensor* t : std::initializer_list<const Tensor*>{&qkv, &z, &a, &b, &stash_qkv, &stash_ab, &conv_ring})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16, "deltanet_verify: bf16 CUDA tensors expected");
  TORCH_CHECK(state.is_contiguous() && state.dim() == 4 && state.size(2) == 128 && state.size(3) == 128,
              "state [B, VH, 128, 128]");
  TORCH_CHECK(state.scalar_type() == at::kFloat || state.scalar_type() == at::kBFloat16, "state fp32/bf16");
  const int B = (int)state.size(0), VH = (int)state.size(1);
  const long C = conv_ring.size(2);
  TORCH_CHECK(conv_ring.is_contiguous() && conv_ring.size(0) == B, "conv_ring [B, R, C]");
  TORCH_CHECK(stash_qkv.is_contiguous() && stash_qkv.dim() == 4 && stash_qkv.size(0) == 2 && stash_qkv.size(1) == B &&
                  stash_qkv.size(2) >= n_tok && stash_qkv.size(3) == C,
              "stash_qkv [2, B, SN >= n_tok, C]");
  const long SN = stash_qkv.size(2);
  TORCH_CHECK(stash_ab.is_contiguous() && stash_ab.numel() == 2L * B * SN * 2 * VH, "stash_ab [2, B, SN, 2*VH]");
  TORCH_CHECK(positions.scalar_type() == at::kInt && pending.scalar_type() == at::kInt && vstep.scalar_type() == at::kInt,
              "positions / pending / vstep int32");
  TORCH_CHECK(positions.numel() == B && pending.numel() == B, "positions / pending: one per sequence");
  for (const Tensor* t : std::initializer_list<const Tensor*>{&qkv, &z, &a, &b})
    TORCH_CHECK(t->dim() == 2 && t->size(0) == (long)B * n_tok && t->stride(1) == 1, "rows [B*n_tok, *]");
  TORCH_CHECK(a.stride(0) == b.stride(0), "a and b share a row stride");
  TORCH_CHECK(qkv.size(1) == C && z.size(1) == (long)VH * 128 && a.size(1) == VH, "row widths");
  const c10::cuda::CUDAGuard guard(state.device());
  auto out = at::empty({(long)B * n_tok, (long)VH * 128}, qkv.options());
  DnVerifyArgs p{};
  p.qkv = cbf(qkv);
  p.qkv_row = qkv.stride(0);
  p.z = cbf(z);
  p.z_row = z.stride(0);
  p.a = cbf(a);
  p.b = cbf(b);
  p.ab_row = a.stride(0);
  p.stash_qkv = mbf(stash_qkv);
  p.stash_ab = mbf(stash_ab);
  p.stash_n = (int)SN;
  p.vstep = vstep.data_ptr<int>();
  p.conv_ring = mbf(conv_ring);
  p.ring_slots = (int)conv_ring.size(1);
  p.state = state.data_ptr();
  p.state_bf16 = state.scalar_type() == at::kBFloat16;
  p.positions = positions.data_ptr<int>();
  p.pending = pending.data_ptr<int>();
  p.conv_w = conv_w.data_ptr<float>();
  p.A_log = A_log.data_ptr<float>();
  p.dt_bias = dt_bias.data_ptr<float>();
  p.norm_w = norm_w.data_ptr<float>();
  p.out = mbf(out);
  p.out_row = out.stride(0);
  p.status = status_dev_ptr();
  p.batch = B;
  p.n_tok = (int)n_tok;
  p.k_heads = (int)k_heads;
  p.v_heads = VH;
  p.l2_eps = 1e-6f;
  p.norm_eps = (float)eps;
  deltanet_verify(p, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

// Routed-expert FFN on rows already grouped by expert (device counts/offsets):
// gate/up GEMM with the SwiGLU epilogue, then the down GEMM.  Used on the
// expert-parallel receive buffer.
Tensor moe_grouped_ffn_op(const Tensor& x_perm, const Tensor& counts, const Tensor& offsets, const Tensor& gate_up,
                          const Tensor& down, int64_t max_rows_per_group, double swiglu_limit) {
  check_bf16(x_perm, "x_perm");
  check_bf16(gate_up, "gate_up");
  check_bf16(down, "down");
  TORCH_CHECK(x_perm.dim() == 2 && x_perm.is_contiguous(), "x_perm [rows, H] contiguous");
  TORCH_CHECK(counts.scalar_type() == at::kInt && offsets.scalar_type() == at::kInt, "counts/offsets int32");
  const c10::cuda::CUDAGuard guard(x_perm.device());
  const int rows = (int)x_perm.size(0), H = (int)x_perm.size(1);
  const int El = (int)gate_up.size(0), I2 = (int)gate_up.size(1), I = I2 / 2;
  TORCH_CHECK(down.size(0) == El && down.size(1) == H && down.size(2) == I, "down [E, H, I]");
  auto y1 = at::empty({std::max(rows, 1), I}, x_perm.options());
  auto y2 = at::empty({std::max(rows, 1), H}, x_perm.options());
  auto st = at::cuda::getCurrentCUDAStream().stream();
  GroupedProblem g{};
  g.W = gate_up.data_ptr();
  g.X = x_perm.data_ptr();
  g.rows_total = rows;
  g.counts = counts.data_ptr<int>();
  g.offsets = offsets.data_ptr<int>();
  g.groups = El;
  g.N = I2;
  g.K = H;
  g.max_rows_per_group = (int)max_rows_per_group;
  g.swiglu = true;
  g.swiglu_limit = (float)swiglu_limit;
  g.out = mbf(y1);
  g.ldo = I;
  g.status = status_dev_ptr();
  grouped_gemm(g, st);
  g.W = down.data_ptr();
  g.X = y1.data_ptr();
  g.N = H;
  g.K = I;
  g.swiglu = false;
  g.swiglu_limit = 0.f;
  g.out = mbf(y2);
  g.ldo = H;
  grouped_gemm(g, st);
  return y2;
}

// moe_grouped_ffn with block-scaled E4M3FN experts (scales per 16 rows x 128
// columns): the expert-parallel receive buffer through the fp8 grouped GEMM.
Tensor moe_grouped_ffn_w8_op(const Tensor& x_perm, const Tensor& counts, const Tensor& offsets,
                             const Tensor& gate_up8, const Tensor& gate_up_s16, const Tensor& down8,
                             const Tensor& down_s16, int64_t max_rows_per_group, double swiglu_limit) {
  check_bf16(x_perm, "x_perm");
  TORCH_CHECK(x_perm.dim() == 2 && x_perm.is_contiguous(), "x_perm [rows, H] contiguous");
  TORCH_CHECK(counts.scalar_type() == at::kInt && offsets.scalar_type() == at::kInt, "counts/offsets int32");
  TORCH_CHECK(gate_up8.is_cuda() && gate_up8.scalar_type() == at::kByte && gate_up8.is_contiguous() &&
                  gate_up8.dim() == 3, "gate_up8: uint8 [E, 2I, H] contiguous");
  TORCH_CHECK(down8.is_cuda() && down8.scalar_type() == at::kByte && down8.is_contiguous() && down8.dim() == 3,
              "down8: uint8 [E, H, I] contiguous");
  check_f32(gate_up_s16, "gate_up_scales16");
  check_f32(down_s16, "down_scales16");
  const c10::cuda::CUDAGuard guard(x_perm.device());
  const int rows = (int)x_perm.size(0), H = (int)x_perm.size(1);
  const int El = (int)gate_up8.size(0), I2 = (int)gate_up8.size(1), I = I2 / 2;
  TORCH_CHECK(gate_up8.size(2) == H && down8.size(0) == El && down8.size(1) == H && down8.size(2) == I,
              "expert shapes: gate_up8 [E, 2I, H], down8 [E, H, I]");
  TORCH_CHECK(gate_up_s16.is_contiguous() && gate_up_s16.numel() == (long)El * (I2 / 16) * ((H + 127) / 128),
              "gate_up_scales16 [E, 2I/16, ceil(H/128)]");
  TORCH_CHECK(down_s16.is_contiguous() && down_s16.numel() == (long)El * (H / 16) * ((I + 127) / 128),
              "down_scales16 [E, H/16, ceil(I/128)]");
  auto y1 = at::empty({std::max(rows, 1), I}, x_perm.options());
  auto y2 = at::empty({std::max(rows, 1), H}, x_perm.options());
  auto st = at::cuda::getCurrentCUDAStream().stream();
  GroupedW8Problem g{};
  g.W = gate_up8.data_ptr<uint8_t>();
  g.scales16 = gate_up_s16.data_ptr<float>();
  g.X = x_perm.data_ptr();
  g.rows_total = rows;
  g.counts = counts.data_ptr<int>();
  g.offsets = offsets.data_ptr<int>();
  g.groups = El;
  g.N = I2;
  g.K = H;
  g.max_rows_per_group = (int)max_rows_per_group;
  g.swiglu = true;
  g.swiglu_limit = (float)swiglu_limit;
  g.out = mbf(y1);
  g.ldo = I;
  g.status = status_dev_ptr();
  grouped_gemm_w8(g, st);
  g.W = down8.data_ptr<uint8_t>();
  g.scales16 = down_s16.data_ptr<float>();
  g.X = y1.data_ptr();
  g.N = H;
  g.K = I;
  g.swiglu = false;
  g.swiglu_limit = 0.f;
  g.out = mbf(y2);
  g.ldo = H;
  grouped_gemm_w8(g, st);
  return y2;
}

// Router-weighted sum of per-(token, slot) expert outputs y[pos_of[t*k+j]]
// (+ the sigmoid-gated shared expert).
Tensor moe_combine_op(const Tensor& y, const Tensor& w, const Tensor& pos_of, const c10::optional<Tensor>& shared_y,
                      const c10::optional<Tensor>& shared_gate) {
  check_bf16(y, "y");
  TORCH_CHECK(y.dim() == 2 && y.is_contiguous(), "y [rows, H] contiguous");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && w.dim() == 2, "w fp32 [T, k]");
  TORCH_CHECK(pos_of.scalar_type() == at::kInt && pos_of.numel() == w.numel(), "pos_of int32 [T*k]");
  const c10::cuda::CUDAGuard guard(y.device());
  const int T = (int)w.size(0), k = (int)w.size(1), H = (int)y.size(1);
  auto out = at::empty({T, H}, y.options());
  MoeCombineArgs c{};
  c.y = cbf(y);
  c.w = w.data_ptr<float>();
  c.pos_of = pos_of.data_ptr<int>();
  c.T = T;
  c.k = k;
  c.H = H;
  if (shared_y.has_value()) {
    check_bf16(*shared_y, "shared_y");
    c.shared_y = cbf(*shared_y);
    c.ld_shared = shared_y->stride(0);
    c.shared_gate = shared_gate.has_value() ? shared_gate->data_ptr<float>() : nullptr;
  }
  c.out = mbf(out);
  c.ldo = out.stride(0);
  if (T > 0) moe_combine(c, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

void register_ext_defs(torch::Library& m) {
  m.def("moe_combine(Tensor y, Tensor w, Tensor pos_of, Tensor? shared_y, Tensor? shared_gate) -> Tensor");
  m.def(
      "moe_grouped_ffn(Tensor x_perm, Tensor counts, Tensor offsets, Tensor gate_up, Tensor down, "
      "int max_rows_per_group, float swiglu_limit) -> Tensor");
  m.def(
      "deltanet_verify(Tensor qkv, Tensor z, Tensor a, Tensor b, Tensor(a!) stash_qkv, Tensor(b!) stash_ab, "
      "Tensor vstep, Tensor(c!) conv_ring, Tensor(d!) state, Tensor positions, Tensor pending, Tensor conv_w, "
      "Tensor A_log, Tensor dt_bias, Tensor norm_w, int k_heads, int n_tok, float eps) -> Tensor");
  m.def("rope_interleaved_(Tensor(a!) x, Tensor cos, Tensor sin, Tensor pos) -> ()");
  m.def("rope_half(Tensor x, Tensor cos, Tensor sin, int B, int S, int H, bool to_heads, float sign, float scale) -> Tensor");
  register_comm_defs(m);
  m.def("moe_topk(Tensor logits, int k, bool renorm, Tensor? bias, int mode, float route_scale) -> (Tensor, Tensor)");
  m.def(
      "moe_experts(Tensor x, Tensor w, Tensor ids, Tensor gate_up, Tensor down, int e0, Tensor? shared_y, "
      "Tensor? shared_gate, float swiglu_limit) -> Tensor");
  m.def(
      "moe_grouped_ffn_w8(Tensor x_perm, Tensor counts, Tensor offsets, Tensor gate_up8, Tensor gate_up_scales16, "
      "Tensor down8, Tensor down_scales16, int max_rows_per_group, float swiglu_limit) -> Tensor");
  m.def(
      "moe_experts_w8(Tensor x, Tensor w, Tensor ids, Tensor gate_up8, Tensor gate_up_scales16, Tensor down8, "
      "Tensor down_scales16, int e0, Tensor? shared_y, Tensor? shared_gate, float swiglu_limit) -> Tensor");
  m.def(
      "hc_pre(Tensor x, Tensor fn, Tensor scale, Tensor base, int sinkhorn_iters, float eps, float norm_eps, "
      "Tensor? mix_in=None) -> (Tensor, Tensor, Tensor)");
  m.def("hc_post(Tensor x, Tensor resid, Tensor post, Tensor comb) -> Tensor");
  m.def(
      "moe_decode(Tensor x, Tensor router, Tensor gate_up, Tensor down, Tensor? gate_up_scales16, "
      "Tensor? down_scales16, int e0, int E, int k, bool renorm, bool has_sg, bool shared_group, int t_lo, int t_hi, "
      "float swiglu_limit) -> Tensor[]");
  m.def(
      "moe_combine_ex(Tensor y, Tensor w, Tensor pos_of, Tensor? pos_sh, Tensor? sg, Tensor? shared_y, "
      "Tensor? shared_gate, int mode, Tensor(a!)? resid, Tensor? norm_w, float eps) -> Tensor");
  m.def("mqa_attn(Tensor q, Tensor kv, Tensor visible, int q_per_seq, float scale, int splits) -> Tensor");
  m.def(
      "deltanet_prefill(Tensor qkv, Tensor z, Tensor a, Tensor b, Tensor(a!) conv_ring, Tensor(b!) state, int start, "
      "Tensor valid_len, Tensor conv_w, Tensor A_log, Tensor dt_bias, Tensor norm_w, int k_heads, float eps, "
      "Tensor? start_t=None) -> Tensor");
  m.def(
      "gqa_prefill(Tensor qg, Tensor k, Tensor v, Tensor q_norm_w, Tensor k_norm_w, Tensor cos, Tensor sin, "
      "Tensor(a!) k_cache, Tensor(b!) v_cache, int start, float eps, Tensor? start_t=None) -> Tensor");
}
void register_ext_impls(torch::Library& m) {
  register_comm_impls(m);
  m.impl("deltanet_verify", &deltanet_verify_op);
  m.impl("moe_topk", &moe_topk_op);
  m.impl("moe_experts", &moe_experts_op);
  m.impl("moe_experts_w8", &moe_experts_w8_op);
  m.impl("moe_grouped_ffn", &moe_grouped_ffn_op);
  m.impl("moe_grouped_ffn_w8", &moe_grouped_ffn_w8_op);
  m.impl("moe_combine", &moe_combine_op);
  m.impl("hc_pre", &hc_pre_op);
  m.impl("hc_post", &hc_post_op);
  m.impl("moe_decode", &moe_decode_op);
  m.impl("moe_combine_ex", &moe_combine_ex_op);
  m.impl("mqa_attn", &mqa_attn_op);
  m.impl("rope_interleaved_", &rope_interleaved_op);
  m.impl("rope_half", &rope_half_op);
  m.impl("deltanet_prefill", &deltanet_prefill_op);
  m.impl("gqa_prefill", &gqa_prefill_op);
}
void register_ext_pybind(pybind11::module& mod) { register_comm_pybind(mod); }
}  // namespace bwn
