// torch.ops.bwn.* registrations: validate tensors, build launch descriptors,
// launch on the current CUDA stream.  Every custom op is one opaque node, the
// role torch_neuronx.nki_op plays for the reference's NKI kernels
// (contrib/qwen3.6-27b/kernels/*_ops.py).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>
#include <torch/library.h>

#include <map>
#include <mutex>
#include <utility>

#include "common/host.h"
#include "kernels/gemm_w8.h"
#include "kernels/launch.h"
#include "ops_ext.h"

namespace bwn {

using at::Tensor;

static inline const __nv_bfloat16* bf(const Tensor& t) {
  return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr());
}
static inline __nv_bfloat16* bfm(const Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "bwn: ", name, " must be a CUDA tensor");
}
void check_bf16(const Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, "bwn: ", name, " must be bfloat16, got ", t.scalar_type());
}
void check_f32(const Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kFloat, "bwn: ", name, " must be float32");
}
static void check_rowmajor(const Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, "bwn: ", name, " must be a 2-D row-major matrix (inner stride 1)");
}

// ---- per (device, stream) scratch for split-K / split-KV ------------------
static std::mutex g_scratch_mu;
static std::map<std::pair<int, cudaStream_t>, Scratch> g_scratch;

Scratch& scratch_for(const Tensor& like, long floats, long tickets) {
  const int dev = like.get_device();
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev).stream();
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  Scratch& s = g_scratch[{dev, st}];
  if (!s.ws.defined() || s.ws.numel() < floats) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    TORCH_CHECK(cs == cudaStreamCaptureStatusNone || !s.ws.defined(),
                "bwn: scratch must be sized before CUDA-graph capture (run the step once eagerly)");
    s.ws = at::empty({std::max<long>(floats, 1 << 20)}, like.options().dtype(at::kFloat));
  }
  if (!s.tickets.defined() || s.tickets.numel() < tickets) {
    s.tickets = at::zeros({std::max<long>(tickets, 4096)}, like.options().dtype(at::kInt));
  }
  return s;
}

// ---------------------------------------------------------------------------
// GEMM
// ---------------------------------------------------------------------------
static constexpr int kSwapMaxTokens = 256;  // tokens up to one 256-wide N tile: weights stream once

// out[M_tok, N_out] (+)= x[M_tok, K] . w[N_w, K]^T with the chosen epilogue.
void linear_into(const Tensor& x, const Tensor& w, const Tensor& out, int64_t epi, const c10::optional<Tensor>& resid) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_rowmajor(x, "x");
  check_rowmajor(w, "w");
  TORCH_CHECK(x.size(1) == w.size(1), "bwn.linear: K mismatch ", x.sizes(), " vs ", w.sizes());
  const c10::cuda::CUDAGuard guard(x.device());
  const int M = (int)x.size(0), Nw = (int)w.size(0), K = (int)x.size(1);
  if (M == 0) return;
  GemmProblem p;
  p.epi = (int)epi;
  p.status = status_dev_ptr();
  if (epi == kEpiF32) {
    check_f32(out, "out");
  } else {
    check_bf16(out, "out");
  }
  check_rowmajor(out, "out");
  if (epi == kEpiResid) {
    TORCH_CHECK(resid.has_value(), "bwn.linear: residual epilogue needs resid");
    check_bf16(*resid, "resid");
    check_rowmajor(*resid, "resid");
    p.resid = bf(*resid);
    p.ldr = resid->stride(0);
  }
  const bool swap = M <= kSwapMaxTokens;
  if (swap) {
    // weights drive the 128-row MMA M dimension; tokens are the N dimension
    p.A = w.data_ptr();
    p.lda = w.stride(0);
    p.B = x.data_ptr();
    p.ldb = x.stride(0);
    p.M = Nw;
    p.N = M;
    p.trans_out = true;
    if (epi == kEpiSwiGLU) TORCH_CHECK(Nw % 32 == 0, "bwn.linear_swiglu: gate/up rows must be a multiple of 32");
  } else {
    p.A = x.data_ptr();
    p.lda = x.stride(0);
    p.B = w.data_ptr();
    p.ldb = w.stride(0);
    p.M = M;
    p.N = Nw;
    p.trans_out = false;
    if (epi == kEpiSwiGLU) TORCH_CHECK(Nw % 32 == 0, "bwn.linear_swiglu: gate/up rows must be a multiple of 32");
  }
  p.K = K;
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  const int bn = gemm_pick_bn(p.N);
  p.bn = (epi == kEpiSwiGLU && !swap && bn < 32) ? 32 : bn;
  const int tiles = ((p.M + 127) / 128) * ((p.N + p.bn - 1) / p.bn);
  const int sms = num_sms();
  if (tiles < 2 * sms) {
    Scratch& s = scratch_for(x, 4L * sms * 128 * p.bn, 2 * sms);
    p.workspace = s.ws.data_ptr<float>();
    p.workspace_floats = s.ws.numel();
    p.tickets = s.tickets.data_ptr<int>();
    p.tickets_len = (int)s.tickets.numel();
  } else {
    p.allow_split = false;
  }
  gemm_bf16(p, at::cuda::getCurrentCUDAStream().stream());
}

// General (non-swapped) GEMM with optional MN-major operands:
//   a_mn=false: A is [M, K]; a_mn=true: A is stored [K, M]
//   b_mn=false: B is [N, K]; b_mn=true: B is stored [K, N]
// out[M, N] (bf16 or fp32 by out's dtype).
void gemm_into(const Tensor& A, bool a_mn, const Tensor& B, bool b_mn, const Tensor& out) {
  check_bf16(A, "A");
  check_bf16(B, "B");
  check_rowmajor(A, "A");
  check_rowmajor(B, "B");
  check_rowmajor(out, "out");
  const c10::cuda::CUDAGuard guard(A.device());
  const int M = (int)(a_mn ? A.size(1) : A.size(0));
  const int K = (int)(a_mn ? A.size(0) : A.size(1));
  const int N = (int)(b_mn ? B.size(1) : B.size(0));
  const int Kb = (int)(b_mn ? B.size(0) : B.size(1));
  TORCH_CHECK(K == Kb, "bwn.gemm: K mismatch");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "bwn.gemm: out shape");
  if (M == 0 || N == 0) return;
  GemmProblem p;
  p.A = A.data_ptr();
  p.lda = A.stride(0);
  p.B = B.data_ptr();
  p.ldb = B.stride(0);
  p.M = M;
  p.N = N;
  p.K = K;
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.status = status_dev_ptr();
  if (out.scalar_type() == at::kFloat) {
    p.epi = kEpiF32;
  } else {
    check_bf16(out, "out");
    p.epi = kEpiBF16;
  }
  int bn = gemm_pick_bn(N);
  if ((a_mn || b_mn) && bn < 64) bn = 64;
  p.bn = bn;
  const int tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
  const int sms = num_sms();
  if (tiles < 2 * sms) {
    Scratch& s = scratch_for(A, 4L * sms * 128 * bn, 2 * sms);
    p.workspace = s.ws.data_ptr<float>();
    p.workspace_floats = s.ws.numel();
    p.tickets = s.tickets.data_ptr<int>();
    p.tickets_len = (int)s.tickets.numel();
  } else {
    p.allow_split = false;
  }
  gemm_bf16(p, at::cuda::getCurrentCUDAStream().stream());
}

Tensor linear_kn(const Tensor& x, const Tensor& w_kn) {
  auto out = at::empty({x.size(0), w_kn.size(1)}, x.options());
  gemm_into(x, false, w_kn, true, out);
  return out;
}

Tensor matmul_tn(const Tensor& a_km, const Tensor& b_kn, bool f32_out) {
  auto out = at::empty({a_km.size(1), b_kn.size(1)}, a_km.options().dtype(f32_out ? at::kFloat : at::kBFloat16));
  gemm_into(a_km, true, b_kn, true, out);
  return out;
}

// FP8 W8A16: out[T, N] = x[T, K] . dequant(w8[N, K], scales[N/128, K/128])^T
void linear_w8_into(const Tensor& x, const Tensor& w8, const Tensor& scales, const Tensor& out, int64_t epi,
                    const c10::optional<Tensor>& resid) {
  check_bf16(x, "x");
  check_rowmajor(x, "x");
  check_cuda(w8, "w8");
  TORCH_CHECK(w8.element_size() == 1 && w8.dim() == 2 && w8.stride(1) == 1, "w8 must be a [N, K] 8-bit matrix");
  check_f32(scales, "scales");
  TORCH_CHECK(scales.dim() == 2 && scales.is_contiguous(), "scales [N/128, K/128]");
  TORCH_CHECK(x.size(1) == w8.size(1), "linear_w8: K mismatch");
  TORCH_CHECK(scales.size(0) == (w8.size(0) + 127) / 128 && scales.size(1) == (w8.size(1) + 127) / 128,
              "linear_w8: scales must be [ceil(N/128), ceil(K/128)]");
  const c10::cuda::CUDAGuard guard(x.device());
  const int T = (int)x.size(0), N = (int)w8.size(0), K = (int)x.size(1);
  if (T == 0) return;
  GemmW8Problem p;
  p.A = w8.data_ptr();
  p.lda = w8.stride(0);
  p.scales = scales.data_ptr<float>();
  p.lds = (int)scales.size(1);
  p.B = x.data_ptr();
  p.ldb = x.stride(0);
  p.M = N;
  p.N = T;
  p.K = K;
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.epi = (int)epi;
  p.status = status_dev_ptr();
  if (epi == kEpiResid) {
    TORCH_CHECK(resid.has_value(), "linear_w8: residual epilogue needs resid");
    p.resid = bf(*resid);
    p.ldr = resid->stride(0);
  }
  const int sms = num_sms();
  Scratch& s = scratch_for(x, 4L * sms * 128 * 128, 2 * sms);
  p.workspace = s.ws.data_ptr<float>();
  p.workspace_floats = s.ws.numel();
  p.tickets = s.tickets.data_ptr<int>();
  p.tickets_len = (int)s.tickets.numel();
  gemm_w8(p, at::cuda::getCurrentCUDAStream().stream());
}

Tensor linear_w8(const Tensor& x, const Tensor& w8, const Tensor& scales, int64_t epi,
                 const c10::optional<Tensor>& resid) {
  const int64_t N = epi == kEpiSwiGLU ? w8.size(0) / 2 : w8.size(0);
  auto out = at::empty({x.size(0), N}, x.options().dtype(epi == kEpiF32 ? at::kFloat : at::kBFloat16));
  linear_w8_into(x, w8, scales, out, epi, resid);
  return out;
}

Tensor linear(const Tensor& x, const Tensor& w) {
  auto out = at::empty({x.size(0), w.size(0)}, x.options());
  linear_into(x, w, out, kEpiBF16, c10::nullopt);
  return out;
}

Tensor linear_f32(const Tensor& x, const Tensor& w) {
  auto out = at::empty({x.size(0), w.size(0)}, x.options().dtype(at::kFloat));
  linear_into(x, w, out, kEpiF32, c10::nullopt);
  return out;
}

Tensor linear_swiglu(const Tensor& x, const Tensor& w_il) {
  auto out = at::empty({x.size(0), w_il.size(0) / 2}, x.options());
  linear_into(x, w_il, out, kEpiSwiGLU, c10::nullopt);
  return out;
}

Tensor linear_residual(const Tensor& x, const Tensor& w, const Tensor& resid) {
  auto out = at::empty({x.size(0), w.size(0)}, x.options());
  linear_into(x, w, out, kEpiResid, resid);
  return out;
}

void linear_out(const Tensor& x, const Tensor& w, Tensor out, int64_t epi, const c10::optional<Tensor>& resid) {
  linear_into(x, w, out, epi, resid);
}

// ---------------------------------------------------------------------------
// norms / embedding / greedy
// ---------------------------------------------------------------------------
Tensor rms_norm_op(const Tensor& x, const Tensor& w, double eps, bool one_plus) {
  check_bf16(x, "x");
  check_f32(w, "w");
  const c10::cuda::CUDAGuard guard(x.device());
  auto x2 = x.reshape({-1, x.size(-1)});
  TORCH_CHECK(x2.stride(-1) == 1, "rms_norm: inner stride must be 1");
  auto out = at::empty_like(x2, x2.options().memory_format(at::MemoryFormat::Contiguous));
  rms_norm(bf(x2), x2.stride(0), w.data_ptr<float>(), bfm(out), out.stride(0), (int)x2.size(0), (int)x2.size(1),
           (float)eps, one_plus, at::cuda::getCurrentCUDAStream().stream());
  return out.view(x.sizes());
}

Tensor add_rms_norm_op(const Tensor& x, Tensor residual, const Tensor& w, double eps) {
  check_bf16(x, "x");
  check_bf16(residual, "residual");
  check_f32(w, "w");
  check_rowmajor(x, "x");
  check_rowmajor(residual, "residual");
  const c10::cuda::CUDAGuard guard(x.device());
  auto out = at::empty({x.size(0), x.size(1)}, x.options());
  add_rms_norm(bf(x), x.stride(0), bfm(residual), residual.stride(0), w.data_ptr<float>(), bfm(out), out.stride(0),
               (int)x.size(0), (int)x.size(1), (float)eps, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

Tensor embedding_op(const Tensor& ids, const Tensor& table, int64_t offset) {
  check_cuda(ids, "ids");
  TORCH_CHECK(ids.scalar_type() == at::kInt, "embedding: ids must be int32");
  check_bf16(table, "table");
  const c10::cuda::CUDAGuard guard(ids.device());
  auto idc = ids.contiguous();
  auto out = at::empty({idc.numel(), table.size(1)}, table.options());
  embedding(idc.data_ptr<int>(), (int)idc.numel(), bf(table), table.size(0), (int)table.size(1), offset, bfm(out),
            at::cuda::getCurrentCUDAStream().stream());
  return out;
}

Tensor argmax_packed_op(const Tensor& logits, int64_t id_offset) {
  check_cuda(logits, "logits");
  check_rowmajor(logits, "logits");
  const c10::cuda::CUDAGuard guard(logits.device());
  auto out = at::empty({logits.size(0)}, logits.options().dtype(at::kLong));
  auto st = at::cuda::getCurrentCUDAStream().stream();
  if (logits.scalar_type() == at::kFloat)
    argmax_packed(logits.data_ptr<float>(), logits.stride(0), (int)logits.size(0), (int)logits.size(1), id_offset,
                  out.data_ptr<int64_t>(), st);
  else if (logits.scalar_type() == at::kBFloat16)
    argmax_packed_bf16(bf(logits), logits.stride(0), (int)logits.size(0), (int)logits.size(1), id_offset,
                       out.data_ptr<int64_t>(), st);
  else
    TORCH_CHECK(false, "argmax_packed: logits must be fp32 or bf16");
  return out;
}

Tensor unpack_argmax_op(const Tensor& packed) {
  check_cuda(packed, "packed");
  const c10::cuda::CUDAGuard guard(packed.device());
  auto out = at::empty({packed.numel()}, packed.options().dtype(at::kInt));
  unpack_argmax(packed.data_ptr<int64_t>(), (int)packed.numel(), out.data_ptr<int>(),
                at::cuda::getCurrentCUDAStream().stream());
  return out;
}

// ---------------------------------------------------------------------------
// DeltaNet / GQA decode
// ---------------------------------------------------------------------------
Tensor deltanet_decode_op(const Tensor& qkv, const Tensor& z, const Tensor& a, const Tensor& b, Tensor conv_ring,
                          Tensor state, const Tensor& positions, const Tensor& conv_w, const Tensor& A_log,
                          const Tensor& dt_bias, const Tensor& norm_w, int64_t k_heads, double eps) {
  check_bf16(qkv, "qkv");
  check_bf16(z, "z");
  check_bf16(a, "a");
  check_bf16(b, "b");
  check_bf16(conv_ring, "conv_ring");
  check_f32(conv_w, "conv_w");
  check_f32(A_log, "A_log");
  check_f32(dt_bias, "dt_bias");
  check_f32(norm_w, "norm_w");
  TORCH_CHECK(positions.scalar_type() == at::kInt && positions.is_contiguous(), "positions must be int32 contiguous");
  TORCH_CHECK(state.is_contiguous() && conv_ring.is_contiguous() && conv_w.is_contiguous(), "state/ring contiguous");
  TORCH_CHECK(state.dim() == 4 && state.size(2) == 128 && state.size(3) == 128, "state must be [B, VH, 128, 128]");
  TORCH_CHECK(state.scalar_type() == at::kFloat || state.scalar_type() == at::kBFloat16, "state fp32/bf16");
  const int B = (int)qkv.size(0), VH = (int)state.size(1);
  const int C = (int)qkv.size(1);
  TORCH_CHECK(C == 2 * k_heads * 128 + VH * 128, "qkv width mismatch");
  TORCH_CHECK(conv_ring.size(0) == B && (conv_ring.size(1) == 4 || conv_ring.size(1) == 8) && conv_ring.size(2) == C,
              "conv_ring [B, 4 or 8, C]");
  TORCH_CHECK(qkv.stride(1) == 1 && z.stride(1) == 1 && a.stride(1) == 1 && b.stride(1) == 1, "inner stride 1");
  TORCH_CHECK(a.stride(0) == b.stride(0), "a and b must share a row stride");
  const c10::cuda::CUDAGuard guard(qkv.device());
  auto out = at::empty({B, VH * 128}, qkv.options());
  DeltaNetDecodeArgs p{};
  p.qkv = bf(qkv);
  p.qkv_stride = qkv.stride(0);
  p.z = bf(z);
  p.z_stride = z.stride(0);
  p.a = bf(a);
  p.b = bf(b);
  p.ab_stride = a.stride(0);
  p.conv_ring = bfm(conv_ring);
  p.ring_slots = (int)conv_ring.size(1);
  p.state = state.data_ptr();
  p.state_bf16 = state.scalar_type() == at::kBFloat16;
  p.positions = positions.data_ptr<int>();
  p.conv_w = conv_w.data_ptr<float>();
  p.A_log = A_log.data_ptr<float>();
  p.dt_bias = dt_bias.data_ptr<float>();
  p.norm_w = norm_w.data_ptr<float>();
  p.out = bfm(out);
  p.out_stride = out.stride(0);
  p.batch = B;
  p.k_heads = (int)k_heads;
  p.v_heads = VH;
  p.l2_eps = 1e-6f;
  p.norm_eps = (float)eps;
  deltanet_decode(p, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

Tensor gqa_decode_op(const Tensor& qg, const Tensor& k_new, const Tensor& v_new, const Tensor& q_norm_w,
                     const Tensor& k_norm_w, const Tensor& cos, const Tensor& sin, Tensor k_cache, Tensor v_cache,
                     const Tensor& positions, double eps, int64_t splits, int64_t n_tok) {
  check_bf16(qg, "qg");
  check_bf16(k_new, "k_new");
  check_bf16(v_new, "v_new");
  check_bf16(k_cache, "k_cache");
  check_bf16(v_cache, "v_cache");
  check_f32(q_norm_w, "q_norm_w");
  check_f32(k_norm_w, "k_norm_w");
  check_f32(cos, "cos");
  check_f32(sin, "sin");
  TORCH_CHECK(positions.scalar_type() == at::kInt && positions.is_contiguous(), "positions int32");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(3) == 256 && k_cache.is_contiguous() && v_cache.is_contiguous(),
              "caches must be contiguous [B, KVH, S_max, 256]");
  TORCH_CHECK(n_tok >= 1 && n_tok <= 16, "n_tok in [1, 16]");
  const int KVH = (int)k_cache.size(1), S = (int)k_cache.size(2);
  const int B = (int)(k_cache.size(0) * n_tok);  // query rows
  TORCH_CHECK(qg.dim() == 3 && qg.size(0) == B && qg.size(2) == 512 && qg.stride(2) == 1 && qg.stride(1) == 512,
              "qg [B * n_tok, QH, 512]");
  TORCH_CHECK(positions.numel() == B, "positions: one per query row");
  TORCH_CHECK(k_new.dim() == 3 && k_new.stride(2) == 1 && k_new.stride(1) == 256, "k_new [B, KVH, 256]");
  TORCH_CHECK(v_new.stride(0) == k_new.stride(0), "k_new and v_new must share a row stride");
  const int QH = (int)qg.size(1);
  const c10::cuda::CUDAGuard guard(qg.device());
  auto out = at::empty({B, QH * 256}, qg.options());
  if (splits <= 0) {
    const int sms = num_sms();
    splits = std::max<int64_t>(1, std::min<int64_t>(64, (2 * sms + B * KVH - 1) / (B * KVH)));
    splits = std::min<int64_t>(splits, (S + 63) / 64);
  }
  Scratch& s = scratch_for(qg, gqa_decode_workspace_floats(B, QH, KVH, (int)splits) + (long)num_sms() * 128 * 256,
                           std::max(B * KVH, num_sms()));
  GqaDecodeArgs p{};
  p.qg = bf(qg);
  p.qg_stride = qg.stride(0);
  p.k_new = bf(k_new);
  p.v_new = bf(v_new);
  p.kv_new_stride = k_new.stride(0);
  p.q_norm_w = q_norm_w.data_ptr<float>();
  p.k_norm_w = k_norm_w.data_ptr<float>();
  p.cos = cos.data_ptr<float>();
  p.sin = sin.data_ptr<float>();
  p.k_cache = bfm(k_cache);
  p.v_cache = bfm(v_cache);
  p.positions = positions.data_ptr<int>();
  p.out = bfm(out);
  p.out_stride = out.stride(0);
  p.workspace = s.ws.data_ptr<float>();
  p.tickets = s.tickets.data_ptr<int>();
  p.status = status_dev_ptr();
  p.batch = B;
  p.q_heads = QH;
  p.kv_heads = KVH;
  p.s_max = S;
  p.rope_dim = (int)cos.size(1);
  p.splits = (int)splits;
  p.eps = (float)eps;
  p.n_tok = (int)n_tok;
  gqa_decode(p, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

int64_t status_op() { return status_read(); }
void status_clear_op() { status_clear(); }
int64_t num_sms_op() { return num_sms(); }

}  // namespace bwn

TORCH_LIBRARY(bwn, m) {
  m.def("linear(Tensor x, Tensor w) -> Tensor");
  m.def("linear_f32(Tensor x, Tensor w) -> Tensor");
  m.def("linear_swiglu(Tensor x, Tensor w_il) -> Tensor");
  m.def("linear_residual(Tensor x, Tensor w, Tensor resid) -> Tensor");
  m.def("linear_out(Tensor x, Tensor w, Tensor(a!) out, int epi, Tensor? resid) -> ()");
  m.def("linear_kn(Tensor x, Tensor w_kn) -> Tensor");
  m.def("linear_w8(Tensor x, Tensor w8, Tensor scales, int epi, Tensor? resid) -> Tensor");
  m.def("matmul_tn(Tensor a_km, Tensor b_kn, bool f32_out) -> Tensor");
  m.def("rms_norm(Tensor x, Tensor w, float eps, bool one_plus) -> Tensor");
  m.def("add_rms_norm(Tensor x, Tensor(a!) residual, Tensor w, float eps) -> Tensor");
  m.def("embedding(Tensor ids, Tensor table, int offset) -> Tensor");
  m.def("argmax_packed(Tensor logits, int id_offset) -> Tensor");
  m.def("unpack_argmax(Tensor packed) -> Tensor");
  m.def(
      "deltanet_decode(Tensor qkv, Tensor z, Tensor a, Tensor b, Tensor(a!) conv_ring, Tensor(b!) state, "
      "Tensor positions, Tensor conv_w, Tensor A_log, Tensor dt_bias, Tensor norm_w, int k_heads, float eps) -> Tensor");
  m.def(
      "gqa_decode(Tensor qg, Tensor k_new, Tensor v_new, Tensor q_norm_w, Tensor k_norm_w, Tensor cos, Tensor sin, "
      "Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor positions, float eps, int splits, int n_tok=1) -> Tensor");
  bwn::register_ext_defs(m);
}

TORCH_LIBRARY_IMPL(bwn, CUDA, m) {
  m.impl("linear", &bwn::linear);
  m.impl("linear_f32", &bwn::linear_f32);
  m.impl("linear_swiglu", &bwn::linear_swiglu);
  m.impl("linear_residual", &bwn::linear_residual);
  m.impl("linear_out", &bwn::linear_out);
  m.impl("linear_kn", &bwn::linear_kn);
  m.impl("linear_w8", &bwn::linear_w8);
  m.impl("matmul_tn", &bwn::matmul_tn);
  m.impl("rms_norm", &bwn::rms_norm_op);
  m.impl("add_rms_norm", &bwn::add_rms_norm_op);
  m.impl("embedding", &bwn::embedding_op);
  m.impl("argmax_packed", &bwn::argmax_packed_op);
  m.impl("unpack_argmax", &bwn::unpack_argmax_op);
  m.impl("deltanet_decode", &bwn::deltanet_decode_op);
  m.impl("gqa_decode", &bwn::gqa_decode_op);
  bwn::register_ext_impls(m);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, mod) {
  mod.def("status", &bwn::status_op, "read the device error-status word of the current device");
  mod.def("status_clear", &bwn::status_clear_op, "clear the device error-status word");
  mod.def("num_sms", &bwn::num_sms_op, "SM count of the current device");
  bwn::register_ext_pybind(mod);
}
