// torch.ops.bwn registrations of the fused NVLink collectives.  Buffer
// addresses (symmetric peer pointers, the NVLS multicast address) come from the
// Python side as integers; this file only validates and launches.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>
#include <torch/library.h>

#include "comm/ep.h"
#include "comm/fused.h"
#include "comm/grad_reduce.h"
#include "common/host.h"
#include "kernels/moe.h"
#include "ops_ext.h"

namespace bwn {
using at::Tensor;

// local_state int32 layout: [0] AR epoch, [1] AR grid ticket, [2] buffer selector,
// [3] norm-kernel ticket, [4] greedy epoch
static CommSignal make_sig(const std::vector<int64_t>& peer_flags, const Tensor& local_state, int64_t rank,
                           int64_t buf_stride) {
  TORCH_CHECK(local_state.scalar_type() == at::kInt && local_state.numel() >= 8, "local_state int32[8+]");
  TORCH_CHECK(peer_flags.size() >= 1 && peer_flags.size() <= 8, "1..8 ranks");
  CommSignal s;
  s.world = (int)peer_flags.size();
  s.rank = (int)rank;
  for (size_t i = 0; i < peer_flags.size(); ++i) s.peer_flags[i] = reinterpret_cast<unsigned*>(peer_flags[i]);
  int* ls = local_state.data_ptr<int>();
  s.epoch = ls + 0;
  s.done_ticket = ls + 1;
  s.sel = ls + 2;
  s.buf_stride = buf_stride;
  return s;
}

// Row-parallel GEMM whose epilogue stores the bf16 partial into this rank's
// symmetric slot and publishes the completion flag to every rank.
static GemmProblem symm_gemm_problem(const Tensor& x, const Tensor& w, int64_t local_base, int64_t buf_stride,
                                     int64_t ldo, const std::vector<int64_t>& peer_flags, const Tensor& local_state,
                                     int64_t rank) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && w.dim() == 2 && w.stride(1) == 1, "row-major x, w");
  const int M = (int)x.size(0), Nw = (int)w.size(0), K = (int)x.size(1);
  GemmProblem p;
  p.epi = kEpiSymm;
  p.status = status_dev_ptr();
  const bool swap = M <= 256;
  if (swap) {
    p.A = w.data_ptr();
    p.lda = w.stride(0);
    p.B = x.data_ptr();
    p.ldb = x.stride(0);
    p.M = Nw;
    p.N = M;
    p.trans_out = true;
  } else {
    p.A = x.data_ptr();
    p.lda = x.stride(0);
    p.B = w.data_ptr();
    p.ldb = w.stride(0);
    p.M = M;
    p.N = Nw;
  }
  p.K = K;
  p.out = reinterpret_cast<void*>(local_base);
  p.ldo = ldo;
  p.sig = make_sig(peer_flags, local_state, rank, buf_stride);
  const int bn = gemm_pick_bn(p.N);
  const int tiles = ((p.M + 127) / 128) * ((p.N + bn - 1) / bn);
  const int sms = num_sms();
  if (tiles < 2 * sms) {
    Scratch& s = scratch_for(x, 4L * sms * 128 * bn, 2 * sms);
    p.workspace = s.ws.data_ptr<float>();
    p.workspace_floats = s.ws.numel();
    p.tickets = s.tickets.data_ptr<int>();
    p.tickets_len = (int)s.tickets.numel();
  }
  return p;
}

void gemm_symm_op(const Tensor& x, const Tensor& w, int64_t local_base, int64_t buf_stride, int64_t ldo,
                  std::vector<int64_t> peer_flags, const Tensor& local_state, int64_t rank) {
  const c10::cuda::CUDAGuard guard(x.device());
  GemmProblem p = symm_gemm_problem(x, w, local_base, buf_stride, ldo, peer_flags, local_state, rank);
  gemm_bf16(p, at::cuda::getCurrentCUDAStream().stream());
}

// F1 in one launch: the row-parallel GEMM stores its partial into this rank's
// symmetric slot and signals; the same CTAs then wait for every rank, read the
// sum through the multicast address, add the residual (in place) and return
// RMSNorm(residual) * (1 + norm_w).
Tensor gemm_symm_norm_op(const Tensor& x, const Tensor& w, int64_t local_base, int64_t mc_base, int64_t buf_stride,
                         std::vector<int64_t> peer_flags, int64_t flags_local, const Tensor& local_state,
                         int64_t rank, Tensor residual, const Tensor& norm_w, double eps, double timeout_s) {
  check_bf16(residual, "residual");
  check_f32(norm_w, "norm_w");
  TORCH_CHECK(residual.dim() == 2 && residual.stride(1) == 1 && residual.size(0) == x.size(0) &&
                  residual.size(1) == w.size(0) && norm_w.numel() == w.size(0),
              "residual [rows, H] with H = w.size(0)");
  const c10::cuda::CUDAGuard guard(x.device());
  GemmProblem p = symm_gemm_problem(x, w, local_base, buf_stride, w.size(0), peer_flags, local_state, rank);
  auto out = at::empty({residual.size(0), residual.size(1)}, residual.options());
  p.epi = kEpiSymmNorm;
  p.tail.mc_base = reinterpret_cast<const __nv_bfloat16*>(mc_base);
  p.tail.flags = reinterpret_cast<const unsigned*>(flags_local);
  p.tail.sel = local_state.data_ptr<int>() + 2;
  p.tail.resid = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  p.tail.ldr = residual.stride(0);
  p.tail.w = norm_w.data_ptr<float>();
  p.tail.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.tail.ldo = out.stride(0);
  p.tail.rows = (int)residual.size(0);
  p.tail.cols = (int)residual.size(1);
  p.tail.eps = (float)eps;
  p.tail.limit_ns = (unsigned long long)(timeout_s * 1e9);
  gemm_bf16(p, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

void symm_put_signal_op(const Tensor& x, int64_t local_base, int64_t buf_stride, std::vector<int64_t> peer_flags,
                        const Tensor& local_state, int64_t rank) {
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x [rows, cols]");
  const c10::cuda::CUDAGuard guard(x.device());
  symm_put_signal(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), (int)x.size(0), (int)x.size(1),
                  reinterpret_cast<__nv_bfloat16*>(local_base), make_sig(peer_flags, local_state, rank, buf_stride),
                  at::cuda::getCurrentCUDAStream().stream());
}

// MoE combine (routed + shared expert rows, fp32, rounded to bf16 once)
// straight into this rank's symmetric slot, with the completion flag published:
// the combine and symm_put_signal in one launch; ar_add_norm follows.
void moe_combine_symm_op(const Tensor& y, const Tensor& w, const Tensor& pos_of, const c10::optional<Tensor>& pos_sh,
                         const c10::optional<Tensor>& sg, const c10::optional<Tensor>& shared_y,
                         const c10::optional<Tensor>& shared_gate, int64_t local_base, int64_t buf_stride,
                         std::vector<int64_t> peer_flags, const Tensor& local_state, int64_t rank) {
  const c10::cuda::CUDAGuard guard(y.device());
  MoeCombineExArgs c = combine_args(y, w, pos_of, pos_sh, sg, shared_y, shared_gate);
  c.mode = kCombineSymm;
  c.symm_base = reinterpret_cast<__nv_bfloat16*>(local_base);
  c.sig = make_sig(peer_flags, local_state, rank, buf_stride);
  moe_combine_ex(c, at::cuda::getCurrentCUDAStream().stream());
}

// The same combine, then (same launch) the sum over ranks through the multicast
// address + residual add (in place) + RMSNorm(1+w): the MoE sub-block's
// expert-parallel reduction in one kernel.  Returns the normed rows.
Tensor moe_combine_symm_norm_op(const Tensor& y, const Tensor& w, const Tensor& pos_of,
                                const c10::optional<Tensor>& pos_sh, const c10::optional<Tensor>& sg,
                                const c10::optional<Tensor>& shared_y, const c10::optional<Tensor>& shared_gate,
                                int64_t local_base, int64_t mc_base, int64_t buf_stride, std::vector<int64_t> peer_flags,
                                int64_t flags_local, const Tensor& local_state, int64_t rank, Tensor residual,
                                const Tensor& norm_w, double eps, double timeout_s) {
  check_bf16(residual, "residual");
  check_f32(norm_w, "norm_w");
  const c10::cuda::CUDAGuard guard(y.device());
  MoeCombineExArgs c = combine_args(y, w, pos_of, pos_sh, sg, shared_y, shared_gate);
  TORCH_CHECK(residual.dim() == 2 && residual.stride(1) == 1 && residual.size(0) == c.T && residual.size(1) == c.H,
              "residual [T, H]");
  auto out = at::empty({c.T, c.H}, residual.options());
  c.mode = kCombineSymmNorm;
  c.symm_base = reinterpret_cast<__nv_bfloat16*>(local_base);
  c.sig = make_sig(peer_flags, local_state, rank, buf_stride);
  c.mc_base = reinterpret_cast<const __nv_bfloat16*>(mc_base);
  c.flags = reinterpret_cast<const unsigned*>(flags_local);
  c.sel_rw = local_state.data_ptr<int>() + 2;
  c.status = status_dev_ptr();
  c.limit_ns = (unsigned long long)(timeout_s * 1e9);
  c.resid = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  c.ldr = residual.stride(0);
  c.norm_w = norm_w.data_ptr<float>();
  c.eps = (float)eps;
  c.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  c.ldo = out.stride(0);
  moe_combine_ex(c, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

Tensor ar_add_norm_op(int64_t mc_base, int64_t buf_stride, int64_t flags_local, int64_t world,
                      const Tensor& local_state, Tensor residual, const Tensor& w, double eps, double timeout_s) {
  check_bf16(residual, "residual");
  check_f32(w, "w");
  TORCH_CHECK(residual.dim() == 2 && residual.stride(1) == 1, "residual [rows, H]");
  const c10::cuda::CUDAGuard guard(residual.device());
  auto out = at::empty_like(residual, residual.options().memory_format(at::MemoryFormat::Contiguous));
  ArNormArgs a{};
  a.mc_base = reinterpret_cast<const __nv_bfloat16*>(mc_base);
  a.buf_stride = buf_stride;
  int* ls = local_state.data_ptr<int>();
  a.sel = ls + 2;
  a.flags = reinterpret_cast<const unsigned*>(flags_local);
  a.world = (int)world;
  a.epoch = ls + 0;
  a.resid = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  a.ldr = residual.stride(0);
  a.w = w.data_ptr<float>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ldo = out.stride(0);
  a.rows = (int)residual.size(0);
  a.cols = (int)residual.size(1);
  a.eps = (float)eps;
  a.status = status_dev_ptr();
  a.limit_ns = (unsigned long long)(timeout_s * 1e9);
  if (a.rows > 0) ar_add_norm(a, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

Tensor ar_hc_post_op(int64_t mc_base, int64_t buf_stride, int64_t flags_local, int64_t world,
                     const Tensor& local_state, const Tensor& resid, const Tensor& post, const Tensor& comb,
                     double timeout_s) {
  check_bf16(resid, "resid");
  check_f32(post, "post");
  check_f32(comb, "comb");
  TORCH_CHECK(resid.dim() == 3 && resid.is_contiguous(), "resid [rows, hc, cols] contiguous");
  const int64_t rows = resid.size(0), hc = resid.size(1);
  TORCH_CHECK(post.is_contiguous() && post.numel() == rows * hc, "post [rows, hc]");
  TORCH_CHECK(comb.is_contiguous() && comb.numel() == rows * hc * hc, "comb [rows, hc, hc]");
  const c10::cuda::CUDAGuard guard(resid.device());
  auto out = at::empty_like(resid);
  ArHcArgs a{};
  a.mc_base = reinterpret_cast<const __nv_bfloat16*>(mc_base);
  a.buf_stride = buf_stride;
  int* ls = local_state.data_ptr<int>();
  a.sel = ls + 2;
  a.flags = reinterpret_cast<const unsigned*>(flags_local);
  a.world = (int)world;
  a.epoch = ls + 0;
  a.resid = reinterpret_cast<const __nv_bfloat16*>(resid.data_ptr());
  a.post = post.data_ptr<float>();
  a.comb = comb.data_ptr<float>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.rows = (int)rows;
  a.cols = (int)resid.size(2);
  a.hc = (int)hc;
  a.status = status_dev_ptr();
  a.limit_ns = (unsigned long long)(timeout_s * 1e9);
  if (a.rows > 0) ar_hc_post(a, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

Tensor greedy_allmax_op(const Tensor& keys, std::vector<int64_t> peer_slots, std::vector<int64_t> peer_flags,
                        int64_t flags_local, const Tensor& local_state, int64_t rank, double timeout_s) {
  check_cuda(keys, "keys");
  TORCH_CHECK(keys.scalar_type() == at::kLong && keys.is_contiguous(), "keys int64");
  TORCH_CHECK(peer_slots.size() == peer_flags.size() && peer_slots.size() <= 8, "peer arrays");
  const c10::cuda::CUDAGuard guard(keys.device());
  auto ids = at::empty({keys.numel()}, keys.options().dtype(at::kInt));
  GreedyArgs a{};
  a.keys = keys.data_ptr<int64_t>();
  a.rows = (int)keys.numel();
  for (size_t i = 0; i < peer_slots.size(); ++i) {
    a.peer_slots[i] = reinterpret_cast<int64_t*>(peer_slots[i]);
    a.peer_flags[i] = reinterpret_cast<unsigned*>(peer_flags[i]);
  }
  a.flags = reinterpret_cast<const unsigned*>(flags_local);
  a.world = (int)peer_slots.size();
  a.rank = (int)rank;
  a.epoch = local_state.data_ptr<int>() + 4;
  a.ids_out = ids.data_ptr<int>();
  a.status = status_dev_ptr();
  a.limit_ns = (unsigned long long)(timeout_s * 1e9);
  greedy_allmax(a, at::cuda::getCurrentCUDAStream().stream());
  return ids;
}

// ---- expert-parallel all-to-all -------------------------------------------
// Symmetric buffer layout (byte offsets, identical on every rank):
//   [flags 3*8 u32][table W*W*E_l i32][recv tags max_recv*4 i32][recv rows max_recv*H bf16][comb T_max*k*H bf16]
static std::vector<int64_t> ep_layout(int64_t world, int64_t e_local, int64_t H, int64_t k, int64_t T_max,
                                      int64_t max_recv) {
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  std::vector<int64_t> off(6);
  off[0] = 0;
  off[1] = up(3 * kEpMaxRanks * 4);
  off[2] = off[1] + up(world * world * e_local * 4);
  off[3] = off[2] + up(max_recv * 16);
  off[4] = off[3] + up(max_recv * H * 2);
  off[5] = off[4] + up(T_max * k * H * 2);  // total bytes
  return off;
}
std::vector<int64_t> ep_layout_op(int64_t world, int64_t e_local, int64_t H, int64_t k, int64_t T_max,
                                  int64_t max_recv) {
  return ep_layout(world, e_local, H, k, T_max, max_recv);
}

// ep_state int32 layout: [0..2] epochs, [3..4] tickets, [5..7] wait outcomes, then recv counts [E_l],
// recv offsets [E_l+1], send slots [W*E_l]
static EpArgs make_ep(const std::vector<int64_t>& peer_base, int64_t rank, int64_t e_local, int64_t H, int64_t k,
                      int64_t T_max, int64_t max_recv, const Tensor& state, double timeout_s) {
  const int W = (int)peer_base.size();
  TORCH_CHECK(W >= 1 && W <= kEpMaxRanks, "ep: 1..8 ranks");
  TORCH_CHECK(state.scalar_type() == at::kInt && state.is_contiguous() &&
                  state.numel() >= 16 + 2 * e_local + 1 + W * e_local,
              "ep: state int32[16 + 2*E_l + 1 + W*E_l]");
  const auto off = ep_layout(W, e_local, H, k, T_max, max_recv);
  EpArgs a{};
  a.world = W;
  a.rank = (int)rank;
  a.e_local = (int)e_local;
  a.H = (int)H;
  a.k = (int)k;
  a.T_max = (int)T_max;
  a.max_recv = (int)max_recv;
  for (int r = 0; r < W; ++r) {
    char* b = reinterpret_cast<char*>(peer_base[r]);
    a.peer_flags[r] = reinterpret_cast<unsigned*>(b + off[0]);
    a.peer_table[r] = reinterpret_cast<int*>(b + off[1]);
    a.peer_recv_tag[r] = reinterpret_cast<int*>(b + off[2]);
    a.peer_recv_x[r] = reinterpret_cast<__nv_bfloat16*>(b + off[3]);
    a.peer_comb[r] = reinterpret_cast<__nv_bfloat16*>(b + off[4]);
  }
  a.flags = a.peer_flags[rank];
  a.table = a.peer_table[rank];
  a.recv_tag = a.peer_recv_tag[rank];
  int* s = state.data_ptr<int>();
  a.epoch_a = s + 0;
  a.epoch_b = s + 1;
  a.epoch_c = s + 2;
  a.ticket_b = s + 3;
  a.ticket_c = s + 4;
  a.ok = s + 5;  // [5..7]
  a.recv_counts = s + 16;
  a.recv_offsets = s + 16 + e_local;
  a.send_ctr = s + 16 + 2 * e_local + 1;
  a.status = status_dev_ptr();
  a.limit_ns = (unsigned long long)(timeout_s * 1e9);
  return a;
}

// Dispatch: counts all-gather, row sends, wait for every source's rows.
void ep_dispatch_op(const Tensor& x, const Tensor& ids, std::vector<int64_t> peer_base, int64_t rank, int64_t e_local,
                    int64_t T_max, int64_t max_recv, Tensor state, double timeout_s) {
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.stride(0) % 8 == 0, "x [T, H] with 16-byte rows");
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous() && ids.dim() == 2 && ids.size(0) == x.size(0),
              "ids int32 [T, k]");
  TORCH_CHECK(x.size(0) <= T_max, "ep_dispatch: more tokens than T_max");
  const c10::cuda::CUDAGuard guard(x.device());
  EpArgs a = make_ep(peer_base, rank, e_local, x.size(1), ids.size(1), T_max, max_recv, state, timeout_s);
  a.T = (int)x.size(0);
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.ldx = x.stride(0);
  a.ids = ids.data_ptr<int>();
  auto st = at::cuda::getCurrentCUDAStream().stream();
  ep_count(a, st);
  ep_send(a, st);
  ep_wait(a, 0, st);
}

// Return: every received row's expert output back to its source; wait for ours.
void ep_return_op(const Tensor& y, std::vector<int64_t> peer_base, int64_t rank, int64_t e_local, int64_t k,
                  int64_t T, int64_t T_max, int64_t max_recv, Tensor state, double timeout_s) {
  check_bf16(y, "y");
  TORCH_CHECK(y.dim() == 2 && y.stride(1) == 1 && y.size(0) >= max_recv && y.stride(0) % 8 == 0, "y [max_recv, H]");
  const c10::cuda::CUDAGuard guard(y.device());
  EpArgs a = make_ep(peer_base, rank, e_local, y.size(1), k, T_max, max_recv, state, timeout_s);
  a.T = (int)T;
  a.y = reinterpret_cast<const __nv_bfloat16*>(y.data_ptr());
  a.ldy = y.stride(0);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  ep_return(a, st);
  ep_wait(a, 1, st);
}

// ---- sequence parallelism: reduce-scatter + norm + all-gather, all-gather -> GEMM
// sp state int32: [0] partial epoch, [1] GEMM done ticket, [2] slot selector,
// [3] unused, [4] gather epoch, [5] gather ticket
void sp_norm_gather_op(int64_t mc_partial, const c10::optional<Tensor>& local_partial, int64_t buf_stride,
                       int64_t flags_local, int64_t world, int64_t rank, Tensor state, Tensor x, const Tensor& w,
                       double eps, int64_t h_mc, std::vector<int64_t> ag_peer_flags, double timeout_s) {
  check_bf16(x, "x");
  check_f32(w, "w");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.stride(0) % 8 == 0, "x [rows, H] with 16-byte rows");
  TORCH_CHECK(state.scalar_type() == at::kInt && state.numel() >= 8, "state int32[8+]");
  TORCH_CHECK(ag_peer_flags.size() == (size_t)world && world >= 1 && world <= 8, "ag flags: one per rank");
  const c10::cuda::CUDAGuard guard(x.device());
  SpNormArgs a{};
  a.mc_partial = reinterpret_cast<const __nv_bfloat16*>(mc_partial);
  if (!mc_partial) {
    TORCH_CHECK(local_partial.has_value(), "sp_norm_gather: a local addend when there is no partial slot");
    check_bf16(*local_partial, "local_partial");
    TORCH_CHECK(local_partial->size(0) == x.size(0) && local_partial->stride(1) == 1, "local_partial [rows, H]");
    a.local_partial = reinterpret_cast<const __nv_bfloat16*>(local_partial->data_ptr());
    a.ldp = local_partial->stride(0);
  }
  int* s = state.data_ptr<int>();
  a.buf_stride = buf_stride;
  a.sel = s + 2;
  a.flags = reinterpret_cast<const unsigned*>(flags_local);
  a.epoch = s + 0;
  a.world = (int)world;
  a.rank = (int)rank;
  a.x = reinterpret_cast<__nv_bfloat16*>(x.data_ptr());
  a.ldx = x.stride(0);
  a.w = w.data_ptr<float>();
  a.h_mc = reinterpret_cast<__nv_bfloat16*>(h_mc);
  a.rows = (int)x.size(0);
  a.cols = (int)x.size(1);
  a.eps = (float)eps;
  for (int r = 0; r < world; ++r) a.ag_peer_flags[r] = reinterpret_cast<unsigned*>(ag_peer_flags[r]);
  a.ag_epoch = s + 4;
  a.ticket = s + 5;
  a.status = status_dev_ptr();
  a.limit_ns = (unsigned long long)(timeout_s * 1e9);
  if (a.rows > 0) sp_norm_gather(a, at::cuda::getCurrentCUDAStream().stream());
}

// Column-parallel GEMM on the gathered rows: waits per owner for its rows.
Tensor linear_ag_op(const Tensor& h, const Tensor& w, int64_t epi, int64_t ag_flags_local, const Tensor& state,
                    int64_t rows_per_rank, int64_t rank, int64_t world, double timeout_s) {
  check_bf16(h, "h");
  check_bf16(w, "w");
  TORCH_CHECK(h.dim() == 2 && h.stride(1) == 1 && w.dim() == 2 && w.is_contiguous(), "row-major h, w");
  TORCH_CHECK(epi == kEpiBF16 || epi == kEpiSwiGLU, "linear_ag: bf16 or SwiGLU epilogue");
  const c10::cuda::CUDAGuard guard(h.device());
  const int M = (int)h.size(0), Nw = (int)w.size(0), K = (int)h.size(1);
  auto out = at::empty({M, epi == kEpiSwiGLU ? Nw / 2 : Nw}, h.options());
  GemmProblem p;
  p.A = h.data_ptr();
  p.lda = h.stride(0);
  p.B = w.data_ptr();
  p.ldb = w.stride(0);
  p.M = M;
  p.N = Nw;
  p.K = K;
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.epi = (int)epi;
  p.bn = epi == kEpiSwiGLU ? std::max(32, gemm_pick_bn(Nw)) : 0;
  p.status = status_dev_ptr();
  p.allow_split = false;
  p.ag.flags = reinterpret_cast<const unsigned*>(ag_flags_local);
  p.ag.epoch = state.data_ptr<int>() + 4;
  p.ag.rows = (int)rows_per_rank;
  p.ag.rank = (int)rank;
  p.ag.world = (int)world;
  p.ag.limit_ns = (unsigned long long)(timeout_s * 1e9);
  gemm_bf16(p, at::cuda::getCurrentCUDAStream().stream());
  return out;
}

// ---- fused data-parallel gradient reduction --------------------------------
static GradBucketArgs make_grad(const Tensor& grad, int64_t local, int64_t mc, int64_t flags_local,
                                const std::vector<int64_t>& peer_flags, int64_t rank, int64_t epoch,
                                const Tensor& ticket, double timeout_s) {
  TORCH_CHECK(grad.is_cuda() && grad.scalar_type() == at::kFloat && grad.is_contiguous(), "grad: fp32 contiguous");
  TORCH_CHECK(ticket.scalar_type() == at::kInt && ticket.numel() >= 2, "ticket int32[2]: CTA ticket, wait outcome");
  TORCH_CHECK(peer_flags.size() >= 1 && peer_flags.size() <= 8, "1..8 ranks");
  GradBucketArgs a{};
  a.world = (int)peer_flags.size();
  a.rank = (int)rank;
  a.n = grad.numel();
  a.grad = grad.data_ptr<float>();
  a.local = reinterpret_cast<__nv_bfloat16*>(local);
  a.mc = reinterpret_cast<__nv_bfloat16*>(mc);
  a.flags = reinterpret_cast<const unsigned*>(flags_local);
  for (size_t i = 0; i < peer_flags.size(); ++i) a.peer_flags[i] = reinterpret_cast<unsigned*>(peer_flags[i]);
  a.epoch = (unsigned)epoch;
  a.ticket = ticket.data_ptr<int>();
  a.scale = 1.f / (float)a.world;
  a.status = status_dev_ptr();
  a.limit_ns = (unsigned long long)(timeout_s * 1e9);
  return a;
}

void grad_bucket_reduce_op(const Tensor& grad, int64_t local, int64_t mc, int64_t flags_local,
                           std::vector<int64_t> peer_flags, int64_t rank, int64_t epoch, Tensor ticket,
                           double timeout_s) {
  const c10::cuda::CUDAGuard guard(grad.device());
  grad_bucket_reduce(make_grad(grad, local, mc, flags_local, peer_flags, rank, epoch, ticket, timeout_s),
                     at::cuda::getCurrentCUDAStream().stream());
}

void grad_bucket_unpack_op(Tensor grad, int64_t local, int64_t mc, int64_t flags_local, std::vector<int64_t> peer_flags,
                           int64_t rank, int64_t epoch, Tensor ticket, double timeout_s) {
  const c10::cuda::CUDAGuard guard(grad.device());
  grad_bucket_unpack(make_grad(grad, local, mc, flags_local, peer_flags, rank, epoch, ticket, timeout_s),
                     at::cuda::getCurrentCUDAStream().stream());
}

void register_comm_defs(torch::Library& m) {
  m.def(
      "sp_norm_gather(int mc_partial, Tensor? local_partial, int buf_stride, int flags_local, int world, int rank, "
      "Tensor(a!) state, Tensor(b!) x, Tensor w, float eps, int h_mc, int[] ag_peer_flags, float timeout_s) -> ()");
  m.def(
      "linear_ag(Tensor h, Tensor w, int epi, int ag_flags_local, Tensor state, int rows_per_rank, int rank, "
      "int world, float timeout_s) -> Tensor");
  m.def(
      "grad_bucket_reduce(Tensor grad, int local, int mc, int flags_local, int[] peer_flags, int rank, int epoch, "
      "Tensor(a!) ticket, float timeout_s) -> ()");
  m.def(
      "grad_bucket_unpack(Tensor(a!) grad, int local, int mc, int flags_local, int[] peer_flags, int rank, "
      "int epoch, Tensor(b!) ticket, float timeout_s) -> ()");
  m.def(
      "ep_dispatch(Tensor x, Tensor ids, int[] peer_base, int rank, int e_local, int T_max, int max_recv, "
      "Tensor(a!) state, float timeout_s) -> ()");
  m.def(
      "ep_return(Tensor y, int[] peer_base, int rank, int e_local, int k, int T, int T_max, int max_recv, "
      "Tensor(a!) state, float timeout_s) -> ()");
  m.def(
      "gemm_symm(Tensor x, Tensor w, int local_base, int buf_stride, int ldo, int[] peer_flags, "
      "Tensor(a!) local_state, int rank) -> ()");
  m.def(
      "gemm_symm_norm(Tensor x, Tensor w, int local_base, int mc_base, int buf_stride, int[] peer_flags, "
      "int flags_local, Tensor(a!) local_state, int rank, Tensor(b!) residual, Tensor norm_w, float eps, "
      "float timeout_s) -> Tensor");
  m.def(
      "symm_put_signal(Tensor x, int local_base, int buf_stride, int[] peer_flags, Tensor(a!) local_state, "
      "int rank) -> ()");
  m.def(
      "moe_combine_symm(Tensor y, Tensor w, Tensor pos_of, Tensor? pos_sh, Tensor? sg, Tensor? shared_y, "
      "Tensor? shared_gate, int local_base, int buf_stride, int[] peer_flags, Tensor(a!) local_state, int rank) -> ()");
  m.def(
      "moe_combine_symm_norm(Tensor y, Tensor w, Tensor pos_of, Tensor? pos_sh, Tensor? sg, Tensor? shared_y, "
      "Tensor? shared_gate, int local_base, int mc_base, int buf_stride, int[] peer_flags, int flags_local, "
      "Tensor(a!) local_state, int rank, Tensor(b!) residual, Tensor norm_w, float eps, float timeout_s) -> Tensor");
  m.def(
      "ar_add_norm(int mc_base, int buf_stride, int flags_local, int world, Tensor(a!) local_state, "
      "Tensor(b!) residual, Tensor w, float eps, float timeout_s) -> Tensor");
  m.def(
      "ar_hc_post(int mc_base, int buf_stride, int flags_local, int world, Tensor(a!) local_state, "
      "Tensor resid, Tensor post, Tensor comb, float timeout_s) -> Tensor");
  m.def(
      "greedy_allmax(Tensor keys, int[] peer_slots, int[] peer_flags, int flags_local, Tensor(a!) local_state, "
      "int rank, float timeout_s) -> Tensor");
}
void register_comm_pybind(pybind11::module& mod) {
  mod.def("ep_layout", &ep_layout_op, "EP all-to-all symmetric buffer offsets: flags, table, tags, rows, comb, total");
}

void register_comm_impls(torch::Library& m) {
  m.impl("sp_norm_gather", &sp_norm_gather_op);
  m.impl("linear_ag", &linear_ag_op);
  m.impl("grad_bucket_reduce", &grad_bucket_reduce_op);
  m.impl("grad_bucket_unpack", &grad_bucket_unpack_op);
  m.impl("ep_dispatch", &ep_dispatch_op);
  m.impl("ep_return", &ep_return_op);
  m.impl("gemm_symm", &gemm_symm_op);
  m.impl("gemm_symm_norm", &gemm_symm_norm_op);
  m.impl("symm_put_signal", &symm_put_signal_op);
  m.impl("moe_combine_symm", &moe_combine_symm_op);
  m.impl("moe_combine_symm_norm", &moe_combine_symm_norm_op);
  m.impl("ar_add_norm", &ar_add_norm_op);
  m.impl("ar_hc_post", &ar_hc_post_op);
  m.impl("greedy_allmax", &greedy_allmax_op);
}
}  // namespace bwn
