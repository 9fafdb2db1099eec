"""Fused compute + collective paths over NVLink 5 / NVSwitch.

* Row-parallel GEMM -> all-reduce -> residual add -> RMSNorm (the reference's
  ``o_proj/out_proj/down_proj`` + ``functional_all_reduce`` + next norm,
  ``contrib/qwen3.6-27b/static_decode.py:798-961``), one launch: the tcgen05
  GEMM epilogue stores its bf16 partial into this rank's slot of a symmetric
  buffer and the last CTA publishes an epoch flag to every rank; the same CTAs
  then wait for every rank's flag, read the sum of all ranks' slots with
  ``multimem.ld_reduce`` (the NVSwitch adds them, fp32 accumulation), add the
  residual and normalise (``gemm_symm_norm``; ``BWN_F1_ONE_KERNEL=0`` runs the
  reduction as a second kernel, ``ar_add_norm``).
* Sharded greedy (``static_decode_35b.py:1534-1564``): packed (logit, id) keys
  exchanged by peer stores, max taken on every rank, one launch.

Buffers are symmetric allocations (``torch.distributed._symmetric_memory`` is
used only to map them: peer pointers and the multicast address); all device
code is in ``csrc/comm/fused_ar.cu`` and ``csrc/kernels/gemm_tc.cu``.  Every
device-side wait is bounded (``timeout_s``) and reports through the status
word instead of hanging.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import ops


class FusedComm:
    FLAGS_AR = 0
    FLAGS_GREEDY = 128
    SLOTS = 256

    def __init__(self, comm, hidden: int, max_rows: int = 256, device=None, timeout_s: float = 5.0):
        self.comm = comm
        self.world, self.rank = comm.size, comm.rank
        self.hidden = hidden
        self.max_rows = max_rows
        self.timeout_s = timeout_s
        dev = device or torch.device("cuda", torch.cuda.current_device())
        group = comm.group or dist.group.WORLD
        slots_bytes = 8 * max_rows * 8
        self.ar_off = ((self.SLOTS + slots_bytes + 255) // 256) * 256
        self.buf_elems = max_rows * hidden  # bf16 elements per slot (two slots)
        total = self.ar_off + 2 * self.buf_elems * 2
        from .symm import allocate, multicast_address
        self.buf, self.hdl = allocate(total, group, dev, "fused_ar")
        mc = multicast_address(self.hdl)
        ptrs = [int(p) for p in self.hdl.buffer_ptrs]
        self.peer_flags_ar = [p + self.FLAGS_AR for p in ptrs]
        self.peer_flags_g = [p + self.FLAGS_GREEDY for p in ptrs]
        self.peer_slots = [p + self.SLOTS for p in ptrs]
        self.mc_ar = mc + self.ar_off
        self.local_ar = ptrs[self.rank] + self.ar_off
        self.state = torch.zeros(8, dtype=torch.int32, device=dev)
        from ..utils import env
        # row-parallel GEMM + reduction + add + RMSNorm as one launch (gemm_symm_norm)
        self.one_kernel = bool(env.get("BWN_F1_ONE_KERNEL"))
        self.hdl.barrier()
        torch.cuda.synchronize(dev)

    def fits(self, rows: int) -> bool:
        return rows <= self.max_rows

    def gemm_allreduce_add_norm(self, a: torch.Tensor, w: torch.Tensor, x: torch.Tensor, norm_w: torch.Tensor,
                                eps: float) -> torch.Tensor:
        """``x += all_reduce(a @ w.T)`` across ranks; returns ``rmsnorm(x)*(1+norm_w)``."""
        o = ops()
        if hasattr(w, "w8"):  # FP8 weight: W8A16 GEMM, then the multicast reduction
            from .. import ops as O
            return self.allreduce_add_norm(O.linear(a, w), x, norm_w, eps)
        if self.one_kernel:
            return o.gemm_symm_norm(a, w, self.local_ar, self.mc_ar, self.buf_elems, self.peer_flags_ar,
                                    self.peer_flags_ar[self.rank], self.state, self.rank, x, norm_w, eps,
                                    self.timeout_s)
        o.gemm_symm(a, w, self.local_ar, self.buf_elems, w.shape[0], self.peer_flags_ar, self.state, self.rank)
        return o.ar_add_norm(self.mc_ar, self.buf_elems, self.peer_flags_ar[self.rank], self.world, self.state,
                             x, norm_w, eps, self.timeout_s)

    def allreduce_add_norm(self, part: torch.Tensor, x: torch.Tensor, norm_w: torch.Tensor,
                           eps: float) -> torch.Tensor:
        o = ops()
        o.symm_put_signal(part.contiguous(), self.local_ar, self.buf_elems, self.peer_flags_ar, self.state,
                          self.rank)
        return o.ar_add_norm(self.mc_ar, self.buf_elems, self.peer_flags_ar[self.rank], self.world, self.state,
                             x, norm_w, eps, self.timeout_s)

    def reduce_add_norm(self, x: torch.Tensor, norm_w: torch.Tensor, eps: float) -> torch.Tensor:
        """``x += sum over ranks of the partials already stored and signalled in
        the symmetric slots`` (e.g. by ``moe_combine_symm``); returns ``rmsnorm(x)*(1+norm_w)``."""
        return ops().ar_add_norm(self.mc_ar, self.buf_elems, self.peer_flags_ar[self.rank], self.world, self.state,
                                 x, norm_w, eps, self.timeout_s)

    def _zero_norm(self, cols: int, dev) -> torch.Tensor:
        w = getattr(self, "_nw0", None)
        if w is None or w.numel() != cols:
            w = self._nw0 = torch.zeros(cols, dtype=torch.float32, device=dev)
        return w

    def allreduce(self, part: torch.Tensor) -> torch.Tensor:
        """Sum of every rank's ``part [rows, hidden]`` through the one-shot NVLS
        reduction (the fused add-norm kernel accumulating into a zeroed residual;
        its normed output is not used)."""
        acc = torch.zeros_like(part)
        self.allreduce_add_norm(part, acc, self._zero_norm(part.shape[1], part.device), 1e-6)
        return acc

    def gemm_allreduce(self, a: torch.Tensor, w) -> torch.Tensor:
        """``all_reduce(a @ w.T)``: the row-parallel GEMM writes its partial into
        this rank's symmetric slot and the reduction reads it through NVLS."""
        acc = torch.zeros(a.shape[0], w.shape[0], dtype=torch.bfloat16, device=a.device)
        self.gemm_allreduce_add_norm(a, w, acc, self._zero_norm(w.shape[0], a.device), 1e-6)
        return acc

    def allreduce_hc_post(self, part: torch.Tensor, resid: torch.Tensor, post: torch.Tensor,
                          comb: torch.Tensor) -> torch.Tensor:
        """DeepSeek V4's hyper-connection post-mix of the all-reduced ``part
        [rows, dim]``: ``out[t, j] = post[t, j] * sum_ranks(part)[t] + sum_i
        comb[t, i, j] * resid[t, i]`` in one kernel after the partial's store
        (``resid [rows, hc, dim]``)."""
        o = ops()
        o.symm_put_signal(part.contiguous(), self.local_ar, self.buf_elems, self.peer_flags_ar, self.state,
                          self.rank)
        return o.ar_hc_post(self.mc_ar, self.buf_elems, self.peer_flags_ar[self.rank], self.world, self.state,
                            resid.contiguous(), post.contiguous(), comb.contiguous(), self.timeout_s)

    def gemm_allreduce_hc_post(self, a: torch.Tensor, w, resid: torch.Tensor, post: torch.Tensor,
                               comb: torch.Tensor) -> torch.Tensor:
        """``hc_post(all_reduce(a @ w.T), resid, post, comb)``: the row-parallel
        GEMM's epilogue stores its partial into this rank's symmetric slot, and
        one kernel reduces it through NVLS and applies the post-mix."""
        o = ops()
        if hasattr(w, "w8"):
            from .. import ops as O
            return self.allreduce_hc_post(O.linear(a, w), resid, post, comb)
        o.gemm_symm(a, w, self.local_ar, self.buf_elems, w.shape[0], self.peer_flags_ar, self.state, self.rank)
        return o.ar_hc_post(self.mc_ar, self.buf_elems, self.peer_flags_ar[self.rank], self.world, self.state,
                            resid.contiguous(), post.contiguous(), comb.contiguous(), self.timeout_s)

    def greedy(self, keys: torch.Tensor) -> torch.Tensor:
        return ops().greedy_allmax(keys.contiguous(), self.peer_slots, self.peer_flags_g,
                                   self.peer_flags_g[self.rank], self.state, self.rank, self.timeout_s)


def enable_fused_comm(model, max_rows: int = 256) -> FusedComm:
    """Route the model's row-parallel reductions and greedy through the fused
    NVLink kernels (decode-sized batches); larger batches keep NCCL.  Works for
    :class:`~bwn.models.qwen36.Qwen36Model` (``cfg.hidden``) and
    :class:`~bwn.models.deepseek_v4.DeepSeekV4Model` (``cfg.dim``)."""
    if model.comm.size <= 1:
        raise RuntimeError("fused comm needs more than one rank")
    from .topology import require_single_domain
    require_single_domain(model.comm, "fused comm")
    hidden = getattr(model.cfg, "hidden", None) or model.cfg.dim
    fc = FusedComm(model.comm, hidden, max_rows, model.device)
    model.fused_comm = fc
    return fc
