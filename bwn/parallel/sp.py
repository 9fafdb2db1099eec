"""Sequence-parallel prefill plumbing: reduce-scatter -> norm -> all-gather ->
GEMM with the collectives inside the kernels.

* row-parallel GEMM (``gemm_symm``): bf16 partial of every token into this
  rank's symmetric slot + completion flags;
* ``sp_norm_gather``: for this rank's shard of rows only, the sum of all
  ranks' partials through the switch (``multimem.ld_reduce``), residual add,
  RMSNorm, and one multicast store of the normed rows into every rank's
  gathered buffer, then a gather flag;
* ``linear_ag``: the next column-parallel GEMM reads the gathered rows; its
  TMA producer waits for each owner's gather flag before loading that owner's
  rows and starts with this rank's own rows, so the gather overlaps the GEMM.

The residual stream stays sharded (``T / world`` rows per rank).  This is the
sequence-parallel variant of the reference's replicated-activation TP
(``contrib/qwen3.6-27b/static_decode.py:798-961`` all-reduces every
row-parallel output).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops as O


class SeqParallel:
    FLAGS = 256  # partial flags at 0, gather flags at 128 (bytes)

    def __init__(self, comm, hidden: int, max_tokens: int, device=None, timeout_s: float = 10.0):
        self.comm, self.W, self.rank = comm, comm.size, comm.rank
        self.H, self.T_max, self.timeout_s = hidden, max_tokens, timeout_s
        dev = device or torch.device("cuda", torch.cuda.current_device())
        self.buf_elems = max_tokens * hidden
        self.off_partial = self.FLAGS
        self.off_h = self.off_partial + 2 * self.buf_elems * 2
        total = self.off_h + self.buf_elems * 2
        group = comm.group or dist.group.WORLD
        from .symm import allocate, multicast_address
        self.buf, self.hdl = allocate(total, group, dev, "seq_parallel")
        mc = multicast_address(self.hdl)
        ptrs = [int(p) for p in self.hdl.buffer_ptrs]
        self.partial_flags = list(ptrs)
        self.gather_flags = [p + 128 for p in ptrs]
        self.local_partial = ptrs[self.rank] + self.off_partial
        self.mc_partial = mc + self.off_partial
        self.mc_h = mc + self.off_h
        self.h = self.buf[self.off_h:self.off_h + self.buf_elems * 2].view(torch.bfloat16).view(max_tokens, hidden)
        self.state = torch.zeros(16, dtype=torch.int32, device=dev)
        self.hdl.barrier()
        torch.cuda.synchronize(dev)

    def row_parallel(self, a: torch.Tensor, w: torch.Tensor) -> None:
        O.ops().gemm_symm(a.contiguous(), w, self.local_partial, self.buf_elems, self.H, self.partial_flags, self.state,
                          self.rank)

    def norm_gather(self, x_shard: torch.Tensor, norm_w: torch.Tensor, eps: float, addend=None) -> None:
        """``x_shard += (sum of partials | addend)``; normed rows gathered into ``self.h``."""
        O.ops().sp_norm_gather(0 if addend is not None else self.mc_partial, addend, self.buf_elems,
                               self.partial_flags[self.rank], self.W, self.rank, self.state, x_shard, norm_w, eps,
                               self.mc_h, self.gather_flags, self.timeout_s)

    def gathered(self, T: int) -> torch.Tensor:
        return self.h[:T]

    def column(self, w: torch.Tensor, T: int, swiglu: bool = False) -> torch.Tensor:
        return O.ops().linear_ag(self.h[:T], w, O.EPI_SWIGLU if swiglu else O.EPI_BF16,
                                 self.gather_flags[self.rank], self.state, T // self.W, self.rank, self.W,
                                 self.timeout_s)


def enable_sequence_parallel(model, max_tokens: int) -> SeqParallel:
    """Full-length prompts of up to ``max_tokens`` tokens (``B*S`` a multiple of
    ``128 * world``) prefill sequence-parallel; other calls keep the replicated path."""
    if model.comm.size <= 1:
        raise RuntimeError("sequence parallelism needs more than one rank")
    from .topology import require_single_domain
    require_single_domain(model.comm, "sequence-parallel prefill")
    sp = SeqParallel(model.comm, model.cfg.hidden, max_tokens, model.device)
    model.seq_parallel = sp
    return sp
