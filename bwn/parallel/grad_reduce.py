"""Data-parallel gradient reduction overlapped with backward, fused with the
cast and 1/world scale (the reference relies on DTensor / FSDP collectives,
``contrib/esm2/train_esm.py:216-226``, ``train_esm_fsdp.py:111-117``).

* Parameters are grouped into buckets in reverse registration order (roughly
  the order backward produces their gradients).  Each bucket owns a flat fp32
  gradient buffer; ``p.grad`` is a view into it (zero it in place between
  steps: ``optimizer.zero_grad(set_to_none=False)``).
* A post-accumulate-grad hook counts the bucket's ready parameters; the last
  one launches, on a side stream, the fused kernels of
  ``csrc/comm/grad_reduce.cu``: pack (fp32 * 1/world -> bf16 into the
  symmetric buffer) and a one-pass NVLS reduce-scatter + all-gather
  (``multimem.ld_reduce`` of this rank's slice, ``multimem.st`` of the sum).
* :meth:`GradReducer.finish` (after ``backward``) launches the remaining
  buckets, unpacks every bucket back into the fp32 gradients and joins the
  side stream.

:class:`NcclGradReducer` is the baseline: one NCCL all-reduce per bucket on
the same buckets.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops as O


class _Bucket:
    def __init__(self, params, n_pad: int, device):
        self.params = params
        self.n = n_pad
        self.flat = torch.zeros(n_pad, dtype=torch.float32, device=device)
        off = 0
        self.views = []
        for p in params:
            v = self.flat[off:off + p.numel()].view_as(p)
            self.views.append(v)
            off += p.numel()
        self.ready = 0
        self.launched = False


def _buckets(model, bucket_elems: int, align: int, device):
    params = [p for p in model.parameters() if p.requires_grad]
    out, cur, size = [], [], 0
    for p in reversed(params):
        cur.append(p)
        size += p.numel()
        if size >= bucket_elems:
            out.append(cur)
            cur, size = [], 0
    if cur:
        out.append(cur)
    res = []
    for ps in out:
        n = sum(p.numel() for p in ps)
        res.append(_Bucket(ps, (n + align - 1) // align * align, device))
    return res


class _HookedReducer:
    def __init__(self, model, comm, bucket_mb: float, align: int):
        self.comm = comm
        self.W = comm.size
        dev = next(model.parameters()).device
        self.buckets = _buckets(model, int(bucket_mb * 2**20 / 4), align, dev)
        self.owner = {}
        for b in self.buckets:
            for p, v in zip(b.params, b.views):
                p.grad = v
                self.owner[p] = b
                p.register_post_accumulate_grad_hook(self._hook)
        self.side = torch.cuda.Stream(dev) if dev.type == "cuda" else None

    def _hook(self, p):
        b = self.owner[p]
        b.ready += 1
        if b.ready == len(b.params) and not b.launched:
            self._launch(b)

    def _launch(self, b):
        b.launched = True
        if self.side is None:
            self._reduce(b)
            return
        ev = torch.cuda.Event()
        ev.record()
        with torch.cuda.stream(self.side):
            self.side.wait_event(ev)
            self._reduce(b)

    def finish(self) -> None:
        for b in self.buckets:
            if not b.launched:
                self._launch(b)
        if self.side is not None:
            with torch.cuda.stream(self.side):
                for b in self.buckets:
                    self._unpack(b)
            torch.cuda.current_stream().wait_stream(self.side)
        else:
            for b in self.buckets:
                self._unpack(b)
        for b in self.buckets:
            b.ready, b.launched = 0, False
            for p, v in zip(b.params, b.views):
                if p.grad is None or p.grad.data_ptr() != v.data_ptr():
                    p.grad = v  # keep gradients in the bucket storage

    def reduce(self, model=None) -> None:
        self.finish()

    def _unpack(self, b):
        pass


class NcclGradReducer(_HookedReducer):
    """One NCCL (or gloo) all-reduce + scale per bucket, overlapped the same way."""

    def __init__(self, model, comm, bucket_mb: float = 32.0):
        super().__init__(model, comm, bucket_mb, align=8)

    def _reduce(self, b):
        dist.all_reduce(b.flat, group=self.comm.group)
        b.flat.div_(self.W)


class GradReducer(_HookedReducer):
    """Fused NVLS reduction (bf16 on the wire, fp32 accumulation in the switch)."""

    FLAG_BYTES = 256  # per bucket: 2 phases x 8 ranks x 4 bytes, padded

    def __init__(self, model, comm, bucket_mb: float = 32.0, timeout_s: float = 30.0):
        from .topology import require_single_domain
        require_single_domain(comm, "fused gradient reduction")
        super().__init__(model, comm, bucket_mb, align=8 * comm.size)
        self.timeout_s = timeout_s
        self.rank = comm.rank
        dev = self.buckets[0].flat.device
        group = comm.group or dist.group.WORLD
        nb = len(self.buckets)
        data_off = (nb * self.FLAG_BYTES + 255) // 256 * 256
        offs, total = [], data_off
        for b in self.buckets:
            offs.append(total)
            total += (b.n * 2 + 255) // 256 * 256
        from .symm import allocate, multicast_address
        self.buf, self.hdl = allocate(total, group, dev, "grad_reduce")
        ptrs = [int(p) for p in self.hdl.buffer_ptrs]
        mc = multicast_address(self.hdl)
        for i, b in enumerate(self.buckets):
            b.local = ptrs[self.rank] + offs[i]
            b.mc = mc + offs[i]
            b.flags_local = ptrs[self.rank] + i * self.FLAG_BYTES
            b.peer_flags = [p + i * self.FLAG_BYTES for p in ptrs]
            b.ticket = torch.zeros(2, dtype=torch.int32, device=dev)  # CTA ticket, last wait's outcome
        self.steps = 0  # flags of step s reach s + 1
        self.hdl.barrier()
        torch.cuda.synchronize(dev)

    def finish(self) -> None:
        super().finish()
        self.steps += 1

    def _reduce(self, b):
        O.ops().grad_bucket_reduce(b.flat, b.local, b.mc, b.flags_local, b.peer_flags, self.rank, self.steps + 1,
                                   b.ticket, self.timeout_s)

    def _unpack(self, b):
        O.ops().grad_bucket_unpack(b.flat, b.local, b.mc, b.flags_local, b.peer_flags, self.rank, self.steps + 1,
                                   b.ticket, self.timeout_s)
