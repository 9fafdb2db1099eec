"""Megatron-style tensor parallelism for training (ESM-2).

The reference applies DTensor ``ColwiseParallel`` to query/key/value and
``intermediate.dense`` and ``RowwiseParallel`` to ``attention.output.dense``
and ``output.dense`` (``contrib/esm2/train_esm.py:208-228``,
``run_esm.py:49-69``).  The same plan here is explicit, without DTensor:

* a column-parallel linear holds ``out/tp`` output rows (and bias slice); its
  input passes through :class:`_CopyToTP` (identity forward, all-reduce of the
  input gradient backward);
* a row-parallel linear holds ``in/tp`` input columns; its output passes through
  :class:`_ReduceFromTP` (all-reduce forward, identity backward) and the bias is
  added once after the reduction;
* attention heads are split across ranks with their q/k/v rows.

Both linears run on the bwn tcgen05 GEMMs (forward and backward) through
:class:`~bwn.models.esm2.BwnLinear`.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..models.esm2 import BwnLinear


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, comm):
        ctx.comm = comm
        return x

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous().clone()
        ctx.comm.all_reduce_(g)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, comm):
        y = x.contiguous().clone()
        comm.all_reduce_(y)
        return y

    @staticmethod
    def backward(ctx, g):
        return g, None


class ColumnParallelLinear(nn.Module):
    def __init__(self, full: nn.Linear, comm):
        super().__init__()
        tp, r = comm.size, comm.rank
        out = full.out_features
        if out % tp:
            raise ValueError(f"{out} output features do not split over {tp} ranks")
        n = out // tp
        self.comm = comm
        with torch.device(full.weight.device):
            self.lin = BwnLinear(full.in_features, n, bias=full.bias is not None)
        with torch.no_grad():
            self.lin.weight.copy_(full.weight[r * n:(r + 1) * n])
            if full.bias is not None:
                self.lin.bias.copy_(full.bias[r * n:(r + 1) * n])

    @property
    def weight(self):
        return self.lin.weight

    def forward(self, x):
        return self.lin(_CopyToTP.apply(x, self.comm))


class RowParallelLinear(nn.Module):
    def __init__(self, full: nn.Linear, comm):
        super().__init__()
        tp, r = comm.size, comm.rank
        inp = full.in_features
        if inp % tp:
            raise ValueError(f"{inp} input features do not split over {tp} ranks")
        n = inp // tp
        self.comm = comm
        with torch.device(full.weight.device):
            self.lin = BwnLinear(n, full.out_features, bias=False)
        with torch.no_grad():
            self.lin.weight.copy_(full.weight[:, r * n:(r + 1) * n])
        self.bias = nn.Parameter(full.bias.detach().clone()) if full.bias is not None else None

    @property
    def weight(self):
        return self.lin.weight

    def forward(self, x):
        y = _ReduceFromTP.apply(self.lin(x), self.comm)
        return y + self.bias.to(y.dtype) if self.bias is not None else y


ESM_TP_PLAN = {
    "attention.self.query": "colwise",
    "attention.self.key": "colwise",
    "attention.self.value": "colwise",
    "attention.output.dense": "rowwise",
    "intermediate.dense": "colwise",
    "output.dense": "rowwise",
}


def apply_esm_tp(model, comm, plan: dict | None = None):
    """Shard every encoder layer of an :class:`~bwn.models.esm2.EsmForMaskedLM`
    in place (embeddings, final norms and LM head stay replicated), through
    :func:`bwn.parallel.plan.parallelize_module` with the reference's layer plan."""
    if comm.size <= 1:
        return model
    from .plan import parallelize_module
    heads = model.cfg.heads
    if heads % comm.size:
        raise ValueError(f"{heads} heads do not split over {comm.size} ranks")
    for layer in model.esm.encoder.layer:
        parallelize_module(layer, comm, plan or ESM_TP_PLAN)
        layer.attention.self.heads = heads // comm.size
    model.tp_comm = comm
    return model


def sync_replicated_grads(model, comm) -> None:
    """Replicated parameters (embeddings, norms, LM head, row-parallel biases)
    receive identical gradients on every rank under this plan, except through
    floating-point reduction order; average them so replicas never drift."""
    if comm.size <= 1:
        return
    for n, p in model.named_parameters():
        if p.grad is None or ".lin." in n:
            continue
        comm.all_reduce_(p.grad)
        p.grad.div_(comm.size)
