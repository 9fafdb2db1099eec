"""A ``parallelize_module``-style tensor-parallel plan API over bwn's sharded
modules.

The reference shards HF ESM-2 and its DeepSeek model with DTensor plans,
``{"attention.self.query": ColwiseParallel(), ...}`` passed to
``torch.distributed.tensor.parallel.parallelize_module``
(``contrib/esm2/run_esm.py:49-69``, ``contrib/esm2/train_esm.py:208-228``,
``contrib/deepseek-v4-flash/run_deepseek_v4_tp.py:655-669``).  The same plan
dictionaries work here: :func:`parallelize_module` replaces each matched module
by an explicit shard whose local tensors are plain tensors and whose
collectives are the :class:`~bwn.parallel.comm.Comm` ones, so the sharded
Linears run on the bwn tcgen05 GEMMs:

* ``nn.Linear`` + colwise: :class:`~bwn.parallel.tensor_parallel.ColumnParallelLinear`
  (``out/tp`` rows; the output stays sharded on its last dim, DTensor's default
  ``Shard(-1)`` output; the input gradient is all-reduced);
* ``nn.Linear`` + rowwise: :class:`~bwn.parallel.tensor_parallel.RowParallelLinear`
  (``in/tp`` columns of a last-dim-sharded input; output all-reduced, bias added once);
* ``nn.Embedding`` + rowwise: :class:`VocabParallelEmbedding` (``vocab/tp``
  rows; ids outside the shard read zeros; output all-reduced).

Plan values may be torch's ``ColwiseParallel()`` / ``RowwiseParallel()``
objects, this module's :class:`Colwise` / :class:`Rowwise`, or the strings
``"colwise"`` / ``"rowwise"``; keys are module paths relative to the
parallelized module and may use ``fnmatch`` wildcards per path component
(``"layers.*.attn.wo_b"``), as DTensor plans may.  Modules whose local shapes
are inferred from their inputs (HF attention reshapes with ``-1`` heads) need
no other change.
"""
from __future__ import annotations

import fnmatch

import torch
import torch.nn as nn
import torch.nn.functional as F

from .tensor_parallel import ColumnParallelLinear, RowParallelLinear, _ReduceFromTP


class Colwise:
    """Shard a Linear's output features across the ranks."""


class Rowwise:
    """Shard a Linear's input features (or an Embedding's vocabulary) across the ranks."""


def _style(v) -> str:
    if isinstance(v, str):
        s = v.lower()
    elif isinstance(v, (Colwise, Rowwise)):
        s = "colwise" if isinstance(v, Colwise) else "rowwise"
    else:  # torch.distributed.tensor.parallel.{Colwise,Rowwise}Parallel and subclasses
        names = [c.__name__ for c in type(v).__mro__]
        s = "colwise" if "ColwiseParallel" in names else "rowwise" if "RowwiseParallel" in names else ""
    if s not in ("colwise", "rowwise"):
        raise ValueError(f"unsupported parallel style {v!r}: expected colwise or rowwise")
    return s


class VocabParallelEmbedding(nn.Module):
    """``vocab/tp`` rows of an embedding table; the looked-up rows of every rank
    are summed (ids outside this rank's range contribute zeros)."""

    def __init__(self, full: nn.Embedding, comm):
        super().__init__()
        tp, r = comm.size, comm.rank
        if full.num_embeddings % tp:
            raise ValueError(f"{full.num_embeddings} rows do not split over {tp} ranks")
        n = full.num_embeddings // tp
        self.comm, self.offset, self.rows = comm, r * n, n
        self.padding_idx = full.padding_idx
        self.weight = nn.Parameter(full.weight.detach()[r * n:(r + 1) * n].clone())

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        local = ids - self.offset
        hit = (local >= 0) & (local < self.rows)
        y = F.embedding(local.clamp(0, self.rows - 1), self.weight) * hit.unsqueeze(-1).to(self.weight.dtype)
        return _ReduceFromTP.apply(y, self.comm)


def _matches(pattern: str, name: str) -> bool:
    p, n = pattern.split("."), name.split(".")
    return len(p) == len(n) and all(fnmatch.fnmatchcase(b, a) for a, b in zip(p, n))


def _replace(root: nn.Module, name: str, new: nn.Module) -> None:
    parent = root.get_submodule(name.rsplit(".", 1)[0]) if "." in name else root
    setattr(parent, name.rsplit(".", 1)[-1], new)


def parallelize_module(module: nn.Module, comm, plan: dict) -> nn.Module:
    """Shard ``module`` in place by ``plan`` (see the module docstring); returns
    it.  A single-rank ``comm`` leaves it unchanged.  Every plan key must match
    at least one Linear / Embedding."""
    if comm.size <= 1:
        return module
    named = dict(module.named_modules())
    for pattern, style in plan.items():
        kind = _style(style)
        hits = [n for n in named if n and _matches(pattern, n)]
        if not hits:
            raise KeyError(f"plan key {pattern!r} matches no submodule")
        for n in hits:
            m = named[n]
            if isinstance(m, nn.Linear):
                new = ColumnParallelLinear(m, comm) if kind == "colwise" else RowParallelLinear(m, comm)
            elif isinstance(m, nn.Embedding) and kind == "rowwise":
                new = VocabParallelEmbedding(m, comm)
            else:
                raise TypeError(f"{n}: {kind} sharding of {type(m).__name__} is not supported")
            _replace(module, n, new)
    return module
