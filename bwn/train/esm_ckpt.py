"""Portable ESM-2 training checkpoints: written once, loadable at any
tensor-parallel or data-parallel degree.

The reference saves one ``checkpoint.pt`` from rank 0 with the model state
moved to CPU, the optimizer and scheduler states, the step and the loss, and
resumes from it with ``--resume`` (``contrib/esm2/train_esm.py:148-178``).
Under tensor parallelism a rank holds only shards, so here the checkpoint is
always the **unsharded** model with HF parameter names plus the AdamW moments
in the same layout (keyed by parameter name, not by optimizer index); shards
are gathered on save and sliced again on load, so a run saved at TP2 resumes
at TP1, TP4 or under data parallelism.  Each rank's data / masking generator
states are kept by rank so a resume at the same world size continues the
exact sample stream.

The sharding of each parameter is read off the modules
(:class:`~bwn.parallel.tensor_parallel.ColumnParallelLinear`: rows,
:class:`~bwn.parallel.tensor_parallel.RowParallelLinear`: columns,
:class:`~bwn.parallel.plan.VocabParallelEmbedding`: rows); every other
parameter is replicated.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def param_layout(model) -> dict[str, tuple[str, int | None]]:
    """``{local name: (unsharded HF name, shard dim or None)}``."""
    from ..parallel.plan import VocabParallelEmbedding
    from ..parallel.tensor_parallel import ColumnParallelLinear, RowParallelLinear
    shard: dict[str, tuple[str, int]] = {}
    for path, mod in model.named_modules():
        pre = path + "." if path else ""
        if isinstance(mod, ColumnParallelLinear):
            shard[pre + "lin.weight"] = (pre + "weight", 0)
            shard[pre + "lin.bias"] = (pre + "bias", 0)
        elif isinstance(mod, RowParallelLinear):
            shard[pre + "lin.weight"] = (pre + "weight", 1)
        elif isinstance(mod, VocabParallelEmbedding):
            shard[pre + "weight"] = (pre + "weight", 0)
    out = {}
    for name, _ in model.named_parameters():
        out[name] = shard.get(name, (name, None))
    return out


def _gather(t: torch.Tensor, dim: int | None, comm) -> torch.Tensor:
    if dim is None or comm is None or comm.size <= 1:
        return t.detach().cpu().clone()
    parts = [torch.empty_like(t) for _ in range(comm.size)]
    dist.all_gather(parts, t.detach().contiguous(), group=comm.group)
    return torch.cat([p.cpu() for p in parts], dim=dim)


def _slice(full: torch.Tensor, dim: int | None, like: torch.Tensor, comm) -> torch.Tensor:
    if dim is None or comm is None or comm.size <= 1:
        return full
    n = like.shape[dim]
    return full.narrow(dim, comm.rank * n, n)


def full_state(model, opt, tp_comm) -> tuple[dict, dict]:
    """Unsharded ``(model_state, moments)``; collective under tensor
    parallelism (every rank must call it)."""
    layout = param_layout(model)
    msd, moments = {}, {}
    for name, p in model.named_parameters():
        canon, dim = layout[name]
        msd[canon] = _gather(p, dim, tp_comm)
        st = opt.state.get(p, {})
        if "exp_avg" in st:
            moments[canon] = {"step": st["step"].detach().cpu().clone() if torch.is_tensor(st["step"])
                              else torch.tensor(float(st["step"])),
                              "exp_avg": _gather(st["exp_avg"], dim, tp_comm),
                              "exp_avg_sq": _gather(st["exp_avg_sq"], dim, tp_comm)}
    return msd, moments


def load_full_state(model, opt, tp_comm, msd: dict, moments: dict) -> None:
    """Slice an unsharded state into this rank's parameters and AdamW moments."""
    layout = param_layout(model)
    with torch.no_grad():
        for name, p in model.named_parameters():
            canon, dim = layout[name]
            if canon not in msd:
                raise KeyError(f"checkpoint has no {canon}")
            p.copy_(_slice(msd[canon], dim, p, tp_comm))
            if canon in moments:
                m = moments[canon]
                opt.state[p] = {"step": m["step"].clone().float(),
                                "exp_avg": _slice(m["exp_avg"], dim, p, tp_comm).to(p.device, p.dtype).clone(),
                                "exp_avg_sq": _slice(m["exp_avg_sq"], dim, p, tp_comm).to(p.device, p.dtype).clone()}


def gather_objects(obj, comm) -> list:
    """Every rank's ``obj`` (collective when the job has several ranks)."""
    if comm is None or comm.size <= 1:
        return [obj]
    out = [None] * comm.size
    dist.all_gather_object(out, obj, group=comm.group)
    return out
