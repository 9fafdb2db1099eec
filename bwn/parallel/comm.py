"""Process-group plumbing for tensor/expert parallelism.

Replaces the reference's ``dist.init_process_group("neuron")`` and
``functional_all_reduce`` (``contrib/qwen3.6-27b/static_decode.py:92-96``,
``contrib/qwen3.6-35b-a3b/static_decode_35b.py:501-506``): a no-op when the
group has one rank, NCCL on GPUs, gloo on CPU (the CPU multi-rank tests).
The fused NVLink compute+collective kernels live in :mod:`bwn.parallel.fused`
and use this object only for bootstrap (rank, size, group).
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


class Comm:
    def __init__(self, group=None, rank: int = 0, size: int = 1):
        self.group = group
        self.rank = rank
        self.size = size
        # cost probe (the reference's NOREDUCE): sum all-reduces become no-ops
        self.no_reduce = os.environ.get("BWN_NO_REDUCE", "0") == "1"

    @staticmethod
    def single() -> "Comm":
        return Comm(None, 0, 1)

    @staticmethod
    def from_group(group=None) -> "Comm":
        if not dist.is_available() or not dist.is_initialized():
            return Comm.single()
        return Comm(group, dist.get_rank(group), dist.get_world_size(group))

    # ---- collectives (in place) ------------------------------------------
    def all_reduce_(self, x: torch.Tensor) -> torch.Tensor:
        if self.size > 1 and not self.no_reduce:
            dist.all_reduce(x, op=dist.ReduceOp.SUM, group=self.group)
        return x

    def all_reduce_max_(self, x: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            dist.all_reduce(x, op=dist.ReduceOp.MAX, group=self.group)
        return x

    def all_gather_last(self, x: torch.Tensor) -> torch.Tensor:
        """Concatenate rank shards along the last dim."""
        if self.size == 1:
            return x
        parts = [torch.empty_like(x) for _ in range(self.size)]
        dist.all_gather(parts, x.contiguous(), group=self.group)
        return torch.cat(parts, dim=-1)

    def all_gather_first(self, x: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return x
        out = torch.empty((self.size * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out

    def all_to_all_single(self, out: torch.Tensor, inp: torch.Tensor, out_splits=None, in_splits=None):
        if self.size == 1:
            out.copy_(inp)
            return out
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
        return out

    def barrier(self) -> None:
        if self.size > 1:
            if torch.cuda.is_available() and dist.get_backend(self.group) == "nccl":
                dist.barrier(group=self.group, device_ids=[torch.cuda.current_device()])
            else:
                dist.barrier(group=self.group)

    def max_scalar(self, v: float, device=None) -> float:
        """Max of a host scalar over ranks (used for max-over-ranks timings)."""
        if self.size == 1:
            return v
        if device is None and dist.get_backend(self.group) == "nccl":
            device = torch.device("cuda", torch.cuda.current_device())
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return float(t.item())


def init_distributed(backend: str | None = None, timeout_s: float = 120.0) -> Comm:
    """Initialise the default process group from torchrun's env (RANK,
    WORLD_SIZE, LOCAL_RANK, MASTER_ADDR/PORT); one process per GPU."""
    if dist.is_initialized():
        return Comm.from_group(None)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return Comm.single()
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local))
    else:
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    return Comm.from_group(None)


def hybrid_groups(tp: int, timeout_s: float = 120.0) -> tuple[Comm, Comm]:
    """Split the world into tensor-parallel groups of ``tp`` consecutive ranks
    and expert-parallel groups of the ranks with the same TP index (strided by
    ``tp``), as the reference's hybrid runner does
    (``contrib/deepseek-v4-flash/run_deepseek_v4_hybrid.py:760-763``).  Every
    rank creates every group, in the same order."""
    world, rank = dist.get_world_size(), dist.get_rank()
    if world % tp:
        raise ValueError(f"tp={tp} must divide the world size {world}")
    ep = world // tp
    tp_group = ep_group = None
    for g in range(ep):
        ranks = list(range(g * tp, (g + 1) * tp))
        grp = dist.new_group(ranks, timeout=datetime.timedelta(seconds=timeout_s))
        if rank in ranks:
            tp_group = grp
    for i in range(tp):
        ranks = list(range(i, world, tp))
        grp = dist.new_group(ranks, timeout=datetime.timedelta(seconds=timeout_s))
        if rank in ranks:
            ep_group = grp
    return (Comm(tp_group, dist.get_rank(tp_group), tp), Comm(ep_group, dist.get_rank(ep_group), ep))
