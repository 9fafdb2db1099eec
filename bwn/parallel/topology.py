"""Interconnect topology of the visible GPUs.

The reference selects a NeuronCore grouping (LNC=1/2) from env
(``contrib/qwen3.6-35b-a3b/kernels/topology_35b.py:6-20``).  On an HGX B200
the question is which data paths the comm layer may use: peer access between
every pair (NVLink through NVSwitch), and NVLink multicast (NVLS) for
``multimem`` reductions.  :func:`probe` answers from the CUDA runtime; the
decision function :func:`choose_comm_path` is pure so it is tested on CPU with
fake topologies.  :func:`require_single_domain` is the check every fused path
runs when it is enabled: a group spanning hosts (a multi-node job) keeps NCCL.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class Topology:
    n_gpus: int
    names: list[str] = field(default_factory=list)
    peer: list[list[bool]] = field(default_factory=list)  # peer[i][j]: i can access j's memory
    multicast: bool = False                              # NVLS multicast objects supported

    @property
    def all_peer(self) -> bool:
        return all(self.peer[i][j] for i in range(self.n_gpus) for j in range(self.n_gpus) if i != j)


def probe() -> Topology:
    if not torch.cuda.is_available():
        return Topology(0)
    n = torch.cuda.device_count()
    peer = [[i == j or torch.cuda.can_device_access_peer(i, j) for j in range(n)] for i in range(n)]
    mc = False
    try:
        from cuda.bindings import driver as drv  # cuda-python
        drv.cuInit(0)
        err, dev = drv.cuDeviceGet(0)
        err, v = drv.cuDeviceGetAttribute(drv.CUdevice_attribute.CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev)
        mc = bool(v) and int(err) == 0
    except Exception:
        mc = False
    return Topology(n, [torch.cuda.get_device_name(i) for i in range(n)], peer, mc)


def choose_comm_path(topo: Topology, world: int, requested: str = "auto") -> str:
    """``"single"`` (one rank), ``"fused_nvls"`` (multimem kernels), ``"fused_p2p"``
    (peer loads/stores only) or ``"nccl"``.  ``requested`` is ``auto|on|off``."""
    if world <= 1:
        return "single"
    if requested == "off":
        return "nccl"
    usable = topo.n_gpus >= world and all(topo.peer[i][j] for i in range(world) for j in range(world))
    if not usable:
        if requested == "on":
            raise RuntimeError("fused comm requested but the ranks' GPUs lack peer access to one another")
        return "nccl"
    return "fused_nvls" if topo.multicast else "fused_p2p"


def hosts_of(comm) -> list[str]:
    """Host name of every rank of ``comm`` (collective over the group)."""
    import socket

    import torch.distributed as dist
    name = socket.gethostname()
    if comm.size <= 1 or not dist.is_initialized():
        return [name]
    out = [None] * comm.size
    dist.all_gather_object(out, name, group=comm.group)
    return out


def require_single_domain(comm, what: str) -> None:
    """The fused kernels address peers' memory directly, so every rank of the
    group must sit in one NVLink / NVSwitch domain (one host here).  Raises
    otherwise (callers fall back to NCCL)."""
    hosts = hosts_of(comm)
    if len(set(hosts)) > 1:
        raise RuntimeError(f"{what}: the group spans hosts {sorted(set(hosts))}; peer-memory kernels need one "
                           "NVLink domain (NCCL is used instead)")
