"""Symmetric-memory helpers shared by the fused collective paths.

:func:`allocate` is the one place the fused paths get their peer-mapped
buffers: it rendezvouses a zeroed buffer across the group and appends a guard
tail of :data:`CANARY_BYTES` filled with :data:`CANARY` after the usable
bytes.  No kernel addresses the tail, so a changed tail means some launch
(this rank's or a peer's store through NVLink) wrote past its region;
:func:`check_canaries` reports it (the GPU tests run it after every test).
"""
from __future__ import annotations

import weakref

import torch

CANARY_BYTES = 4096
CANARY = 0xA5

_guarded: list[tuple[weakref.ref, int, str]] = []


def multicast_address(hdl) -> int:
    """The NVLS multicast address of a rendezvoused symmetric buffer.

    PyTorch can report multicast support and still skip creating the multicast
    object (it logs "Gracefully skipping multicast initialization", e.g. on a
    one-rank group); the address is then 0 and a ``multimem`` access to it
    would fault.  Both conditions are checked here so a caller falls back (or
    fails on the host) instead."""
    mc = int(hdl.multicast_ptr) if getattr(hdl, "has_multicast_support", False) else 0
    if mc == 0:
        raise RuntimeError("NVLS multicast is not available for this group")
    return mc


def allocate(nbytes: int, group, device, name: str = "symm"):
    """``(buf, hdl)``: ``nbytes`` zeroed bytes of symmetric memory rendezvoused
    over ``group`` (``buf`` is the usable prefix; peer pointers and the
    multicast address from ``hdl`` start at its first byte), followed by the
    guard tail."""
    import torch.distributed._symmetric_memory as symm
    # torch releases before 2.9 want symmetric memory enabled per group first;
    # later ones deprecate the call (it warns on every rank)
    if tuple(int(x) for x in torch.__version__.split(".")[:2]) < (2, 9):
        symm.enable_symm_mem_for_group(group.group_name)
    full = symm.empty(nbytes + CANARY_BYTES, dtype=torch.uint8, device=device)
    full[:nbytes].zero_()
    full[nbytes:].fill_(CANARY)
    torch.cuda.synchronize(device)
    hdl = symm.rendezvous(full, group)
    _guarded.append((weakref.ref(full), nbytes, name))
    return full[:nbytes], hdl


def tail_intact(full: torch.Tensor, nbytes: int) -> bool:
    return bool((full[nbytes:] == CANARY).all())


def check_canaries() -> list[str]:
    """Names of the live symmetric buffers whose guard tail changed (dead
    buffers are dropped from the registry).  Synchronizes the device."""
    bad, live = [], []
    for ref, nbytes, name in _guarded:
        full = ref()
        if full is None:
            continue
        live.append((ref, nbytes, name))
        if not tail_intact(full, nbytes):
            bad.append(name)
    _guarded[:] = live
    return bad
