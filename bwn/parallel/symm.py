"""Symmetric-memory helpers shared by the fused collective paths."""
from __future__ import annotations


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
