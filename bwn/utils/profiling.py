"""Profiling helpers: NVTX ranges and the constant-token profile loop.

The reference's ``PROFILE_STEPS=N`` runs warm-up and then N constant-token
decode steps so a device trace holds nothing else
(``contrib/qwen3.6-27b/static_decode.py:1344-1371``); :func:`profile_steps`
is that loop over a captured :class:`~bwn.runtime.static_decode.StaticDecoder`.
NVTX ranges (``BWN_NVTX=1``) label layers and ops for timeline tools.
"""
from __future__ import annotations

import contextlib

import torch

from . import env


@contextlib.contextmanager
def nvtx(name: str):
    on = env.get("BWN_NVTX") and torch.cuda.is_available()
    if on:
        torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        if on:
            torch.cuda.nvtx.range_pop()


def profile_steps(decoder, n: int, warmup: int = 3) -> float:
    """Replay ``warmup`` + ``n`` decode steps (a captured step runs the same
    kernels whatever the token values); returns ms per step over the ``n``
    steps (CUDA events)."""
    for _ in range(warmup):
        decoder.step_device()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with nvtx(f"profile_steps[{n}]"):
        a.record()
        for _ in range(n):
            decoder.step_device()
        b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / max(n, 1)
