"""Device timers: CUDA events on the launching stream, synchronised on both
sides; multi-GPU numbers are the max over ranks."""
from __future__ import annotations

import time

import torch


class CudaTimer:
    def __init__(self, device=None):
        self.cuda = torch.cuda.is_available()
        if self.cuda:
            self.start = torch.cuda.Event(enable_timing=True)
            self.end = torch.cuda.Event(enable_timing=True)

    def __enter__(self):
        if self.cuda:
            torch.cuda.synchronize()
            self.start.record()
        else:
            self.t0 = time.perf_counter()
        return self

    def __exit__(self, *exc):
        if self.cuda:
            self.end.record()
            torch.cuda.synchronize()
            self.ms = self.start.elapsed_time(self.end)
        else:
            self.ms = (time.perf_counter() - self.t0) * 1e3
        return False


def flush_l2(nbytes: int = 256 << 20, device="cuda") -> None:
    """Write a buffer larger than the 126 MB L2 so the next kernel starts cold."""
    buf = torch.empty(nbytes // 4, dtype=torch.float32, device=device)
    buf.fill_(1.0)
