"""Structured run metrics: one JSON object per line.

Every rank records its own timings; :meth:`MetricsLog.reduce_max` turns a
per-rank value into the max over ranks (the only multi-GPU number reported).
The reference prints rank-0 summaries only (``static_decode_35b.py:3088-3097``);
the printed one-line summaries stay in the drivers.
"""
from __future__ import annotations

import json
import os
import time

import torch


class MetricsLog:
    def __init__(self, path: str | None, comm=None, run: dict | None = None):
        self.comm = comm
        self.rank = comm.rank if comm is not None else 0
        self.path = path
        self.records: list[dict] = []
        if run:
            self.log("run", **run)

    def reduce_max(self, v: float) -> float:
        if self.comm is None or self.comm.size == 1:
            return float(v)
        return float(self.comm.max_scalar(float(v)))

    def log(self, event: str, **fields) -> dict:
        rec = {"t": time.time(), "event": event, "rank": self.rank, **fields}
        if torch.cuda.is_available() and torch.cuda.is_initialized():
            rec["peak_mem_gb"] = round(torch.cuda.max_memory_allocated() / 1e9, 3)
        self.records.append(rec)
        if self.path and self.rank == 0:
            d = os.path.dirname(self.path)
            if d:
                os.makedirs(d, exist_ok=True)
            with open(self.path, "a") as f:
                f.write(json.dumps(rec, default=str) + "\n")
        return rec

    def timing(self, name: str, ms: float, **fields) -> dict:
        """Log ``name`` as the max over ranks of ``ms`` (every rank must call)."""
        return self.log(name, ms=self.reduce_max(ms), ms_local=ms, **fields)


def read_jsonl(path: str) -> list[dict]:
    with open(path) as f:
        return [json.loads(line) for line in f if line.strip()]
