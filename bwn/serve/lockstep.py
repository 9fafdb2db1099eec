"""Serving a tensor / expert-parallel model: one engine per rank, in lockstep.

Every rank holds its shard of the model and an identical
:class:`~bwn.serve.continuous.ContinuousEngine`; only rank 0 talks HTTP.
Before each engine step rank 0 broadcasts the requests admitted since the last
step over a CPU (gloo) control group; every follower adds the same requests in
the same order and runs the same step, so admission, slot assignment and the
collectives inside the decode step line up across ranks.  The control group has
no deadline (a server may idle for hours); the compute group keeps its short
timeout.  (The reference's multi-core serving runs inside its vLLM fork,
``contrib/qwen3.6-27b/deploy/serve_qwen35.sh``.)
"""
from __future__ import annotations

import dataclasses
import datetime

import torch.distributed as dist


def control_group():
    """A gloo group over every rank for control messages, without a deadline."""
    return dist.new_group(backend="gloo", timeout=datetime.timedelta(days=365))


class LockstepEngine:
    """Rank 0's handle: the ContinuousEngine API, broadcasting each step's new
    requests (and aborts / stop) to the followers first."""

    def __init__(self, engine, group):
        self.e, self.group = engine, group
        self.pending = []
        self.max_batch = engine.max_batch

    @property
    def stats(self):
        return self.e.stats

    def add(self, req) -> int:
        rid = self.e.add(req)  # a request the engine rejects is not sent
        self.pending.append(dataclasses.replace(req, on_token=None))  # callbacks stay on rank 0
        return rid

    def idle(self) -> bool:
        return self.e.idle()

    def _send(self, kind: str, reqs=()):
        dist.broadcast_object_list([(kind, list(reqs))], src=0, group=self.group)

    def step(self):
        reqs, self.pending = self.pending, []
        self._send("step", reqs)
        return self.e.step()

    def abort_all(self) -> None:
        self.pending = []
        self._send("abort")
        self.e.abort_all()

    def stop(self) -> None:
        self._send("stop")


class LockstepBatchEngine:
    """Rank 0's handle of a batch engine (static or speculative): each batch is
    broadcast, then generated on every rank."""

    def __init__(self, engine, group):
        self.e, self.group = engine, group
        self.max_batch = engine.max_batch

    def generate(self, reqs):
        sent = [dataclasses.replace(r, on_token=None) for r in reqs]
        dist.broadcast_object_list([("generate", sent)], src=0, group=self.group)
        return self.e.generate(reqs)

    def stop(self) -> None:
        dist.broadcast_object_list([("stop", [])], src=0, group=self.group)


def follow(engine, group) -> None:
    """A follower rank: replay rank 0's requests and steps (or batches) until
    it stops.  A batch the engine rejects is rejected on every rank alike; a
    step that fails here fails on rank 0 too, which then broadcasts an abort,
    so the follower stays in its loop instead of leaving rank 0 waiting."""
    while True:
        msg = [None]
        dist.broadcast_object_list(msg, src=0, group=group)
        kind, reqs = msg[0]
        if kind == "stop":
            return
        if kind == "abort":
            engine.abort_all()
        elif kind == "generate":
            try:
                engine.generate(reqs)
            except ValueError:
                pass
        else:
            try:
                for r in reqs:
                    engine.add(r)
                engine.step()
            except Exception:  # noqa: BLE001 - rank 0 fails the same step and broadcasts "abort"
                engine.abort_all()
