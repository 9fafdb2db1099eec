"""In-flight (continuous) batching over the CUDA-graph decoder.

The reference serves through a vLLM fork whose scheduler admits requests into
a running batch (``contrib/qwen3.6-27b/deploy/serve_qwen35.sh``,
``VLLM_NEURON_ASSESSMENT.md``).  Here the decode step stays one captured CUDA
graph over ``max_batch`` static rows ("slots"):

* a waiting request is admitted into a free slot between decode steps: the
  slot's state rows are reset and the prompt is prefilled through a batch-1
  view of the static state (its own start position), so the other slots keep
  their sequences;
* every decode step advances all slots; a slot leaves the batch as soon as its
  request reaches ``max_tokens`` or a stop id, and the next request can take
  it on the following step;
* idle slots still ride in the fixed-shape step; their positions are pinned to
  0 before each step so they never write past their cache rows;
* with ``sampling=True`` each slot samples at its request's temperature
  (Gumbel-max on the sharded head, :meth:`~bwn.models.qwen36.Qwen36Model.sample`);
  temperature 0 stays greedy.

Greedy outputs are those of the request run alone (tested on CPU).
"""
from __future__ import annotations

import itertools
import time
from collections import deque
from dataclasses import dataclass, field

import torch

from ..runtime.static_decode import StaticDecoder
from .engine import Request, Result


@dataclass
class _Slot:
    rid: int
    req: Request
    tokens: list[int] = field(default_factory=list)
    t_admit: float = 0.0
    prefill_ms: float = 0.0


def _row_view(st, r: int):
    """A batch-1 state whose tensors are views of row ``r`` (prefill writes in place)."""
    return type(st)(conv=st.conv[:, r:r + 1], ssm=st.ssm[:, r:r + 1], k_cache=st.k_cache[:, r:r + 1],
                    v_cache=st.v_cache[:, r:r + 1], positions=st.positions[r:r + 1])


class ContinuousEngine:
    def __init__(self, model, max_batch: int, max_seq: int, use_graph: bool = True, bucket: int = 0,
                 sampling: bool = False, seed: int = 0):
        self.model = model
        self.max_batch = max_batch
        self.max_seq = max_seq
        self.bucket = bucket
        self.sampling = sampling
        self.dec = StaticDecoder(model, max_batch, max_seq, use_graph=use_graph, sampling=sampling, seed=seed)
        self.dec.capture()
        self.dev = model.device
        self.slots: list[_Slot | None] = [None] * max_batch
        self.waiting: deque[tuple[int, Request]] = deque()
        self._ids = itertools.count()
        self.stats = {"admitted": 0, "finished": 0, "steps": 0}
        self._idle_key: tuple = ()
        self._idle_idx = None

    # ----------------------------------------------------------------- API
    def add(self, req: Request) -> int:
        """Queue a request; returns its id."""
        if not req.prompt:
            raise ValueError("empty prompt")
        if req.temperature > 0 and not self.sampling:
            raise ValueError("temperature > 0 needs an engine built with sampling=True")
        if len(req.prompt) + req.max_tokens > self.max_seq:
            raise ValueError(f"prompt ({len(req.prompt)}) + {req.max_tokens} new tokens exceed max_seq {self.max_seq}")
        rid = next(self._ids)
        self.waiting.append((rid, req))
        return rid

    def idle(self) -> bool:
        return not self.waiting and all(s is None for s in self.slots)

    def step(self) -> list[tuple[int, Result]]:
        """Admit waiting requests into free slots, run one decode step over the
        batch, return the requests that finished (``(id, Result)``)."""
        done: list[tuple[int, Result]] = []
        for r in range(self.max_batch):
            if self.slots[r] is None and self.waiting:
                rid, req = self.waiting.popleft()
                fin = self._admit(r, rid, req)
                if fin is not None:
                    done.append(fin)
        active = [r for r, s in enumerate(self.slots) if s is not None]
        if not active:
            return done
        idle = tuple(r for r in range(self.max_batch) if self.slots[r] is None)
        if idle:  # keep idle rows inside their caches
            if idle != self._idle_key:  # the index tensor changes only when a slot fills or frees
                self._idle_key, self._idle_idx = idle, torch.tensor(idle, device=self.dev)
            self.dec.st.positions.index_fill_(0, self._idle_idx, 0)
        t0 = time.perf_counter()
        nxt = self.dec.step()  # device tokens already hold every slot's last id
        self.stats["steps"] += 1
        dt = (time.perf_counter() - t0) * 1e3
        for r in active:
            s = self.slots[r]
            s.tokens.append(int(nxt[r]))
            if s.req.on_token is not None:
                s.req.on_token(s.tokens[-1])
            fin = self._maybe_finish(r, dt)
            if fin is not None:
                done.append(fin)
        return done

    def abort_all(self) -> None:
        """Drop every waiting and running request (after an error)."""
        self.slots = [None] * self.max_batch
        self.waiting.clear()

    def run(self, reqs: list[Request]) -> list[Result]:
        """Convenience: serve ``reqs`` to completion, results in input order."""
        ids = [self.add(q) for q in reqs]
        out: dict[int, Result] = {}
        while not self.idle():
            for rid, res in self.step():
                out[rid] = res
        return [out[i] for i in ids]

    # ------------------------------------------------------------- internals
    def _admit(self, r: int, rid: int, req: Request):
        st = self.dec.st
        st.reset(rows=[r])
        t0 = time.perf_counter()
        prompt = torch.tensor([req.prompt], dtype=torch.long, device=self.dev)
        if self.sampling:
            self.dec.temperature[r] = float(req.temperature)
        if req.temperature > 0:  # the first token is sampled as well
            view = _row_view(st, r)
            S, bucket = prompt.shape[1], self.bucket or prompt.shape[1]
            for c0 in range(0, S, bucket):
                h = self.model.prefill_hidden(prompt[:, c0:c0 + bucket], view, None)
            first = self.model.sample(h, self.dec.temperature[r:r + 1], self.dec.gen)
        else:
            first = self.model.prefill(prompt, _row_view(st, r), None, self.bucket)
        self.dec.tokens[r:r + 1].copy_(first.to(self.dec.tokens.dtype))
        tok = int(first[0])
        ms = (time.perf_counter() - t0) * 1e3
        self.slots[r] = _Slot(rid, req, [tok], time.perf_counter(), ms)
        self.stats["admitted"] += 1
        if req.on_token is not None:
            req.on_token(tok)
        return self._maybe_finish(r, 0.0)

    def _maybe_finish(self, r: int, step_ms: float):
        s = self.slots[r]
        if len(s.tokens) < s.req.max_tokens and not s.req.stopped(s.tokens):
            return None
        toks = s.tokens[:s.req.max_tokens]
        stop = s.req.stopped(toks)
        decode_ms = (time.perf_counter() - s.t_admit) * 1e3
        self.slots[r] = None
        self.stats["finished"] += 1
        return s.rid, Result(toks, "stop" if stop else "length", s.prefill_ms, decode_ms)
