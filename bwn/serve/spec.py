"""EAGLE3 speculative serving (the reference's vLLM EAGLE3 mode,
``contrib/qwen3.6-27b/deploy/serve_eagle3.sh``, ``eagle3_config.yaml``:
greedy, a 1-layer draft proposing ``num_draft`` tokens per step).

Requests are grouped by prompt length (the speculative step verifies the same
number of rows for every sequence of a batch from a shared start) into
batches of at most ``max_batch``; each batch runs
:class:`~bwn.runtime.spec_decode.SpecDecoder` steps until every row has its
``max_tokens`` or a stop id.  Greedy speculation emits exactly the target's
greedy tokens, so results equal plain greedy generation; the draft only
changes how many tokens each step yields (reported as ``accepted_per_step``).
"""
from __future__ import annotations

import time
from collections import defaultdict

from ..runtime.spec_decode import SpecDecoder
from .engine import Request, Result


class SpecEngine:
    def __init__(self, model, draft, max_batch: int, max_seq: int, num_draft: int = 4, use_graph: bool = True):
        self.model, self.draft = model, draft
        self.max_batch, self.max_seq, self.num_draft = max_batch, max_seq, num_draft
        self.use_graph = use_graph
        self._decoders: dict[int, SpecDecoder] = {}  # one captured decoder per batch size
        self.stats = {"batches": 0, "steps": 0, "accepted_drafts": 0}

    def _decoder(self, b: int) -> SpecDecoder:
        d = self._decoders.get(b)
        if d is None:
            d = SpecDecoder(self.model, self.draft, b, self.max_seq, self.num_draft, use_graph=self.use_graph)
            d.capture()
            self._decoders[b] = d
        return d

    def generate(self, reqs: list[Request]) -> list[Result]:
        for r in reqs:
            if not r.prompt:
                raise ValueError("empty prompt")
            if r.temperature > 0:
                raise ValueError("speculative serving is greedy")
            if len(r.prompt) + r.max_tokens + self.num_draft + 1 > self.max_seq:
                raise ValueError(f"prompt ({len(r.prompt)}) + {r.max_tokens} new tokens exceed max_seq {self.max_seq}")
        groups: dict[int, list[int]] = defaultdict(list)
        for i, r in enumerate(reqs):
            groups[len(r.prompt)].append(i)
        out: list[Result | None] = [None] * len(reqs)
        for idx in groups.values():
            for c in range(0, len(idx), self.max_batch):
                part = idx[c:c + self.max_batch]
                for i, res in zip(part, self._run([reqs[i] for i in part])):
                    out[i] = res
        return out

    def _run(self, reqs: list[Request]) -> list[Result]:
        import torch
        dec = self._decoder(len(reqs))
        dec.reset()
        t0 = time.perf_counter()
        first = dec.prefill(torch.tensor([r.prompt for r in reqs], dtype=torch.long)).cpu().tolist()
        t1 = time.perf_counter()
        gen = [[int(x)] for x in first]
        done = [len(g) >= r.max_tokens or r.stopped(g) for g, r in zip(gen, reqs)]
        steps = 0
        while not all(done):
            ids, cnt = dec.step()
            steps += 1
            for b, r in enumerate(reqs):
                if done[b]:
                    continue
                for x in ids[b, :int(cnt[b])].tolist():
                    gen[b].append(int(x))
                    if len(gen[b]) >= r.max_tokens or r.stopped(gen[b]):
                        done[b] = True
                        break
        t2 = time.perf_counter()
        self.stats["batches"] += 1
        self.stats["steps"] += steps
        self.stats["accepted_drafts"] += int(dec.accepted_total.sum())
        res = []
        for g, r in zip(gen, reqs):
            toks = g[:r.max_tokens]
            stop = r.stopped(toks)
            res.append(Result(toks, "stop" if stop else "length", (t1 - t0) * 1e3, (t2 - t1) * 1e3))
        return res
