"""Static-batch generation engine over the CUDA-graph decoder.

The reference serves through a vLLM fork (``contrib/qwen3.6-27b/deploy/serve_qwen35.sh``,
``serve_eagle3.sh``: greedy sampling, fixed batch/sequence buckets).  This engine
is the same contract in-process: requests are grouped into a batch of at most
``max_batch`` rows, prompts are right-padded to one length (``valid_len`` keeps
pad rows out of every state), one prefill, then greedy decode steps of the
captured graph until every row has its tokens or its stop id.  Unused rows of a
partial batch ride along and are discarded.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Callable

import torch

from ..runtime.static_decode import StaticDecoder


@dataclass
class Request:
    prompt: list[int]
    max_tokens: int = 16
    stop: list[int] = field(default_factory=list)
    temperature: float = 0.0  # 0: greedy; > 0: sampled (engines built with sampling=True)
    # called with each new token id as the continuous engine produces it (streaming);
    # engines that finish a request at once leave it to the caller
    on_token: Callable[[int], None] | None = field(default=None, compare=False, repr=False)
    # multi-token stop sequences: generation stops once the output ends with one of them
    stop_seqs: list[list[int]] = field(default_factory=list)

    def stopped(self, tokens: list[int]) -> bool:
        """Whether ``tokens`` (generated so far) end with a stop id or a stop sequence."""
        if not tokens:
            return False
        if tokens[-1] in self.stop:
            return True
        return any(q and len(tokens) >= len(q) and tokens[-len(q):] == q for q in self.stop_seqs)


@dataclass
class Result:
    tokens: list[int]
    finish_reason: str  # "length" | "stop"
    prefill_ms: float
    decode_ms: float


class GenerationEngine:
    def __init__(self, model, max_batch: int, max_seq: int, use_graph: bool = True, pad_to: int = 64):
        self.model = model
        self.max_batch = max_batch
        self.max_seq = max_seq
        self.pad_to = pad_to
        self.dec = StaticDecoder(model, max_batch, max_seq, use_graph=use_graph)
        self.dec.capture()
        self.dev = model.device

    def _sync(self):
        if self.dev.type == "cuda":
            torch.cuda.synchronize(self.dev)

    def generate(self, reqs: list[Request]) -> list[Result]:
        if not reqs:
            return []
        if any(r.temperature > 0 for r in reqs):
            raise ValueError("the static-batch engine is greedy; sampling runs on the continuous scheduler")
        if len(reqs) > self.max_batch:
            out = []
            for i in range(0, len(reqs), self.max_batch):
                out += self.generate(reqs[i:i + self.max_batch])
            return out
        B = self.max_batch
        L = max(len(r.prompt) for r in reqs)
        L = (L + self.pad_to - 1) // self.pad_to * self.pad_to
        steps = max(r.max_tokens for r in reqs)
        if L + steps > self.max_seq:
            raise ValueError(f"prompt ({L} padded) + {steps} new tokens exceed max_seq {self.max_seq}")
        ids = torch.zeros(B, L, dtype=torch.long)
        valid = torch.ones(B, dtype=torch.int32)
        for i, r in enumerate(reqs):
            if not r.prompt:
                raise ValueError("empty prompt")
            ids[i, :len(r.prompt)] = torch.tensor(r.prompt)
            valid[i] = len(r.prompt)
        self.dec.reset()
        self._sync()
        t0 = time.perf_counter()
        first = self.dec.prefill(ids, valid.to(self.dev)).cpu()
        self._sync()
        t1 = time.perf_counter()
        gen = [[int(first[i])] for i in range(len(reqs))]
        done = [r.max_tokens <= 1 or r.stopped(gen[i]) for i, r in enumerate(reqs)]
        while not all(done):
            nxt = self.dec.step()
            for i, r in enumerate(reqs):
                if done[i]:
                    continue
                gen[i].append(int(nxt[i]))
                done[i] = len(gen[i]) >= r.max_tokens or r.stopped(gen[i])
        t2 = time.perf_counter()
        res = []
        for i, r in enumerate(reqs):
            toks = gen[i][:r.max_tokens]
            stop = r.stopped(toks)
            res.append(Result(toks, "stop" if stop else "length", (t1 - t0) * 1e3, (t2 - t1) * 1e3))
        return res
