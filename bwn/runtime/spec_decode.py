"""EAGLE3 speculative decoding over a Qwen3.6 target (greedy).

One step, entirely on the device and captured as one CUDA graph:

1. verify: the target runs ``N = num_draft + 1`` tokens per sequence
   (``[last token, d1..dK]``) at positions ``p..p+N-1`` -- DeltaNet layers
   first commit the previous step's accepted tokens (deferred commit), GQA
   layers append K/V at the new positions;
2. accept: the longest prefix of drafts equal to the target's greedy ids,
   ``m`` drafts, plus the target's own next id (``bonus``); ``a = m + 1``
   tokens become committed, positions advance by ``a``;
3. draft: the EAGLE3 draft re-reads the N verify rows (target features of the
   accepted positions, next-token embeddings) to rebuild its KV rows, then
   drafts ``K`` tokens from row ``m`` autoregressively.

Greedy speculative decoding emits exactly the target's greedy sequence; the
draft only changes how many tokens a step yields.  The reference runs the same
loop inside vLLM (``contrib/qwen3.6-27b/deploy/serve_eagle3.sh``,
``eagle3_config.yaml``: 3 speculative tokens, verify length 4).
"""
from __future__ import annotations

import torch

from ..models.eagle3 import Eagle3Draft


def accept_greedy(tok: torch.Tensor, tgt: torch.Tensor):
    """``tok [B, N]`` verify inputs ``[t0, d1..dK]``, ``tgt [B, N]`` target greedy
    ids at those rows.  Returns ``(m [B] accepted drafts, bonus [B],
    out [B, N] emitted ids with -1 padding)`` -- emitted = ``d1..dm, bonus``."""
    B, N = tok.shape
    match = (tok[:, 1:] == tgt[:, :-1]).int()
    m = torch.cumprod(match, dim=1).sum(dim=1)  # [B]
    bonus = tgt.gather(1, m.long()[:, None])[:, 0]
    j = torch.arange(N, device=tok.device)[None]
    shifted = torch.cat([tok[:, 1:], tok[:, :1]], dim=1)
    out = torch.where(j < m[:, None], shifted, torch.where(j == m[:, None], bonus[:, None], torch.full_like(tok, -1)))
    return m.int(), bonus.int(), out.int()


class SpecDecoder:
    def __init__(self, target, draft: Eagle3Draft, batch: int, max_seq: int, num_draft: int = 4,
                 use_graph: bool = True):
        self.t, self.d = target, draft
        self.B, self.K, self.N = batch, num_draft, num_draft + 1
        dev = target.device
        self.st = target.new_state(batch, max_seq, ring_slots=8)
        self.sp = target.new_spec_state(batch, self.N)
        self.dst = draft.new_state(batch, max_seq)
        target.ensure_rope(max_seq)
        if getattr(target, "shard_embed", False):
            raise ValueError("the EAGLE3 draft reads the full embedding table; run the target with BWN_SHARD_EMBED=0")
        draft.bind_embedding(target.g["embed"])
        self.tok = torch.zeros(batch, self.N, dtype=torch.int32, device=dev)    # next verify input
        self.out = torch.full((batch, self.N), -1, dtype=torch.int32, device=dev)  # emitted this step
        self.n_out = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.accepted_total = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.steps = 0
        self.use_graph = use_graph and dev.type == "cuda"
        self.graph = None
        self._host_out = None
        self.oracle = None  # [B, T] known continuation: drafts read from it (acceptance upper bound)
        self.oracle_base = 0

    # ------------------------------------------------------------- drafting
    def _draft_from(self, r: torch.Tensor, d1: torch.Tensor, pos0: torch.Tensor) -> None:
        """Fill ``tok[:, 1:]`` with K drafts: ``d1`` already drafted by a row at
        ``pos0 - 1`` whose hidden is ``r``; each further draft row sits at
        ``pos0 + j``."""
        if self.oracle is not None:
            # benchmark mode: draft the known continuation (every draft accepted)
            idx = (pos0[:, None].long() - self.oracle_base + 1 + torch.arange(self.K, device=pos0.device)[None])
            idx = idx.clamp(0, self.oracle.shape[1] - 1)
            self.tok[:, 1:] = self.oracle.gather(1, idx)
            return
        self.tok[:, 1] = d1
        hid = r
        for j in range(1, self.K):
            hid, ids = self.d.rows(hid, self.tok[:, j], (pos0 + (j - 1)).int(), self.dst, 1)
            self.tok[:, j + 1] = ids

    def set_oracle(self, continuation: torch.Tensor, prompt_len: int) -> None:
        """Draft from a known greedy continuation ``[B, T]`` (token at position
        ``prompt_len + i`` is column ``i``) instead of the draft model: the
        all-accepted upper bound of a step, for measurement."""
        self.oracle = continuation.to(self.t.device).int().contiguous()
        self.oracle_base = prompt_len

    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """Process ``prompt [B, S]`` (shared length); returns the first generated ids."""
        t, d = self.t, self.d
        dev = t.device
        prompt = prompt.to(dev)
        B, S = prompt.shape
        feats: list[torch.Tensor] = []
        h = t.prefill_hidden(prompt, self.st, None, 64, d.cfg.feat_layers, feats)
        g0 = t.greedy(h)
        nxt = torch.cat([prompt[:, 1:].int(), g0[:, None].int()], dim=1)
        r, ids = d.prefill(d.fuse(feats), nxt, self.dst)
        last = torch.arange(B, device=dev) * S + (S - 1)
        self.tok[:, 0] = g0
        self._draft_from(r[last], ids[last], torch.full((B,), S, dtype=torch.int32, device=dev))
        self.sp.pending.zero_()
        return g0

    # ----------------------------------------------------------------- step
    def _step_body(self) -> None:
        t, d = self.t, self.d
        B, N = self.B, self.N
        p0 = self.st.positions.clone()
        h, feats = t.verify_hidden(self.tok, self.st, self.sp, d.cfg.feat_layers)
        tgt = t.greedy(h).view(B, N)
        m, bonus, out = accept_greedy(self.tok, tgt)
        a = m + 1
        self.out.copy_(out)
        self.n_out.copy_(a)
        self.accepted_total.add_(m.long())
        self.st.positions.add_(a)
        self.sp.pending.copy_(a)
        self.sp.vstep.add_(1)
        # draft: rebuild the N rows (next-token inputs: accepted drafts, then the bonus)
        j = torch.arange(N, device=p0.device)[None]
        nxt = torch.where(j < m[:, None], torch.cat([self.tok[:, 1:], self.tok[:, :1]], 1), bonus[:, None])
        rows_pos = (p0[:, None] + j).reshape(-1).int()
        r, ids = d.rows(d.fuse(feats), nxt.reshape(-1), rows_pos, self.dst, N)
        sel = torch.arange(B, device=p0.device) * N + m.long()
        self.tok[:, 0] = bonus
        self._draft_from(r[sel], ids[sel], (p0 + a).int())

    def capture(self) -> None:
        if not self.use_graph:
            return
        snap = [x.clone() for x in self._mutable()]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._step_body()  # sizes per-stream scratch before capture
            torch.cuda.synchronize()
            for x, y in zip(self._mutable(), snap):
                x.copy_(y)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=s):
                self._step_body()
        torch.cuda.current_stream().wait_stream(s)
        for x, y in zip(self._mutable(), snap):
            x.copy_(y)
        torch.cuda.synchronize()

    def reset(self) -> None:
        """Back to the state of a fresh decoder (a new batch of prompts); the
        captured graph stays valid (same buffers)."""
        self.st.reset()
        self.sp.pending.zero_()
        self.sp.vstep.zero_()
        self.tok.zero_()
        self.out.fill_(-1)
        self.n_out.zero_()
        self.accepted_total.zero_()
        self.steps = 0

    def _mutable(self):
        st, sp, ds = self.st, self.sp, self.dst
        return [st.conv, st.ssm, st.k_cache, st.v_cache, st.positions, sp.stash_qkv, sp.stash_ab, sp.pending,
                sp.vstep, ds.k_cache, ds.v_cache, self.tok, self.out, self.n_out, self.accepted_total]

    def step_device(self) -> None:
        if self.graph is not None:
            self.graph.replay()
        else:
            self._step_body()
        self.steps += 1

    def step(self):
        """One speculative step; returns host ``(ids [B, N], counts [B])`` of the
        tokens emitted this step (row b: ``ids[b, :counts[b]]``)."""
        self.step_device()
        if self._host_out is None:
            pin = self.t.device.type == "cuda"
            self._host_out = (torch.empty(self.out.shape, dtype=torch.int32, pin_memory=pin),
                              torch.empty(self.n_out.shape, dtype=torch.int32, pin_memory=pin))
        self._host_out[0].copy_(self.out, non_blocking=True)
        self._host_out[1].copy_(self.n_out, non_blocking=True)
        if self.t.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        return self._host_out

    def generate(self, prompt: torch.Tensor, max_new: int) -> list[list[int]]:
        """Greedy continuation of ``prompt`` with ``max_new`` tokens per row."""
        g0 = self.prefill(prompt).cpu().tolist()
        res = [[int(x)] for x in g0]
        while min(len(r) for r in res) < max_new:
            ids, cnt = self.step()
            for b in range(self.B):
                res[b].extend(int(x) for x in ids[b, :int(cnt[b])])
        return [r[:max_new] for r in res]

    def mean_accepted(self) -> float:
        """Mean accepted drafts per step and sequence."""
        return float(self.accepted_total.float().mean()) / max(self.steps, 1)

    def finish(self) -> None:
        """Commit the last accepted tokens (for plain decode afterwards)."""
        self.t.commit_pending(self.st, self.sp)

    def release(self) -> None:
        self.graph = None
