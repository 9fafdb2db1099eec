"""Protein sequence data for ESM-2 MLM fine-tuning (``contrib/esm2/train_esm.py``):

* :func:`load_fasta` streams a FASTA file (multi-line records, sequences
  shorter than 10 residues dropped, ``load_fasta`` ``train_esm.py:60-79``);
* :func:`split_dataset` holds out a seeded ``eval_fraction`` (at least one
  sequence, ``split_dataset`` ``:82-88``);
* :class:`SequenceBatches` draws training batches with replacement from a
  seeded generator and tokenizes them to a fixed ``max_len`` (``<cls>`` +
  residues truncated to ``max_len - 2`` + ``<eos>``, right-padded), so every
  step has the same shape (``create_batch`` ``:119-131``); the evaluation
  batches walk the held-out set in order.
"""
from __future__ import annotations

import random
from typing import Iterator

import torch

from ..config import ESM_ALPHABET, ESM2Config

MIN_RESIDUES = 10


def load_fasta(path: str, min_len: int = MIN_RESIDUES) -> list[str]:
    """Sequences of a FASTA file (header lines start with ``>``; a record's
    sequence lines are concatenated); records shorter than ``min_len`` are skipped."""
    seqs: list[str] = []
    cur: list[str] = []

    def flush():
        if cur:
            s = "".join(cur)
            if len(s) >= min_len:
                seqs.append(s)
            cur.clear()

    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            if line.startswith(">"):
                flush()
            else:
                cur.append(line)
    flush()
    return seqs


def split_dataset(seqs: list[str], eval_fraction: float = 0.1, seed: int = 42) -> tuple[list[str], list[str]]:
    """``(train, eval)``: a seeded shuffle, the first ``max(1, int(n * eval_fraction))``
    sequences held out."""
    order = list(seqs)
    random.Random(seed).shuffle(order)
    n_eval = max(1, int(len(order) * eval_fraction))
    return order[n_eval:], order[:n_eval]


def encode(seqs: list[str], cfg: ESM2Config, max_len: int) -> tuple[torch.Tensor, torch.Tensor]:
    """``(ids [B, max_len], attention_mask [B, max_len])``: ``<cls>``, residues
    (unknown letters -> ``<unk>``), ``<eos>``, ``<pad>`` to ``max_len``; a
    sequence longer than ``max_len - 2`` residues is truncated and keeps its ``<eos>``."""
    if max_len < 3:
        raise ValueError("max_len must leave room for <cls>, a residue and <eos>")
    idx = {t: i for i, t in enumerate(ESM_ALPHABET)}
    unk = idx["<unk>"]
    ids = torch.full((len(seqs), max_len), cfg.pad_token_id, dtype=torch.long)
    am = torch.zeros(len(seqs), max_len, dtype=torch.long)
    for b, s in enumerate(seqs):
        body = [idx.get(c, unk) for c in s[:max_len - 2]]
        row = [cfg.cls_token_id] + body + [cfg.eos_token_id]
        ids[b, :len(row)] = torch.tensor(row)
        am[b, :len(row)] = 1
    return ids, am


class SequenceBatches:
    """Fixed-shape tokenized batches over a list of sequences."""

    def __init__(self, seqs: list[str], cfg: ESM2Config, batch: int, max_len: int, seed: int = 0):
        if not seqs:
            raise ValueError("no sequences")
        self.seqs, self.cfg, self.batch, self.max_len = seqs, cfg, batch, max_len
        self.rng = random.Random(seed)

    def sample(self) -> tuple[torch.Tensor, torch.Tensor]:
        """``batch`` sequences drawn with replacement."""
        return encode(self.rng.choices(self.seqs, k=self.batch), self.cfg, self.max_len)

    def sequential(self) -> Iterator[tuple[torch.Tensor, torch.Tensor]]:
        """The sequences in order, ``max(1, len // batch)`` full batches (a set
        smaller than one batch gives one short batch)."""
        n = max(1, len(self.seqs) // self.batch)
        for i in range(n):
            chunk = self.seqs[i * self.batch:(i + 1) * self.batch]
            if chunk:
                yield encode(chunk, self.cfg, self.max_len)

    def state_dict(self) -> dict:
        return {"rng": self.rng.getstate()}

    def load_state_dict(self, sd: dict) -> None:
        self.rng.setstate(sd["rng"])
