"""ESM-2 masked-language-model fine-tuning (``contrib/esm2/train_esm.py``).

* synthetic protein batches (uniform over the 20 standard amino acids, with
  ``<cls>``/``<eos>``), BERT masking 15% with the 80/10/10 mask/random/keep split
  (``mask_tokens``, ``train_esm.py:93-116``);
* AdamW (wd 0.01) on fp32 master weights, bf16 GEMMs, cosine LR with warmup
  (``get_cosine_schedule_with_warmup``, ``:136-143``);
* loss over masked positions divided by all positions (the reference's static
  divisor, ``forward_with_loss`` ``:231-245``) or by masked positions;
* data parallelism: gradients averaged across ranks (NCCL baseline, or the
  fused NVLink reduce of :mod:`bwn.parallel.grad_reduce`);
* checkpoint / resume of model, optimizer, schedule, step and RNG
  (``save_checkpoint`` / ``load_checkpoint``, ``:148-178``).
"""
from __future__ import annotations

import math
import os
from dataclasses import asdict, dataclass

import torch

from ..config import ESM2_SIZES, ESM_ALPHABET, ESM_STANDARD_AA, ESM2Config
from ..models.esm2 import EsmForMaskedLM, mlm_loss

AA_IDS = [ESM_ALPHABET.index(a) for a in ESM_STANDARD_AA]


@dataclass
class MLMConfig:
    model: str = "8M"
    batch: int = 8
    seq_len: int = 256          # residues per sequence (BOS/EOS added)
    lr: float = 1e-4
    weight_decay: float = 0.01
    warmup: int = 10
    total_steps: int = 1000
    mask_prob: float = 0.15
    loss_divisor: str = "tokens"
    seed: int = 0
    bf16: bool = True


def synthetic_batch(cfg: ESM2Config, batch: int, seq_len: int, gen: torch.Generator):
    """``[B, seq_len+2]`` ids: ``<cls>`` + uniform amino acids + ``<eos>``."""
    aa = torch.tensor(AA_IDS)[torch.randint(0, len(AA_IDS), (batch, seq_len), generator=gen)]
    ids = torch.cat([torch.full((batch, 1), cfg.cls_token_id), aa, torch.full((batch, 1), cfg.eos_token_id)], 1)
    return ids, torch.ones_like(ids)


def mask_tokens(ids: torch.Tensor, cfg: ESM2Config, gen: torch.Generator, mask_prob: float = 0.15):
    """BERT masking: choose ``mask_prob`` of non-special positions; of those 80%
    -> ``<mask>``, 10% -> random token, 10% unchanged.  Returns
    ``(input_ids, labels, loss_mask)`` with labels clamped to valid ids."""
    ids = ids.clone()
    labels = ids.clone()
    special = (ids == cfg.cls_token_id) | (ids == cfg.eos_token_id) | (ids == cfg.pad_token_id)
    prob = torch.full(ids.shape, mask_prob).masked_fill(special, 0.0)
    chosen = torch.bernoulli(prob, generator=gen).bool()
    replace = torch.bernoulli(torch.full(ids.shape, 0.8), generator=gen).bool() & chosen
    ids[replace] = cfg.mask_token_id
    rand = torch.bernoulli(torch.full(ids.shape, 0.5), generator=gen).bool() & chosen & ~replace
    ids[rand] = torch.randint(cfg.vocab, ids.shape, generator=gen)[rand]
    return ids, labels, chosen.float()


def cosine_with_warmup(step: int, warmup: int, total: int) -> float:
    if step < warmup:
        return float(step + 1) / float(max(1, warmup))
    prog = float(step - warmup) / float(max(1, total - warmup))
    return max(0.0, 0.5 * (1.0 + math.cos(math.pi * min(1.0, prog))))


class MLMTrainer:
    def __init__(self, model: EsmForMaskedLM, tcfg: MLMConfig, comm=None, grad_reducer=None):
        self.model = model
        self.cfg = tcfg
        self.comm = comm
        self.grad_reducer = grad_reducer
        self.step_idx = 0
        self.opt = torch.optim.AdamW(model.parameters(), lr=tcfg.lr, weight_decay=tcfg.weight_decay,
                                     betas=(0.9, 0.999), eps=1e-8)
        self.sched = torch.optim.lr_scheduler.LambdaLR(
            self.opt, lambda s: cosine_with_warmup(s, tcfg.warmup, tcfg.total_steps))
        self.gen = torch.Generator().manual_seed(tcfg.seed + (comm.rank if comm else 0))

    def next_batch(self):
        mcfg = self.model.cfg
        ids, am = synthetic_batch(mcfg, self.cfg.batch, self.cfg.seq_len, self.gen)
        ids, labels, lm = mask_tokens(ids, mcfg, self.gen, self.cfg.mask_prob)
        return ids, am, labels, lm

    def loss(self, ids, am, labels, lm):
        # residual stream and LayerNorms in fp32; every Linear runs on the bf16
        # tcgen05 GEMMs (forward and backward) when the model is on a GPU
        logits = self.model(ids, am)
        return mlm_loss(logits, labels, lm, self.cfg.loss_divisor)

    def step(self, batch=None) -> torch.Tensor:
        dev = next(self.model.parameters()).device
        ids, am, labels, lm = [t.to(dev, non_blocking=True) for t in (batch or self.next_batch())]
        # a bucketed reducer owns the gradient storage: zero it in place
        self.opt.zero_grad(set_to_none=self.grad_reducer is None)
        loss = self.loss(ids, am, labels, lm)
        loss.backward()
        if self.comm is not None and self.comm.size > 1:
            if self.grad_reducer is not None:
                self.grad_reducer.finish()
            else:
                for p in self.model.parameters():
                    if p.grad is not None:
                        self.comm.all_reduce_(p.grad)
                        p.grad.div_(self.comm.size)
        self.opt.step()
        self.sched.step()
        self.step_idx += 1
        return loss.detach()

    @torch.no_grad()
    def evaluate(self, batches: int = 2) -> dict:
        gen = torch.Generator().manual_seed(12345)
        dev = next(self.model.parameters()).device
        tot = 0.0
        for _ in range(batches):
            ids, am = synthetic_batch(self.model.cfg, self.cfg.batch, self.cfg.seq_len, gen)
            ids, labels, lm = mask_tokens(ids, self.model.cfg, gen, self.cfg.mask_prob)
            tot += float(self.loss(ids.to(dev), am.to(dev), labels.to(dev), lm.to(dev)))
        loss = tot / batches
        return {"loss": loss, "perplexity": math.exp(min(loss, 50.0))}

    # ------------------------------------------------------------ checkpoint
    def state_dict(self) -> dict:
        return {
            "model": {k: v.detach().cpu() for k, v in self.model.state_dict().items()},
            "optim": self.opt.state_dict(),
            "sched": self.sched.state_dict(),
            "step": self.step_idx,
            "rng": self.gen.get_state(),
            "torch_rng": torch.get_rng_state(),
            "config": asdict(self.cfg),
        }

    def save(self, path: str) -> None:
        """Atomic save (write to a temp file, then rename)."""
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        tmp = path + ".tmp"
        torch.save(self.state_dict(), tmp)
        os.replace(tmp, path)

    def load(self, path: str) -> None:
        ck = torch.load(path, map_location="cpu", weights_only=False)
        self.model.load_state_dict(ck["model"])
        self.opt.load_state_dict(ck["optim"])
        self.sched.load_state_dict(ck["sched"])
        self.step_idx = ck["step"]
        self.gen.set_state(ck["rng"])
        torch.set_rng_state(ck["torch_rng"])


def build_esm(size: str = "8M", device="cpu", seed: int = 0) -> EsmForMaskedLM:
    return EsmForMaskedLM(ESM2_SIZES[size]).init_weights(seed).to(device)
