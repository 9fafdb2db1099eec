"""ESM-2 masked-language-model fine-tuning (``contrib/esm2/train_esm.py``).

* FASTA data with a held-out eval split (:mod:`bwn.train.esm_data`) or
  synthetic protein batches (uniform over the 20 standard amino acids, with
  ``<cls>``/``<eos>``); BERT masking 15% with the 80/10/10 mask/random/keep split
  (``mask_tokens``, ``train_esm.py:93-116``);
* AdamW (wd 0.01) on fp32 master weights, bf16 GEMMs, cosine LR with warmup
  (``get_cosine_schedule_with_warmup``, ``:136-143``);
* loss over masked positions divided by all positions (the reference's static
  divisor, ``forward_with_loss`` ``:231-245``) or by masked positions;
* data parallelism: gradients averaged across ranks (NCCL baseline, or the
  fused NVLink reduce of :mod:`bwn.parallel.grad_reduce`);
* checkpoint / resume of model, optimizer, schedule, step and RNG
  (``save_checkpoint`` / ``load_checkpoint``, ``:148-178``);
* :func:`main`: the training command (``run_training`` ``:250-370``):
  periodic evaluation with perplexity, periodic and final checkpoints, resume.

    python -m bwn.train.esm_mlm --model-size 8M --fasta seqs.fasta --num-steps 100
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m bwn.train.esm_mlm --model-size 15B --parallel tp
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
    """One optimizer step per :meth:`step`.  ``data`` / ``eval_data``
    (:class:`~bwn.train.esm_data.SequenceBatches`) supply real sequences;
    without them the batches are synthetic."""

    def __init__(self, model: EsmForMaskedLM, tcfg: MLMConfig, comm=None, grad_reducer=None, data=None,
                 eval_data=None):
        self.model = model
        self.cfg = tcfg
        self.comm = comm
        self.grad_reducer = grad_reducer
        self.data = data
        self.eval_data = eval_data
        self.step_idx = 0
        self.opt = torch.optim.AdamW(model.parameters(), lr=tcfg.lr, weight_decay=tcfg.weight_decay,
                                     betas=(0.9, 0.999), eps=1e-8)
        self.sched = torch.optim.lr_scheduler.LambdaLR(
            self.opt, lambda s: cosine_with_warmup(s, tcfg.warmup, tcfg.total_steps))
        self.gen = torch.Generator().manual_seed(tcfg.seed + (comm.rank if comm else 0))

    def next_batch(self):
        mcfg = self.model.cfg
        if self.data is not None:
            ids, am = self.data.sample()
        else:
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
        """Mean masked-LM loss and perplexity over the held-out sequences (in
        order, fixed masking seed) or ``batches`` synthetic batches."""
        gen = torch.Generator().manual_seed(12345)
        dev = next(self.model.parameters()).device
        if self.eval_data is not None:
            src = self.eval_data.sequential()
        else:
            src = (synthetic_batch(self.model.cfg, self.cfg.batch, self.cfg.seq_len, gen) for _ in range(batches))
        was_training = self.model.training
        self.model.eval()
        tot, n = 0.0, 0
        for ids, am in src:
            ids, labels, lm = mask_tokens(ids, self.model.cfg, gen, self.cfg.mask_prob)
            tot += float(self.loss(ids.to(dev), am.to(dev), labels.to(dev), lm.to(dev)))
            n += 1
        self.model.train(was_training)
        loss = tot / max(1, n)
        return {"loss": loss, "perplexity": math.exp(min(loss, 50.0))}

    # ------------------------------------------------------------ checkpoint
    def _job_comm(self):
        """The job's ranks: the data-parallel group, or the tensor-parallel one."""
        if self.comm is not None and self.comm.size > 1:
            return self.comm
        return getattr(self.model, "tp_comm", None)

    def state_dict(self) -> dict:
        """Portable checkpoint (:mod:`bwn.train.esm_ckpt`): the unsharded model
        and AdamW moments by parameter name, scheduler, step, and every rank's
        generator states.  Collective on multi-rank jobs."""
        from .esm_ckpt import full_state, gather_objects
        msd, moments = full_state(self.model, self.opt, getattr(self.model, "tp_comm", None))
        mine = {"gen": self.gen.get_state(), "data": self.data.state_dict() if self.data is not None else None}
        return {
            "format": CKPT_FORMAT,
            "model": msd,
            "moments": moments,
            "optim_groups": [{k: v for k, v in g.items() if k != "params"} for g in self.opt.param_groups],
            "sched": self.sched.state_dict(),
            "step": self.step_idx,
            "rngs": gather_objects(mine, self._job_comm()),
            # tensor-parallel ranks (and a single process) draw one shared sample stream
            "shared_stream": self.comm is None or self.comm.size <= 1,
            "torch_rng": torch.get_rng_state(),
            "config": asdict(self.cfg),
        }

    def save(self, path: str) -> None:
        """Every rank calls it; the job's rank 0 writes atomically (temp file, rename)."""
        sd = self.state_dict()
        jc = self._job_comm()
        if jc is not None and jc.rank != 0:
            return
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        tmp = path + ".tmp"
        torch.save(sd, tmp)
        os.replace(tmp, path)

    def load(self, path: str) -> None:
        """Resume from a portable checkpoint at any tensor/data-parallel degree.
        A shared sample stream (single process or tensor-parallel ranks)
        continues on any number of tensor-parallel ranks; data-parallel ranks
        continue their own streams at the saved world size; otherwise the
        generators are re-seeded from (seed, rank, step)."""
        from .esm_ckpt import load_full_state
        ck = torch.load(path, map_location="cpu", weights_only=False)
        if ck.get("format") != CKPT_FORMAT:
            raise ValueError(f"{path}: not a {CKPT_FORMAT} checkpoint")
        load_full_state(self.model, self.opt, getattr(self.model, "tp_comm", None), ck["model"], ck["moments"])
        for g, saved in zip(self.opt.param_groups, ck["optim_groups"]):
            g.update(saved)
        self.sched.load_state_dict(ck["sched"])
        self.step_idx = ck["step"]
        torch.set_rng_state(ck["torch_rng"])
        jc = self._job_comm()
        world, rank = (jc.size, jc.rank) if jc is not None else (1, 0)
        rngs = ck["rngs"]
        shared_now = self.comm is None or self.comm.size <= 1
        mine = rngs[0] if (ck.get("shared_stream") and shared_now) else rngs[rank] if len(rngs) == world else None
        if mine is not None:
            self.gen.set_state(mine["gen"])
            if self.data is not None and mine["data"] is not None:
                self.data.load_state_dict(mine["data"])
        else:
            s = self.cfg.seed * 1_000_003 + self.step_idx
            self.gen.manual_seed(s + (rank if self.comm is not None else 0))
            if self.data is not None:
                self.data.rng.seed(s + rank)


CKPT_FORMAT = "bwn-esm-portable-1"


def build_esm(size: str = "8M", device="cpu", seed: int = 0) -> EsmForMaskedLM:
    return EsmForMaskedLM(ESM2_SIZES[size]).init_weights(seed).to(device)


def main(argv=None):
    import argparse
    import json
    import time

    from ..parallel.comm import init_distributed
    from .esm_data import SequenceBatches, load_fasta, split_dataset
    from .esm_infer import DEFAULT_SEQUENCES

    ap = argparse.ArgumentParser(description="ESM-2 masked-LM fine-tuning")
    ap.add_argument("--model-size", default="8M", choices=sorted(ESM2_SIZES))
    ap.add_argument("--max-seq-len", type=int, default=128, help="tokens per sequence incl. <cls>/<eos>")
    ap.add_argument("--batch-size", type=int, default=4, help="sequences per data-parallel rank")
    ap.add_argument("--num-steps", type=int, default=100)
    ap.add_argument("--lr", type=float, default=5e-5)
    ap.add_argument("--warmup-steps", type=int, default=10)
    ap.add_argument("--fasta", default=None, help="FASTA file (train/eval split automatically)")
    ap.add_argument("--eval-fraction", type=float, default=0.1)
    ap.add_argument("--eval-every", type=int, default=25, help="0 disables")
    ap.add_argument("--log-every", type=int, default=5)
    ap.add_argument("--save-every", type=int, default=50, help="0 disables")
    ap.add_argument("--checkpoint-dir", default="./checkpoints")
    ap.add_argument("--resume", default=None, help="checkpoint directory to resume from")
    ap.add_argument("--stop-after", type=int, default=0,
                    help="end this invocation after N steps with a checkpoint (a preempted job; the schedule "
                         "still spans --num-steps); 0 runs to --num-steps")
    ap.add_argument("--parallel", default="auto", choices=["auto", "dp", "tp"],
                    help="auto: tensor-parallel for 3B/15B, data-parallel otherwise")
    ap.add_argument("--reducer", default="nccl", choices=["nccl", "fused"], help="data-parallel gradient reduction")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu", action="store_true")
    a = ap.parse_args(argv)

    comm = init_distributed("gloo" if a.cpu or not torch.cuda.is_available() else None)
    dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() and not a.cpu \
        else torch.device("cpu")
    mode = a.parallel if a.parallel != "auto" else ("tp" if a.model_size in ("3B", "15B") else "dp")
    tp = comm.size > 1 and mode == "tp"
    model = build_esm(a.model_size, device=dev, seed=a.seed)
    reducer = None
    if tp:
        from ..parallel.tensor_parallel import apply_esm_tp
        model = apply_esm_tp(model, comm)
    elif comm.size > 1 and a.reducer == "fused":
        from ..parallel.grad_reduce import GradReducer
        reducer = GradReducer(model, comm, bucket_mb=64)
    seqs = load_fasta(a.fasta) if a.fasta else list(DEFAULT_SEQUENCES)
    train, held = split_dataset(seqs, a.eval_fraction)
    mcfg = model.cfg
    # tensor-parallel ranks must see the same batch; data-parallel ranks draw their own
    data_seed = a.seed if tp else a.seed + comm.rank
    data = SequenceBatches(train, mcfg, a.batch_size, a.max_seq_len, seed=data_seed)
    eval_data = SequenceBatches(held, mcfg, a.batch_size, a.max_seq_len)
    tcfg = MLMConfig(model=a.model_size, batch=a.batch_size, seq_len=a.max_seq_len - 2, lr=a.lr,
                     warmup=a.warmup_steps, total_steps=a.num_steps, seed=a.seed)
    trainer = MLMTrainer(model, tcfg, None if tp else comm, grad_reducer=reducer, data=data, eval_data=eval_data)
    if tp:
        trainer.gen.manual_seed(a.seed)  # identical masking on every tensor-parallel rank
    log = (lambda **kv: print(json.dumps(kv), flush=True)) if comm.rank == 0 else (lambda **kv: None)
    if a.resume:
        path = os.path.join(a.resume, "checkpoint.pt")
        if os.path.exists(path):
            trainer.load(path)
            log(event="resumed", step=trainer.step_idx, path=path)
        else:
            log(event="no_checkpoint", path=path)
    log(event="start", model=a.model_size, parallel=f"tp{comm.size}" if tp else f"dp{comm.size}",
        train_sequences=len(train), eval_sequences=len(held), steps=a.num_steps, start=trainer.step_idx)

    def save():  # collective: shards are gathered, rank 0 writes
        trainer.save(os.path.join(a.checkpoint_dir, "checkpoint.pt"))

    t0 = time.perf_counter()
    start = trainer.step_idx
    end = min(a.num_steps, start + a.stop_after) if a.stop_after > 0 else a.num_steps
    total = 0.0
    for step in range(start, end):
        loss = float(trainer.step())
        total += loss
        if step % max(1, a.log_every) == 0 or step == end - 1:
            log(event="step", step=step, loss=round(loss, 4), lr=trainer.sched.get_last_lr()[0],
                elapsed_s=round(time.perf_counter() - t0, 2))
        if a.eval_every > 0 and (step + 1) % a.eval_every == 0:
            ev = trainer.evaluate()  # every rank: tensor-parallel forward passes are collective
            log(event="eval", step=step + 1, **ev)
        if a.save_every > 0 and (step + 1) % a.save_every == 0:
            save()
    dt = time.perf_counter() - t0
    n = max(1, end - start)
    if end < a.num_steps:
        save()
        log(event="stopped", step=end, seconds=round(dt, 2))
        if comm.size > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return
    ev = trainer.evaluate()
    save()
    log(event="done", steps=n, seconds=round(dt, 2), avg_loss=round(total / n, 4),
        samples_per_s=round(n * a.batch_size * (1 if tp else comm.size) / max(dt, 1e-9), 2), final_eval=ev)
    if comm.size > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
