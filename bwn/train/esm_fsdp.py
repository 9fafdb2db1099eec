"""ESM-2 fully-sharded data-parallel training (``contrib/esm2/train_esm_fsdp.py``).

The reference wraps the HF model in FSDP ``FULL_SHARD`` with one unit per
``EsmLayer`` and trains eagerly, masking every chosen position to ``<mask>``
and using the HF loss (mean over masked positions) (``train_esm_fsdp.py:56-67,
103-127``).  Here the same sharding uses FSDP2 ``fully_shard`` (per-parameter
DTensor shards, reduce-scatter of gradients, all-gather before each layer)
over the bwn model, whose Linears still run on the tcgen05 GEMMs once FSDP
has gathered their weights.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..config import ESM2Config


def shard_esm_fsdp(model, world: int, device_type: str = "cuda", reshard_after_forward: bool = True):
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.fsdp import fully_shard

    mesh = init_device_mesh(device_type, (world,))
    for layer in model.esm.encoder.layer:
        fully_shard(layer, mesh=mesh, reshard_after_forward=reshard_after_forward)
    fully_shard(model, mesh=mesh, reshard_after_forward=reshard_after_forward)
    return model


def mask_all_chosen(ids: torch.Tensor, cfg: ESM2Config, gen: torch.Generator, prob: float = 0.15):
    """The FSDP script's masking: chosen non-special positions all become
    ``<mask>``; labels are ``-100`` elsewhere (``train_esm_fsdp.py:76-89``)."""
    ids = ids.clone()
    labels = ids.clone()
    special = (ids == cfg.cls_token_id) | (ids == cfg.eos_token_id) | (ids == cfg.pad_token_id)
    chosen = torch.bernoulli(torch.full(ids.shape, prob).masked_fill(special, 0.0), generator=gen).bool()
    labels[~chosen] = -100
    ids[chosen] = cfg.mask_token_id
    return ids, labels


def hf_mlm_loss(logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    """HF ``EsmForMaskedLM`` loss: cross entropy over labelled positions."""
    return F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), labels.reshape(-1).long(), ignore_index=-100)


def main(argv=None) -> None:
    """FSDP MLM fine-tuning command (``contrib/esm2/train_esm_fsdp.py:85-166``):
    the model sharded per layer over every rank, AdamW, masking of every chosen
    position, the HF loss; logs loss per step and steps/s.  Synthetic protein
    batches, or ``--fasta`` sequences.

        torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m bwn.train.esm_fsdp --model-size 3B
    """
    import argparse
    import json
    import time

    from ..config import ESM2_SIZES
    from ..parallel.comm import init_distributed
    from .esm_data import SequenceBatches, load_fasta
    from .esm_mlm import build_esm, synthetic_batch

    ap = argparse.ArgumentParser(description="ESM-2 MLM fine-tuning with FSDP")
    ap.add_argument("--model-size", default="3B", choices=sorted(ESM2_SIZES))
    ap.add_argument("--num-steps", type=int, default=10)
    ap.add_argument("--batch-size", type=int, default=2, help="sequences per rank")
    ap.add_argument("--max-seq-len", type=int, default=128)
    ap.add_argument("--lr", type=float, default=5e-5)
    ap.add_argument("--fasta", default=None)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-compile", action="store_true", help="accepted for the reference's command line: steps always run eagerly")
    ap.add_argument("--cpu", action="store_true")
    a = ap.parse_args(argv)

    cpu = a.cpu or not torch.cuda.is_available()
    comm = init_distributed("gloo" if cpu else "nccl")
    dev = torch.device("cpu") if cpu else torch.device("cuda", torch.cuda.current_device())
    model = build_esm(a.model_size, device=dev, seed=a.seed)
    cfg = model.cfg
    if comm.size > 1:
        model = shard_esm_fsdp(model, comm.size, device_type=dev.type)
    opt = torch.optim.AdamW(model.parameters(), lr=a.lr, foreach=False)
    gen = torch.Generator().manual_seed(a.seed + comm.rank)
    data = SequenceBatches(load_fasta(a.fasta), cfg, a.batch_size, a.max_seq_len, seed=a.seed + comm.rank) \
        if a.fasta else None
    log = (lambda **kv: print(json.dumps(kv), flush=True)) if comm.rank == 0 else (lambda **kv: None)
    n_params = sum(p.numel() for p in model.parameters())
    log(event="start", model=a.model_size, world=comm.size, local_params=n_params)
    t0 = time.perf_counter()
    loss = None
    for step in range(a.num_steps):
        ids, am = data.sample() if data is not None else synthetic_batch(cfg, a.batch_size, a.max_seq_len - 2, gen)
        ids, labels = mask_all_chosen(ids, cfg, gen)
        opt.zero_grad()
        loss = hf_mlm_loss(model(ids.to(dev), am.to(dev)), labels.to(dev))
        loss.backward()
        opt.step()
        log(event="step", step=step, loss=round(float(loss), 4), elapsed_s=round(time.perf_counter() - t0, 2))
    dt = time.perf_counter() - t0
    log(event="done", steps=a.num_steps, seconds=round(dt, 2), steps_per_s=round(a.num_steps / dt, 3),
        samples_per_s=round(a.num_steps * a.batch_size * comm.size / dt, 2))
    if comm.size > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
