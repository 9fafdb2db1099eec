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
