"""Qwen3.6 sparse MoE block: softmax router -> top-k -> renormalise, routed
SwiGLU experts, sigmoid-gated shared expert (HF ``Qwen3_5MoeSparseMoeBlock``;
reference ``moe_forward`` ``contrib/qwen3.6-35b-a3b/static_decode_35b.py:701-833``
and ``_moe`` ``:1110-1185``).

Expert layout across the tensor-parallel ranks: each rank holds ``E/tp``
experts (``moe_sharding="ep"``) or a ``1/tp`` slice of every expert's
intermediate width (``"tp"``, the reference's MOE_DECODE_TP, balanced however
the tokens route); in both, each rank holds the ``1/tp`` slice of the shared
expert.  The function returns this rank's partial output; the
caller's reduction (the reference's EP combine by all-reduce, or the fused
all-to-all path of :mod:`bwn.parallel.ep`) sums the partials.
"""
from __future__ import annotations

import torch

from .. import ops as O
from ..ops import reference as R


def route(model, L, h: torch.Tensor):
    """Router logits (fp32) -> (weights [T,k] fp32, ids [T,k] int32)."""
    cfg = model.cfg
    if h.is_cuda:
        logits = O.linear_f32(h, L["router"])
        return O.moe_topk_softmax(logits, cfg.top_k, cfg.norm_topk_prob)
    logits = h.float() @ L["router"].float().t()
    return R.moe_route_softmax(logits, cfg.top_k, cfg.norm_topk_prob)


def qwen_moe_forward(model, L, h: torch.Tensor) -> torch.Tensor:
    """This rank's partial MoE output ``[T, H]`` (bf16): routed experts held
    locally plus this rank's tensor-parallel slice of the gated shared expert."""
    d = model.d
    act = O.linear_swiglu(h, L["shared_gate_up"])
    sy = O.linear(act, L["shared_down"])
    sg = O.linear_f32(h, L["shared_gate"])
    if model.moe_shared_only:  # cost probe (the reference's MOE_SHARED_ONLY): routed experts skipped
        return (torch.sigmoid(sg.float().reshape(-1, 1)) * sy.float()).to(h.dtype)
    w, ids = route(model, L, h)
    return O.moe_experts(h, w, ids, L["experts_gate_up"], L["experts_down"], d.expert_offset, shared=(sy, sg))
