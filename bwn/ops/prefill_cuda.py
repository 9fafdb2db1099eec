"""CUDA prefill ops: chunked DeltaNet (dn_prefill_prep + dn_chunk + ring
update) and the prefix-aware tcgen05 flash attention (prep + flash_prefill)."""
from __future__ import annotations

import torch

from ._ext import ops


def deltanet_prefill(qkv, z, a, b, conv_ring, state, start_pos, valid_len, conv_w, A_log, dt_bias, norm_w,
                     k_heads, eps):
    vl = valid_len.to(device=qkv.device, dtype=torch.int32).contiguous()
    return ops().deltanet_prefill(qkv, z, a, b, conv_ring, state, int(start_pos), vl, conv_w, A_log, dt_bias, norm_w,
                                  k_heads, eps)


def gqa_prefill(qg, k, v, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, start_pos, eps):
    return ops().gqa_prefill(qg, k, v, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, int(start_pos), eps)
