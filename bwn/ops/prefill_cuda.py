"""CUDA prefill ops: chunked DeltaNet (dn_prefill_prep + dn_chunk + ring
update) and the prefix-aware tcgen05 flash attention (prep + flash_prefill).

``start_pos`` is a host int or an int32 device tensor whose element 0 is the
chunk's start position; the tensor form is read by the kernels at run time, so
no host sync is needed and one captured graph serves every chunk offset."""
from __future__ import annotations

import torch

from ._ext import ops


def _start(start_pos):
    if torch.is_tensor(start_pos):
        return 0, start_pos
    return int(start_pos), None


def deltanet_prefill(qkv, z, a, b, conv_ring, state, start_pos, valid_len, conv_w, A_log, dt_bias, norm_w,
                     k_heads, eps):
    vl = valid_len.to(device=qkv.device, dtype=torch.int32).contiguous()
    s, s_t = _start(start_pos)
    return ops().deltanet_prefill(qkv, z, a, b, conv_ring, state, s, vl, conv_w, A_log, dt_bias, norm_w,
                                  k_heads, eps, s_t)


def gqa_prefill(qg, k, v, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, start_pos, eps):
    s, s_t = _start(start_pos)
    return ops().gqa_prefill(qg, k, v, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, s, eps, s_t)
