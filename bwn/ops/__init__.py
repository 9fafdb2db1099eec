"""Public op API.  CUDA tensors run the hand-written sm_100a kernels registered
as ``torch.ops.bwn.*``; CPU tensors run the fp32 PyTorch references in
:mod:`bwn.ops.reference` (the CPU test tier and numerics oracle).

Weight layouts the kernels expect (produced by :mod:`bwn.io.loader`):

* linear weights are ``[N_out, K]`` row-major bf16 (``nn.Linear`` layout);
* SwiGLU gate/up weights are interleaved in blocks of 16 rows
  (``[g0..g15, u0..u15, g16..g31, u16..u31, ...]``) so the GEMM epilogue finds
  each gate next to its up partner (:func:`interleave_gate_up`).
"""
from __future__ import annotations

import torch

from . import reference as ref
from ._ext import available, check_status, ops, require, status, status_clear  # noqa: F401

EPI_BF16, EPI_RESID, EPI_SWIGLU, EPI_F32 = 0, 1, 2, 3


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, block: int = 16) -> torch.Tensor:
    """Pack ``gate [I, K]`` and ``up [I, K]`` into the block-16 interleaved ``[2I, K]``."""
    I, K = gate.shape
    assert I % block == 0, f"intermediate {I} must be a multiple of {block}"
    g = gate.reshape(I // block, block, K)
    u = up.reshape(I // block, block, K)
    return torch.stack([g, u], dim=1).reshape(2 * I, K)


def deinterleave_gate_up(w: torch.Tensor, block: int = 16):
    n2, K = w.shape
    x = w.reshape(n2 // (2 * block), 2, block, K)
    return x[:, 0].reshape(n2 // 2, K), x[:, 1].reshape(n2 // 2, K)


# --------------------------------------------------------------------------
# GEMMs (a weight is a bf16 [N, K] tensor or an FP8Weight: W8A16, 128x128 blocks)
# --------------------------------------------------------------------------
def _is_fp8(w) -> bool:
    return hasattr(w, "w8") and hasattr(w, "scales")


def _dense(w):
    return w.dequant() if _is_fp8(w) else w


def linear(x: torch.Tensor, w) -> torch.Tensor:
    """``x @ w.T`` (bf16 in/out, fp32 accumulate) on the tcgen05 GEMM."""
    if x.is_cuda:
        if _is_fp8(w):
            return ops().linear_w8(x, w.w8, w.scales, EPI_BF16, None)
        return ops().linear(x, w)
    return ref.linear(x, _dense(w).to(x.dtype))


def linear_into(x: torch.Tensor, w, out: torch.Tensor) -> torch.Tensor:
    """``out[:] = x @ w.T`` where ``x`` and ``out`` may be row-strided views
    (a column slice of a wider matrix): the tcgen05 GEMM reads ``x`` and writes
    ``out`` through their row strides, so no gather or concatenation is
    launched.  Views whose base or row stride is not 16-byte aligned (the TMA
    rule) go through a contiguous copy instead."""
    if x.is_cuda and not _is_fp8(w) and all(
            t.stride(1) == 1 and t.data_ptr() % 16 == 0 and t.stride(0) % 8 == 0 for t in (x, out)):
        ops().linear_out(x, w, out, EPI_BF16, None)
        return out
    out.copy_(linear(x.contiguous() if x.is_cuda else x, w))
    return out


def linear_f32(x: torch.Tensor, w) -> torch.Tensor:
    if x.is_cuda:
        if _is_fp8(w):
            return ops().linear_w8(x, w.w8, w.scales, EPI_F32, None)
        return ops().linear_f32(x, w)
    return x.float() @ _dense(w).float().t()


def linear_swiglu(x: torch.Tensor, w_il) -> torch.Tensor:
    """``silu(x @ Wg.T) * (x @ Wu.T)`` with the block-16 interleaved weight."""
    if x.is_cuda:
        if _is_fp8(w_il):
            return ops().linear_w8(x, w_il.w8, w_il.scales, EPI_SWIGLU, None)
        return ops().linear_swiglu(x, w_il)
    w_il = _dense(w_il)
    y = x.float() @ w_il.float().t()
    n2 = y.shape[-1]
    y = y.reshape(*y.shape[:-1], n2 // 32, 2, 16)
    return (torch.nn.functional.silu(y[..., 0, :]) * y[..., 1, :]).reshape(*y.shape[:-3], n2 // 2).to(x.dtype)


def linear_residual(x: torch.Tensor, w, resid: torch.Tensor) -> torch.Tensor:
    """``resid + x @ w.T`` with the add fused into the GEMM epilogue."""
    if x.is_cuda:
        if _is_fp8(w):
            return ops().linear_w8(x, w.w8, w.scales, EPI_RESID, resid)
        return ops().linear_residual(x, w, resid)
    return (x.float() @ _dense(w).float().t() + resid.float()).to(x.dtype)


def linear_bias(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``x @ w.T + b`` with the bias added in the GEMM epilogue: the residual
    epilogue reads a row stride of 0, so every output row adds the same bf16
    bias vector (one rounding, no separate elementwise kernel)."""
    if x.is_cuda:
        bb = b.to(torch.bfloat16).contiguous()
        return ops().linear_residual(x, w, bb.expand(x.shape[0], bb.shape[0]))
    return (x.float() @ _dense(w).float().t() + b.float()).to(x.dtype)


def linear_kn(x: torch.Tensor, w_kn: torch.Tensor) -> torch.Tensor:
    """``x @ w`` with ``w`` stored ``[K, N]`` (MN-major B operand); used for
    input gradients ``dX = dY @ W``."""
    if x.is_cuda:
        return ops().linear_kn(x, w_kn)
    return (x.float() @ w_kn.float()).to(x.dtype)


def matmul_tn(a_km: torch.Tensor, b_kn: torch.Tensor, f32_out: bool = False) -> torch.Tensor:
    """``a.T @ b`` for ``a [K, M]``, ``b [K, N]`` (both MN-major); used for weight
    gradients ``dW = dY.T @ X``."""
    if a_km.is_cuda:
        return ops().matmul_tn(a_km, b_kn, f32_out)
    y = a_km.float().t() @ b_kn.float()
    return y if f32_out else y.to(a_km.dtype)


# --------------------------------------------------------------------------
# norms / embedding / greedy
# --------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, one_plus: bool = True) -> torch.Tensor:
    if x.is_cuda:
        return ops().rms_norm(x, w, eps, one_plus)
    return ref.rms_norm(x, w, eps, one_plus)


def add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``residual += x`` (in place) and return ``rmsnorm(residual) * (1+w)``."""
    if x.is_cuda:
        return ops().add_rms_norm(x, residual, w, eps)
    r, n = ref.add_rms_norm(x, residual, w, eps)
    residual.copy_(r)
    return n


def embedding(ids: torch.Tensor, table: torch.Tensor, offset: int = 0) -> torch.Tensor:
    """Rows ``table[ids - offset]``; ids outside the local shard give zero rows."""
    if table.is_cuda:
        return ops().embedding(ids.int(), table, offset)
    local = ids.long() - offset
    ok = (local >= 0) & (local < table.shape[0])
    rows = table[local.clamp(0, table.shape[0] - 1)]
    return rows * ok[..., None].to(rows.dtype)


def argmax_packed(logits: torch.Tensor, id_offset: int = 0) -> torch.Tensor:
    """Per row int64 key ``((orderable(max) ^ 2^31) << 32) | (2^32-1 - id)``: a
    signed int64 max over shards (NCCL MAX all-reduce, the fused greedy) selects
    the largest logit and, on ties, the lowest global id."""
    if logits.is_cuda:
        return ops().argmax_packed(logits, id_offset)
    lf = logits.float()
    m, _ = lf.max(-1)
    ids = torch.arange(lf.shape[-1])
    first = torch.where(lf == m[:, None], ids, torch.full_like(ids, lf.shape[-1])).min(-1).values + id_offset
    u = (m + 0.0).view(torch.int32).long() & 0xFFFFFFFF  # + 0.0: -0.0 keys like +0.0 (ties, lowest id)
    neg = (u & 0x80000000) != 0
    ordv = torch.where(neg, (~u) & 0xFFFFFFFF, u | 0x80000000)
    hi = (ordv ^ 0x80000000) - ((ordv ^ 0x80000000) >= 0x80000000).long() * (1 << 32)  # as signed 32-bit
    return (hi << 32) | (0xFFFFFFFF - first)


def unpack_argmax(packed: torch.Tensor) -> torch.Tensor:
    if packed.is_cuda:
        return ops().unpack_argmax(packed)
    return (0xFFFFFFFF - (packed & 0xFFFFFFFF)).int()


# --------------------------------------------------------------------------
# DeltaNet / GQA decode
# --------------------------------------------------------------------------
def deltanet_decode(qkv, z, a, b, conv_ring, state, positions, conv_w, A_log, dt_bias, norm_w,
                    k_heads: int, eps: float = 1e-6) -> torch.Tensor:
    """One fused gated-DeltaNet decode step; updates ``conv_ring`` and ``state``
    in place and returns the RMSNormGated output ``[B, VH*128]``."""
    if qkv.is_cuda:
        return ops().deltanet_decode(qkv, z, a, b, conv_ring, state, positions, conv_w, A_log, dt_bias, norm_w,
                                     k_heads, eps)
    VH = state.shape[1]
    return ref.deltanet_decode(qkv, a, b, z, conv_ring, state, positions, conv_w, A_log, dt_bias, norm_w,
                               k_heads, state.shape[2], state.shape[3], eps)[:, : VH * state.shape[3]]


def deltanet_verify(qkv, z, a, b, stash_qkv, stash_ab, vstep, conv_ring, state, positions, pending, conv_w, A_log,
                    dt_bias, norm_w, k_heads: int, n_tok: int, eps: float = 1e-6) -> torch.Tensor:
    """Speculative verify of ``n_tok`` tokens per sequence with deferred commit
    (rows ``[B*n_tok, *]``): the stashed tokens the last step accepted
    (``pending``) are committed to the state first; the new tokens only produce
    outputs and are stashed for the next commit."""
    if qkv.is_cuda:
        return ops().deltanet_verify(qkv, z, a, b, stash_qkv, stash_ab, vstep, conv_ring, state, positions, pending,
                                     conv_w, A_log, dt_bias, norm_w, k_heads, n_tok, eps)
    return ref.deltanet_verify(qkv, z, a, b, stash_qkv, stash_ab, vstep, conv_ring, state, positions, pending, conv_w,
                               A_log, dt_bias, norm_w, k_heads, n_tok, eps)


def gqa_decode(qg, k_new, v_new, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, positions,
               eps: float = 1e-6, splits: int = 0, n_tok: int = 1) -> torch.Tensor:
    """Fused gated GQA decode step (appends K/V at ``positions``); ``n_tok``
    query rows per cache sequence for speculative verification."""
    if qg.is_cuda:
        return ops().gqa_decode(qg, k_new, v_new, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, positions,
                                eps, splits, n_tok)
    return ref.gqa_decode(qg, k_new, v_new, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, positions, eps, n_tok)


# --------------------------------------------------------------------------
# prefill
# --------------------------------------------------------------------------
def _host_start(start_pos) -> int:
    return int(start_pos.reshape(-1)[0].item()) if torch.is_tensor(start_pos) else int(start_pos)


def deltanet_prefill(qkv, z, a, b, conv_ring, state, start_pos, valid_len, conv_w, A_log, dt_bias, norm_w,
                     k_heads: int, eps: float = 1e-6, chunk: int = 64) -> torch.Tensor:
    """Gated-DeltaNet over a prompt chunk ``qkv [B,S,C]`` (conv ring + recurrent
    state carried in and out).  ``start_pos``: host int, or an int32 device
    tensor (element 0) read by the kernels at run time.  Returns ``[B, S, VH*128]``."""
    if qkv.is_cuda:
        return _prefill_cuda().deltanet_prefill(qkv, z, a, b, conv_ring, state, start_pos, valid_len, conv_w, A_log,
                                                dt_bias, norm_w, k_heads, eps)
    return ref.deltanet_prefill(qkv, a, b, z, conv_ring, state, _host_start(start_pos), valid_len, conv_w, A_log,
                                dt_bias, norm_w, k_heads, state.shape[2], state.shape[3], eps, chunk)


def gqa_prefill(qg, k, v, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, start_pos,
                eps: float = 1e-6) -> torch.Tensor:
    """Gated GQA over a prompt chunk: q/k norm + RoPE at ``start_pos``, K/V
    written to cache rows ``[start, start+S)``, causal attention over the used
    prefix, sigmoid gate.  ``qg [B,S,QH,2D]``, ``k/v [B,S,KVH,D]`` -> ``[B,S,QH*D]``."""
    if qg.is_cuda:
        return _prefill_cuda().gqa_prefill(qg, k, v, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, start_pos, eps)
    B, S, QH, D2 = qg.shape
    D = D2 // 2
    start_pos = _host_start(start_pos)
    q, gate = qg.float().split(D, dim=-1)
    c = cos[start_pos:start_pos + S][None, :, None]
    s = sin[start_pos:start_pos + S][None, :, None]
    q = ref.apply_partial_rope(ref.rms_norm(q, q_norm_w, eps), c, s)
    kk = ref.apply_partial_rope(ref.rms_norm(k.float(), k_norm_w, eps), c, s)
    k_cache[:, :, start_pos:start_pos + S] = kk.transpose(1, 2).to(k_cache.dtype)
    v_cache[:, :, start_pos:start_pos + S] = v.transpose(1, 2).to(v_cache.dtype)
    o = ref.attention_prefill(q.transpose(1, 2), k_cache, v_cache, start_pos)  # [B, QH, S, D]
    o = o.transpose(1, 2) * torch.sigmoid(gate)
    return o.reshape(B, S, QH * D).to(qg.dtype)


def _prefill_cuda():
    from . import prefill_cuda
    return prefill_cuda


# --------------------------------------------------------------------------
# MoE
# --------------------------------------------------------------------------
def moe_topk_softmax(logits: torch.Tensor, k: int, renorm: bool = True):
    """softmax -> top-k -> (renormalise); returns ``(w [T,k] fp32, ids [T,k] int32)``."""
    if logits.is_cuda:
        return ops().moe_topk(logits.float().contiguous(), k, renorm, None, 0, 1.0)
    return ref.moe_route_softmax(logits, k, renorm)


def moe_topk_deepseek(logits: torch.Tensor, bias, k: int, score_func: str = "sqrtsoftplus",
                      route_scale: float = 1.5):
    if logits.is_cuda:
        mode = 1 if score_func == "sqrtsoftplus" else 2
        b = bias.float().contiguous() if bias is not None else None
        return ops().moe_topk(logits.float().contiguous(), k, True, b, mode, route_scale)
    return ref.moe_route_deepseek(logits, bias, k, score_func, route_scale)


def moe_experts(x, w, ids, gate_up_il, down, expert_offset: int = 0, shared=None, swiglu_limit: float = 0.0):
    """This rank's routed-expert partial (plus, when ``shared=(y, gate_logit)``
    is given, ``sigmoid(gate_logit) * y``).  The experts are bf16 tensors or
    :class:`~bwn.io.fp8.FP8Experts` (fp8 grouped GEMM on the GPU)."""
    if hasattr(gate_up_il, "scales16"):
        if x.is_cuda:
            sy, sg = (shared if shared is not None else (None, None))
            return ops().moe_experts_w8(x, w.float().contiguous(), ids.int().contiguous(), gate_up_il.w8,
                                        gate_up_il.scales16, down.w8, down.scales16, expert_offset, sy,
                                        sg.float().reshape(-1).contiguous() if sg is not None else None,
                                        swiglu_limit)
        # the GPU kernel rounds each dequantized weight to bf16
        gate_up_il = gate_up_il.dequant().to(torch.bfloat16).to(x.dtype)
        down = down.dequant().to(torch.bfloat16).to(x.dtype)
    if x.is_cuda:
        sy, sg = (shared if shared is not None else (None, None))
        return ops().moe_experts(x, w.float().contiguous(), ids.int().contiguous(), gate_up_il, down, expert_offset,
                                 sy, sg.float().reshape(-1).contiguous() if sg is not None else None, swiglu_limit)
    E, n2, H = gate_up_il.shape
    xg = gate_up_il.reshape(E, n2 // 32, 2, 16, H)
    gu = torch.cat([xg[:, :, 0].reshape(E, n2 // 2, H), xg[:, :, 1].reshape(E, n2 // 2, H)], dim=1)
    out = ref.moe_experts(x, w, ids, gu, down, expert_offset, swiglu_limit)
    if shared is not None:
        sy, sg = shared
        out = out + torch.sigmoid(sg.float().reshape(-1, 1)) * sy.float()
    return out.to(x.dtype)


# --------------------------------------------------------------------------
# DeepSeek V4: hyper-connections, single-KV-head attention
# --------------------------------------------------------------------------
_hc_fn_cache: dict = {}


def _hc_fn_bf16(fn: torch.Tensor) -> torch.Tensor:
    key = (fn.data_ptr(), fn._version, tuple(fn.shape))
    w = _hc_fn_cache.get(key)
    if w is None:
        rows = (fn.shape[0] + 7) // 8 * 8
        w = torch.zeros(rows, fn.shape[1], dtype=torch.bfloat16, device=fn.device)
        w[:fn.shape[0]] = fn
        if len(_hc_fn_cache) > 256:
            _hc_fn_cache.clear()
        _hc_fn_cache[key] = w
    return w


def hc_pre(x, fn, scale, base, iters: int = 20, eps: float = 1e-6, norm_eps: float = 1e-6):
    """Hyper-Connection pre-mix of ``x [T, hc, dim]``.  With ``fn [(2+hc)*hc, hc*dim]``
    returns ``(y [T,dim], post [T,hc], comb [T,hc,hc])``; with ``fn [hc, hc*dim]``
    (the head) returns ``(y, None, None)``."""
    if x.is_cuda:
        x = x.contiguous()
        T, hc, dim = x.shape
        mix = None
        from ..utils import env
        if env.get("BWN_HC_GEMM") and (hc * dim) % 64 == 0:
            # every token's mix GEMV as one tensor-core GEMM (split over K at decode
            # sizes) against a bf16 copy of fn (rows padded to 8), read by the kernel
            mix = linear_f32(x.view(T, hc * dim), _hc_fn_bf16(fn))
        y, post, comb = ops().hc_pre(x, fn.float().contiguous(), scale.float().contiguous(),
                                     base.float().contiguous(), iters, eps, norm_eps, mix)
        return (y, None, None) if fn.shape[0] == x.shape[1] else (y, post, comb)
    return ref.hc_pre(x, fn, scale, base, iters, eps, norm_eps)


def hc_post(x, resid, post, comb):
    if x.is_cuda:
        return ops().hc_post(x.contiguous(), resid.contiguous(), post.contiguous(), comb.contiguous())
    return ref.hc_post(x, resid, post, comb)


def mqa_attn(q, kv, visible, q_per_seq: int, scale: float, splits: int = 0):
    """Attention of ``q [rows, H, D]`` over one shared K/V head per sequence
    ``kv [B, T, D]``; row ``r`` (sequence ``r // q_per_seq``) sees keys
    ``[0, visible[r])``."""
    if q.is_cuda:
        return ops().mqa_attn(q.contiguous(), kv, visible.int().contiguous(), q_per_seq, scale, splits)
    return ref.mqa_attn(q, kv, visible, q_per_seq, scale)


def rope_half(x, cos, sin, B: int, S: int, H: int, to_heads: bool, sign: float = 1.0, scale: float = 1.0):
    """Rotate-half RoPE (ESM-2) fused with ``scale`` and the layout change:
    ``to_heads``: ``x [B*S, H*D] -> [B, H, S, D]``; otherwise ``x [B, H, S, D] ->
    [B*S, H*D]``.  ``sign=-1`` rotates by the negative angle (the backward).
    ``cos``/``sin``: ``[>= S, D/2]`` fp32 tables."""
    if x.is_cuda:
        return ops().rope_half(x.contiguous(), cos, sin, B, S, H, to_heads, sign, scale)
    D = x.numel() // (B * S * H)
    xs = x.reshape(B, S, H, D) if to_heads else x.reshape(B, H, S, D).transpose(1, 2)
    x1, x2 = xs.float().split(D // 2, dim=-1)
    c = cos[:S][None, :, None]
    s = sin[:S][None, :, None] * sign
    y = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1) * scale
    y = y.to(x.dtype)
    return y.transpose(1, 2).contiguous() if to_heads else y.reshape(B * S, H * D)


def rope_interleaved_(x, cos, sin, pos):
    """In place: interleaved-pair RoPE on the trailing ``2*cos.shape[1]`` dims of
    ``x [rows, H, D]`` at ``pos [rows]``."""
    if x.is_cuda:
        ops().rope_interleaved_(x, cos, sin, pos.int().contiguous())
        return x
    c = cos[pos.long()][:, None]
    s = sin[pos.long()][:, None]
    x.copy_(ref.apply_interleaved_rope(x, c, s))
    return x
