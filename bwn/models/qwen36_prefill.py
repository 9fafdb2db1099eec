"""Prompt processing for :class:`~bwn.models.qwen36.Qwen36Model`.

One chunk of ``S`` tokens per sequence at a shared start position (the
reference's bucketed chunked prefill, ``static_decode_35b.py:2497-2678``,
``_deltanet_prefill`` ``:2137-2258``, ``_gqa_prefill_chunk`` ``:2316-2449``):

* all projections run on the flattened ``[B*S, H]`` token matrix (tcgen05 GEMMs
  in the normal orientation, 128x256 tiles);
* DeltaNet: causal conv with the ring as history, then the chunked gated delta
  rule carrying the recurrent state in and out (pad rows get ``g = beta = 0``);
* GQA: q/k norm + partial RoPE at the runtime offset, K/V written into the
  cache, prefix-aware causal attention over ``[0, start+S)``, sigmoid gate.
"""
from __future__ import annotations

import torch

from .. import ops as O


def _trace_layer(model, mode: int, start: int, i: int, kind: str, x: torch.Tensor, state: torch.Tensor) -> None:
    """Per-layer numeric trace of a prefill chunk (``BWN_PREFILL_TRACE``; the
    reference's PREFILL_TRACE_LAYER / _FINITE, ``static_decode_35b.py:2457-2470``):
    finiteness and max-abs of the residual stream and of the layer's carried
    state, printed on rank 0; mode 2 also raises at the first non-finite layer."""
    def stat(t):
        f = t.float()
        fin = torch.isfinite(f)
        return bool(fin.all()), float(f[fin].abs().max()) if bool(fin.any()) else float("nan")
    (xf, xm), (sf, sm) = stat(x), stat(state)
    if model.rank == 0:
        print(f"[prefill-trace] start={start} layer={i} type={kind} residual finite={xf} max={xm:.4e} "
              f"state finite={sf} max={sm:.4e}", flush=True)
    if mode >= 2 and not (xf and sf):
        raise FloatingPointError(f"prefill: non-finite values after layer {i} ({kind}) at start={start}")


def prefill_hidden(model, tokens: torch.Tensor, st, valid_len, chunk: int = 64, feat_layers=(), feats_out=None,
                   all_rows: bool = False) -> torch.Tensor:
    """Returns the final-normed hidden of each sequence's last valid row ``[B, H]``
    (every row ``[B*S, H]`` with ``all_rows``); the residual stream after each of
    ``feat_layers`` is appended to ``feats_out`` (``[B*S, H]``, for EAGLE3)."""
    cfg, d = model.cfg, model.d
    B, S = tokens.shape
    dev = tokens.device
    # the chunk's shared start is the largest row position (rows whose prompt
    # ended in an earlier chunk sit behind it and have no valid rows here); it
    # stays on the device and the kernels read it at run time, so a chunk needs
    # no host sync and one captured graph serves every offset
    start = st.positions.amax().reshape(1) if dev.type == "cuda" else int(st.positions.max())
    model.ensure_rope(st.k_cache.shape[3] if dev.type == "cuda" else start + S)
    if valid_len is None:
        valid_len = torch.full((B,), S, dtype=torch.int32, device=dev)
    valid_len = valid_len.to(dev).int()
    T = B * S
    x = model.embed(tokens.reshape(T))  # [T, H]
    h = O.rms_norm(x, model.layers[0]["in_norm"], cfg.rms_eps)
    captured = {}
    from ..utils import env
    trace = env.get("BWN_PREFILL_TRACE")
    di = gi = 0
    for i in range(cfg.num_layers):
        L = model.layers[i]
        if cfg.layer_type(i) == "deltanet":
            C, Z, VH = d.dn_qkv_dim, d.dn_value_dim, d.dn_v_heads
            proj = O.linear(h, L["in_proj"]).view(B, S, -1)
            o = O.deltanet_prefill(proj[..., :C], proj[..., C:C + Z], proj[..., C + Z + VH:],
                                   proj[..., C + Z:C + Z + VH], st.conv[di], st.ssm[di], start, valid_len,
                                   L["conv_w"], L["A_log"], L["dt_bias"], L["norm_w"], d.dn_k_heads, cfg.rms_eps,
                                   chunk)
            h = model._row_parallel(o.reshape(T, -1), L["out_proj"], x, L["post_norm"])
            di += 1
        else:
            D, QH, KVH = cfg.head_dim, d.q_heads, d.kv_heads
            proj = O.linear(h, L["qkv_proj"]).view(B, S, -1)
            qg = proj[..., :QH * 2 * D].reshape(B, S, QH, 2 * D)
            k = proj[..., QH * 2 * D:QH * 2 * D + KVH * D].reshape(B, S, KVH, D)
            v = proj[..., QH * 2 * D + KVH * D:].reshape(B, S, KVH, D)
            o = O.gqa_prefill(qg, k, v, L["q_norm"], L["k_norm"], model.rope_cos, model.rope_sin,
                              st.k_cache[gi], st.v_cache[gi], start, cfg.rms_eps)
            h = model._row_parallel(o.reshape(T, -1), L["o_proj"], x, L["post_norm"])
            gi += 1
        nxt = model.layers[i + 1]["in_norm"] if i + 1 < cfg.num_layers else model.g["final_norm"]
        if cfg.is_moe:
            h = model.moe_residual(i, h, x, nxt)
        else:
            act = model._mlp(i, h)
            h = model._row_parallel(act, L["down"], x, nxt)
        if feats_out is not None and i in feat_layers:
            captured[i] = x.clone()
        if trace:
            dn = cfg.layer_type(i) == "deltanet"
            _trace_layer(model, trace, int(st.positions.max()), i, cfg.layer_type(i), x,
                         st.ssm[di - 1] if dn else st.k_cache[gi - 1])
    if feats_out is not None:
        feats_out.extend(captured[i] for i in feat_layers)
    st.positions.add_(valid_len)
    if all_rows:
        return h
    last = (valid_len.long() - 1).clamp(min=0) + torch.arange(B, device=dev) * S
    return h[last]


def prefill_hidden_sp(model, tokens: torch.Tensor, st, sp, chunk: int = 64) -> torch.Tensor:
    """Sequence-parallel prefill of full-length rows (``tokens [B, S]``, no
    padding, ``B*S`` a multiple of ``128 * world``) through :class:`bwn.parallel.sp.SeqParallel`:
    the residual stream is sharded by rows, every row-parallel output is
    reduce-scattered + normed + all-gathered in one kernel, and each
    column-parallel GEMM reads the gathered rows as they arrive.  MoE layers use
    the expert-parallel all-to-all on the row shard.  Returns the final-normed
    hidden of each sequence's last token ``[B, H]``."""
    cfg, d = model.cfg, model.d
    B, S = tokens.shape
    T = B * S
    W, r = model.tp, model.rank
    if T % (128 * W) or T > sp.T_max:
        raise ValueError(f"sequence-parallel prefill needs B*S a multiple of {128 * W} and <= {sp.T_max}")
    Ts = T // W
    dev = tokens.device
    start = st.positions.amax().reshape(1)  # read by the kernels at run time
    model.ensure_rope(st.k_cache.shape[3])
    valid_len = torch.full((B,), S, dtype=torch.int32, device=dev)
    x_full = model.embed(tokens.reshape(T))
    x = x_full[r * Ts:(r + 1) * Ts].contiguous()  # residual shard
    h = O.rms_norm(x_full, model.layers[0]["in_norm"], cfg.rms_eps)
    del x_full
    eps = cfg.rms_eps
    di = gi = 0

    def col(w, first, swiglu=False):
        if first:
            return O.linear_swiglu(h, w) if swiglu else O.linear(h, w)
        return sp.column(w, T, swiglu)

    for i in range(cfg.num_layers):
        L = model.layers[i]
        first = i == 0
        if cfg.layer_type(i) == "deltanet":
            C, Z, VH = d.dn_qkv_dim, d.dn_value_dim, d.dn_v_heads
            proj = col(L["in_proj"], first).view(B, S, -1)
            o = O.deltanet_prefill(proj[..., :C], proj[..., C:C + Z], proj[..., C + Z + VH:],
                                   proj[..., C + Z:C + Z + VH], st.conv[di], st.ssm[di], start, valid_len,
                                   L["conv_w"], L["A_log"], L["dt_bias"], L["norm_w"], d.dn_k_heads, eps, chunk)
            sp.row_parallel(o.reshape(T, -1), L["out_proj"])
            di += 1
        else:
            D, QH, KVH = cfg.head_dim, d.q_heads, d.kv_heads
            proj = col(L["qkv_proj"], first).view(B, S, -1)
            qg = proj[..., :QH * 2 * D].reshape(B, S, QH, 2 * D)
            k = proj[..., QH * 2 * D:QH * 2 * D + KVH * D].reshape(B, S, KVH, D)
            v = proj[..., QH * 2 * D + KVH * D:].reshape(B, S, KVH, D)
            o = O.gqa_prefill(qg, k, v, L["q_norm"], L["k_norm"], model.rope_cos, model.rope_sin,
                              st.k_cache[gi], st.v_cache[gi], start, eps)
            sp.row_parallel(o.reshape(T, -1), L["o_proj"])
            gi += 1
        sp.norm_gather(x, L["post_norm"], eps)
        nxt = model.layers[i + 1]["in_norm"] if i + 1 < cfg.num_layers else model.g["final_norm"]
        if cfg.is_moe:
            ep = getattr(model, "ep_a2a", None)
            if ep is None or Ts > ep.T_max:
                raise RuntimeError("sequence-parallel MoE layers need the expert-parallel all-to-all sized for the shard")
            from .moe import route
            hs = sp.gathered(T)[r * Ts:(r + 1) * Ts]
            w, ids = route(model, L, hs)
            sy = O.linear(O.linear_swiglu(hs, L["shared_gate_up_full"]), L["shared_down_full"])
            sg = O.linear_f32(hs, L["shared_gate"])
            ys = ep.moe(hs, w, ids, L["experts_gate_up"], L["experts_down"], shared=(sy, sg))
            sp.norm_gather(x, nxt, eps, addend=ys)
        else:
            act = sp.column(L["gate_up"], T, swiglu=True)
            sp.row_parallel(act, L["down"])
            sp.norm_gather(x, nxt, eps)
        h = None
    st.positions.add_(valid_len)
    hf = sp.gathered(T)
    last = torch.arange(B, device=dev) * S + (S - 1)
    return hf[last].clone()
