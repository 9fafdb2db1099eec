"""Plain-PyTorch fp32 reference implementations of every bwn op.

These are the numerics oracles the CUDA kernels are tested against, and the
code path used when tensors live on the CPU (the CPU test tier).  Each function
states the reference behaviour it reproduces.

Conventions shared with the CUDA kernels:

* DeltaNet conv history is an R-slot ring ``conv_ring[B, R, C]`` (R = 4, or 8
  when multi-token verify is used): the qkv row of token position ``t`` lives in
  slot ``t % R``.  A decode step at position ``p`` reads slots
  ``(p-3..p-1) % R`` and writes slot ``p % R``; no reader ever needs
  the slot being written, so one launch may update the ring in place while other
  CTAs still read it.  (The reference keeps a shifted ``[QKV, 3]`` window,
  ``contrib/qwen3.6-27b/kernels/deltanet_full.py:82-134``.)
* DeltaNet recurrent state is ``[B, VH, Dk, Dv]`` fp32 (HF layout).
* KV cache is ``[B, KVH, S_max, D]`` bf16; the row for position ``p`` is written
  by the decode kernel itself (append-after-attention with the current row
  included in the softmax, ``qwen3.6-35b-a3b/BENCHMARK.md:600-606``).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


# --------------------------------------------------------------------------
# norms / activations
# --------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, one_plus: bool = True) -> torch.Tensor:
    """``x * rsqrt(mean(x^2)+eps) * (1+w)`` (``qwen3.6-27b/static_decode.py:322-335``)."""
    xf = x.float()
    n = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    wf = w.float()
    return (n * ((1.0 + wf) if one_plus else wf)).to(x.dtype)


def add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float = 1e-6):
    """``residual += x`` then RMSNorm(1+w) of the new residual; returns (residual, normed)."""
    r = (residual.float() + x.float()).to(residual.dtype)
    return r, rms_norm(r, w, eps)


def rms_norm_gated(o: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``w * rmsnorm(o) * silu(z)`` per head (``qwen3.6-27b/static_decode.py:338-342``)."""
    of = o.float()
    n = of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + eps)
    return (w.float() * n * F.silu(z.float())).to(z.dtype)


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``x / max(||x||, eps)`` -- the reference's ``F.normalize`` semantics."""
    return F.normalize(x.float(), p=2, dim=-1, eps=eps)


def swiglu(gate_up: torch.Tensor, limit: float = 0.0) -> torch.Tensor:
    """``silu(g) * u`` over a packed ``[..., 2I]`` (gate || up) row.

    With ``limit > 0`` both halves are clamped first (DeepSeek ``swiglu_limit``,
    ``run_deepseek_v4_tp.py:380-394``): ``g <= limit``, ``|u| <= limit``.
    """
    g, u = gate_up.float().chunk(2, dim=-1)
    if limit > 0:
        g = g.clamp(max=limit)
        u = u.clamp(-limit, limit)
    return (F.silu(g) * u).to(gate_up.dtype)


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ w.T`` with fp32 accumulation, output in x's dtype."""
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    return y.to(x.dtype)


# --------------------------------------------------------------------------
# RoPE
# --------------------------------------------------------------------------
def rope_table(max_pos: int, rot_dim: int, theta: float, device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 ``cos, sin`` of shape ``[max_pos, rot_dim]`` (half-split, HF layout)."""
    inv = 1.0 / (theta ** (torch.arange(0, rot_dim, 2, dtype=torch.float64) / rot_dim))
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().float().to(device), emb.sin().float().to(device)


def apply_partial_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate the first ``cos.shape[-1]`` dims (rotate-half pairing), pass the rest
    (``qwen3.6-27b/static_decode.py:356-369``).  ``cos``/``sin`` broadcast over x."""
    r = cos.shape[-1]
    xf = x.float()
    xr, xp = xf[..., :r], xf[..., r:]
    x1, x2 = xr[..., : r // 2], xr[..., r // 2:]
    rot = torch.cat([-x2, x1], dim=-1)
    return torch.cat([xr * cos + rot * sin, xp], dim=-1).to(x.dtype)


def apply_interleaved_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """RoPE on the trailing ``2*cos.shape[-1]`` dims with interleaved (even, odd)
    pairs (DeepSeek, ``run_deepseek_v4_tp.py:147-160``).  ``cos``/``sin`` have
    ``rope_dim/2`` entries."""
    r = 2 * cos.shape[-1]
    xf = x.float()
    xp, xr = xf[..., :-r], xf[..., -r:]
    a, b = xr[..., 0::2], xr[..., 1::2]
    ra = a * cos - b * sin
    rb = a * sin + b * cos
    out = torch.stack([ra, rb], dim=-1).flatten(-2)
    return torch.cat([xp, out], dim=-1).to(x.dtype)


# --------------------------------------------------------------------------
# gated DeltaNet
# --------------------------------------------------------------------------
def deltanet_gates(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor):
    """``g = -exp(A_log) * softplus(a + dt_bias)``, ``beta = sigmoid(b)``."""
    g = -A_log.float().exp() * F.softplus(a.float() + dt_bias.float())
    return g, b.float().sigmoid()


def deltanet_decode(
    qkv: torch.Tensor,        # [B, C] bf16, C = 2*KH*Dk + VH*Dv (pre-conv)
    a: torch.Tensor,          # [B, VH]
    b: torch.Tensor,          # [B, VH]
    z: torch.Tensor,          # [B, VH*Dv]
    conv_ring: torch.Tensor,  # [B, 4, C]   (updated in place)
    state: torch.Tensor,      # [B, VH, Dk, Dv] fp32/bf16 (updated in place)
    positions: torch.Tensor,  # [B] int
    conv_w: torch.Tensor,     # [C, 4]
    A_log: torch.Tensor,      # [VH]
    dt_bias: torch.Tensor,    # [VH]
    norm_w: torch.Tensor,     # [Dv]
    k_heads: int,
    k_dim: int,
    v_dim: int,
    eps: float = 1e-6,
) -> torch.Tensor:
    """One recurrent gated-delta-rule decode step, fused like the reference's
    ``nki_deltanet_full(_batched)`` (``qwen3.6-27b/kernels/deltanet_full.py:54-427``):
    conv4 + SiLU, L2 norm + 1/sqrt(Dk) q scale, gates, ``S*=exp(g); kv=S^T k;
    d=beta(v-kv); S+=k d^T; o=S^T q``, then RMSNormGated.  Returns ``[B, VH*Dv]``."""
    B, C = qkv.shape
    VH = a.shape[1]
    KD = k_heads * k_dim
    pos = positions.long()
    ks = conv_w.shape[1]
    rows = torch.arange(B, device=qkv.device)
    R = conv_ring.shape[1]  # ring slots (4, or 8 for multi-token verify)
    hist = [conv_ring[rows, (pos - (ks - 1) + j) % R].float() for j in range(ks - 1)]
    xs = torch.stack(hist + [qkv.float()], dim=-1)  # [B, C, ks]
    y = F.silu((xs * conv_w.float().unsqueeze(0)).sum(-1))
    conv_ring[rows, pos % R] = qkv.to(conv_ring.dtype)
    q = y[:, :KD].reshape(B, k_heads, k_dim)
    k = y[:, KD:2 * KD].reshape(B, k_heads, k_dim)
    v = y[:, 2 * KD:].reshape(B, VH, v_dim)
    q = l2norm(q) * (1.0 / math.sqrt(k_dim))
    k = l2norm(k)
    rep = VH // k_heads
    q = q.repeat_interleave(rep, dim=1)
    k = k.repeat_interleave(rep, dim=1)
    g, beta = deltanet_gates(a, b, A_log, dt_bias)
    S = state.float() * g.exp()[..., None, None]
    kv = torch.einsum("bhkv,bhk->bhv", S, k)
    delta = beta[..., None] * (v - kv)
    S = S + k[..., :, None] * delta[..., None, :]
    o = torch.einsum("bhkv,bhk->bhv", S, q)
    state.copy_(S.to(state.dtype))
    out = rms_norm_gated(o, z.reshape(B, VH, v_dim), norm_w, eps)
    return out.reshape(B, VH * v_dim)


def causal_conv1d_prefill(x: torch.Tensor, conv_w: torch.Tensor, init_ring: torch.Tensor | None,
                          start_pos: int = 0):
    """Depthwise causal conv (kernel ks) + SiLU over a sequence ``x [B, S, C]``.

    History before ``start_pos`` comes from ``init_ring [B, ks, C]`` (ring slots);
    zeros when absent.  Returns ``(y [B,S,C] fp32, history [B, ks-1, C])`` where
    history holds the rows of positions ``start_pos+S-(ks-1) .. start_pos+S-1``.
    """
    B, S, C = x.shape
    ks = conv_w.shape[1]
    if init_ring is not None:
        hist = torch.stack(
            [init_ring[:, (start_pos - (ks - 1) + j) % init_ring.shape[1]] for j in range(ks - 1)], dim=1
        ).float()
        if start_pos < ks - 1:
            hist[:, : (ks - 1) - start_pos] = 0
    else:
        hist = x.new_zeros(B, ks - 1, C, dtype=torch.float32)
    xx = torch.cat([hist, x.float()], dim=1)  # [B, S+ks-1, C]
    y = torch.zeros(B, S, C, dtype=torch.float32, device=x.device)
    for j in range(ks):
        y = y + xx[:, j:j + S] * conv_w[:, j].float()
    return F.silu(y), xx[:, S:]


def chunk_gated_delta_rule(q, k, v, g, beta, state=None, chunk: int = 64):
    """Chunked gated delta rule, fp32 (the reference's torch fallback
    ``neuron_chunk_gated_delta_rule``, ``qwen3.6-27b/chunked_prefill.py:16-172``).

    ``q,k [B,H,S,Dk]`` (already L2-normed; q already scaled), ``v [B,H,S,Dv]``,
    ``g, beta [B,H,S]``.  Per chunk of C tokens with in-chunk cumulative decay
    ``G``: ``A = -tril(diag(beta) K K^T * exp(G_i - G_j), -1)``; ``T = (I - A)^-1``
    applied to ``beta V`` and ``beta K exp(G)``; intra-chunk output plus the
    inter-chunk contribution of the carried state, then the state update.
    Returns ``(o [B,H,S,Dv] fp32, final_state [B,H,Dk,Dv] fp32)``.
    """
    B, H, S, Dk = k.shape
    Dv = v.shape[-1]
    pad = (chunk - S % chunk) % chunk
    q, k, v = [F.pad(t.float(), (0, 0, 0, pad)) for t in (q, k, v)]
    g = F.pad(g.float(), (0, pad))
    beta = F.pad(beta.float(), (0, pad))
    n = (S + pad) // chunk
    q, k, v = [t.reshape(B, H, n, chunk, -1) for t in (q, k, v)]
    g = g.reshape(B, H, n, chunk).cumsum(-1)
    beta = beta.reshape(B, H, n, chunk)
    st = torch.zeros(B, H, Dk, Dv, dtype=torch.float32, device=q.device) if state is None else state.float().clone()
    out = torch.empty(B, H, n, chunk, Dv, dtype=torch.float32, device=q.device)
    lower = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool, device=q.device), -1)
    incl = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool, device=q.device), 0)
    eye = torch.eye(chunk, device=q.device)
    for c in range(n):
        qc, kc, vc, gc, bc = q[:, :, c], k[:, :, c], v[:, :, c], g[:, :, c], beta[:, :, c]
        diff = gc[..., :, None] - gc[..., None, :]
        # mask before exp: masked entries may overflow
        dec = torch.where(incl, diff, torch.full_like(diff, -float("inf"))).exp()
        A = -(bc[..., :, None] * (kc @ kc.transpose(-1, -2)) * dec).masked_fill(~lower, 0)
        T = torch.linalg.solve_triangular(eye - A, eye.expand_as(A).contiguous(), upper=False)
        u = T @ (bc[..., None] * vc)
        w = T @ (bc[..., None] * kc * gc.exp()[..., None])
        vn = u - w @ st
        att = (qc @ kc.transpose(-1, -2)) * dec
        out[:, :, c] = (qc * gc.exp()[..., None]) @ st + att @ vn
        gl = gc[..., -1:]
        st = st * gl[..., None].exp() + (kc * (gl - gc).exp()[..., None]).transpose(-1, -2) @ vn
    return out.reshape(B, H, n * chunk, Dv)[:, :, :S], st


def recurrent_gated_delta_rule(q, k, v, g, beta, state=None):
    """Token-by-token oracle of :func:`chunk_gated_delta_rule` (same layouts)."""
    B, H, S, Dk = k.shape
    Dv = v.shape[-1]
    st = torch.zeros(B, H, Dk, Dv, dtype=torch.float32, device=q.device) if state is None else state.float().clone()
    out = torch.empty(B, H, S, Dv, dtype=torch.float32, device=q.device)
    for t in range(S):
        st = st * g[:, :, t].float().exp()[..., None, None]
        kv = torch.einsum("bhkv,bhk->bhv", st, k[:, :, t].float())
        d = beta[:, :, t].float()[..., None] * (v[:, :, t].float() - kv)
        st = st + k[:, :, t].float()[..., :, None] * d[..., None, :]
        out[:, :, t] = torch.einsum("bhkv,bhk->bhv", st, q[:, :, t].float())
    return out, st


def deltanet_prefill(
    qkv: torch.Tensor,        # [B, S, C]
    a: torch.Tensor,          # [B, S, VH]
    b: torch.Tensor,          # [B, S, VH]
    z: torch.Tensor,          # [B, S, VH*Dv]
    conv_ring: torch.Tensor,  # [B, 4, C]   (updated: last 3 rows written to their slots)
    state: torch.Tensor,      # [B, VH, Dk, Dv] (updated)
    start_pos: int,
    valid_len: torch.Tensor | None,  # [B] number of real rows in this chunk (pad rows get g=beta=0)
    conv_w, A_log, dt_bias, norm_w,
    k_heads: int, k_dim: int, v_dim: int, eps: float = 1e-6, chunk: int = 64,
) -> torch.Tensor:
    """DeltaNet layer core over a prompt chunk (``_deltanet_prefill``,
    ``qwen3.6-35b-a3b/static_decode_35b.py:2137-2258``).  Pad rows (beyond
    ``valid_len``) get ``beta = g = 0`` so they leave the state untouched
    (``static_decode_35b.py:2172-2192``)."""
    B, S, C = qkv.shape
    VH = a.shape[-1]
    KD = k_heads * k_dim
    y, _ = causal_conv1d_prefill(qkv, conv_w, conv_ring, start_pos)
    q = y[..., :KD].reshape(B, S, k_heads, k_dim)
    k = y[..., KD:2 * KD].reshape(B, S, k_heads, k_dim)
    v = y[..., 2 * KD:].reshape(B, S, VH, v_dim)
    q = l2norm(q) * (1.0 / math.sqrt(k_dim))
    k = l2norm(k)
    rep = VH // k_heads
    q = q.repeat_interleave(rep, 2).transpose(1, 2)
    k = k.repeat_interleave(rep, 2).transpose(1, 2)
    v = v.transpose(1, 2)
    g, beta = deltanet_gates(a, b, A_log, dt_bias)
    g, beta = g.transpose(1, 2), beta.transpose(1, 2)  # [B, VH, S]
    if valid_len is not None:
        live = torch.arange(S, device=qkv.device)[None, :] < valid_len.to(qkv.device)[:, None]
        g = g * live[:, None]
        beta = beta * live[:, None]
    o, st = chunk_gated_delta_rule(q, k, v, g, beta, state, chunk)
    state.copy_(st.to(state.dtype))
    # conv ring: store the last (ks-1) valid rows of each sequence (the only
    # history the next decode step reads)
    ks = conv_w.shape[1]
    for bi in range(B):
        n = S if valid_len is None else int(valid_len[bi])
        for t in range(max(0, n - (ks - 1)), n):
            conv_ring[bi, (start_pos + t) % conv_ring.shape[1]] = qkv[bi, t].to(conv_ring.dtype)
    o = o.transpose(1, 2)  # [B, S, VH, Dv]
    out = rms_norm_gated(o, z.reshape(B, S, VH, v_dim), norm_w, eps)
    return out.reshape(B, S, VH * v_dim)


# --------------------------------------------------------------------------
# gated GQA attention
# --------------------------------------------------------------------------
def gqa_decode(
    qg: torch.Tensor,        # [B, QH, 2*D]  (query || gate per head, pre-norm)
    k_new: torch.Tensor,     # [B, KVH, D]   pre-norm
    v_new: torch.Tensor,     # [B, KVH, D]
    q_norm_w: torch.Tensor,  # [D]
    k_norm_w: torch.Tensor,  # [D]
    cos: torch.Tensor,       # [S_max, R]
    sin: torch.Tensor,       # [S_max, R]
    k_cache: torch.Tensor,   # [B, KVH, S_max, D] (row `pos` written)
    v_cache: torch.Tensor,
    positions: torch.Tensor, # [B] (one per query row)
    eps: float = 1e-6,
    n_tok: int = 1,
) -> torch.Tensor:
    """Gated GQA decode step (the reference's GQA tail + stateful KV append,
    ``qwen3.6-35b-a3b/kernels/gqa_tail_35b.py:52-394``): q/k RMSNorm(1+w),
    partial RoPE, append K/V at ``pos``, softmax over ``[0, pos]``, P.V,
    ``* sigmoid(gate)``.  Returns ``[B, QH*D]``.  With ``n_tok > 1`` the query
    rows are ``n_tok`` consecutive tokens per cache sequence (speculative
    verify): all new K/V rows are written first, then each row attends causally
    up to its own position."""
    B, QH, D2 = qg.shape
    D = D2 // 2
    KVH = k_new.shape[1]
    rep = QH // KVH
    q, gate = qg.float().split(D, dim=-1)
    pos = positions.long()
    c, s = cos[pos].float()[:, None], sin[pos].float()[:, None]
    q = apply_partial_rope(rms_norm(q, q_norm_w, eps), c, s)
    k = apply_partial_rope(rms_norm(k_new.float(), k_norm_w, eps), c, s)
    seq = torch.arange(B, device=qg.device) // n_tok
    k_cache[seq, :, pos] = k.to(k_cache.dtype)
    v_cache[seq, :, pos] = v_new.to(v_cache.dtype)
    out = torch.empty(B, QH, D, dtype=torch.float32, device=qg.device)
    for bi in range(B):
        L = int(pos[bi]) + 1
        kk = k_cache[bi // n_tok, :, :L].float().repeat_interleave(rep, 0)  # [QH, L, D]
        vv = v_cache[bi // n_tok, :, :L].float().repeat_interleave(rep, 0)
        sc = torch.einsum("hd,hld->hl", q[bi], kk) / math.sqrt(D)
        p = sc.softmax(-1)
        out[bi] = torch.einsum("hl,hld->hd", p, vv)
    out = out * torch.sigmoid(gate)
    return out.reshape(B, QH * D).to(qg.dtype)


def attention_prefill(
    q: torch.Tensor,        # [B, QH, S, D]  (normed + roped)
    k_cache: torch.Tensor,  # [B, KVH, S_max, D] (rows [0, start+S) valid)
    v_cache: torch.Tensor,
    start_pos: int,
    scale: float | None = None,
    causal: bool = True,
) -> torch.Tensor:
    """Prefix-aware causal attention: query row ``i`` sits at position
    ``start_pos+i`` and attends to cache rows ``[0, start_pos+i]`` (the CTE
    prefill over the used prefix, ``qwen3.6-35b-a3b/static_decode_35b.py:2316-2449``)."""
    B, QH, S, D = q.shape
    KVH = k_cache.shape[1]
    L = start_pos + S
    kk = k_cache[:, :, :L].float().repeat_interleave(QH // KVH, 1)
    vv = v_cache[:, :, :L].float().repeat_interleave(QH // KVH, 1)
    sc = torch.einsum("bhsd,bhld->bhsl", q.float(), kk) * (scale if scale is not None else 1.0 / math.sqrt(D))
    if causal:
        qpos = torch.arange(S, device=q.device)[:, None] + start_pos
        kpos = torch.arange(L, device=q.device)[None, :]
        sc = sc.masked_fill(kpos > qpos, -float("inf"))
    return torch.einsum("bhsl,bhld->bhsd", sc.softmax(-1), vv)


# --------------------------------------------------------------------------
# MoE
# --------------------------------------------------------------------------
def moe_route_softmax(logits: torch.Tensor, top_k: int, renorm: bool = True):
    """Qwen router: softmax -> top-k -> renormalise (HF ``Qwen3_5MoeTopKRouter``).
    Returns ``(weights [T,k] fp32, ids [T,k] int32)``."""
    p = logits.float().softmax(-1)
    w, i = torch.topk(p, top_k, dim=-1)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return w, i.int()


def moe_route_deepseek(logits: torch.Tensor, bias: torch.Tensor | None, top_k: int,
                       score_func: str = "sqrtsoftplus", route_scale: float = 1.5):
    """DeepSeek V4 gate (``run_deepseek_v4_tp.py:397-428``): score by
    ``sqrt(softplus(x))`` or ``sigmoid``; bias only affects selection;
    renormalise the selected scores and multiply by ``route_scale``."""
    lf = logits.float()
    s = F.softplus(lf).sqrt() if score_func == "sqrtsoftplus" else lf.sigmoid()
    sel = s + bias.float() if bias is not None else s
    idx = torch.topk(sel, top_k, dim=-1).indices
    w = s.gather(-1, idx)
    w = w / w.sum(-1, keepdim=True) * route_scale
    return w, idx.int()


def moe_experts(x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, gate_up: torch.Tensor,
                down: torch.Tensor, expert_offset: int = 0, swiglu_limit: float = 0.0) -> torch.Tensor:
    """Routed experts over the experts held locally (global ids
    ``[expert_offset, expert_offset+E_local)``); slots routed elsewhere contribute
    nothing, so summing the per-rank results gives the full MoE (the EP combine of
    ``static_decode_35b.py:810-821``).  ``gate_up [E,2I,H]``, ``down [E,H,I]``."""
    T, H = x.shape
    E = gate_up.shape[0]
    out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    xf = x.float()
    for e in range(E):
        hit = (ids == (e + expert_offset))
        t_idx, slot = hit.nonzero(as_tuple=True)
        if t_idx.numel() == 0:
            continue
        h = swiglu(xf[t_idx] @ gate_up[e].float().t(), swiglu_limit)
        y = h.float() @ down[e].float().t()
        out.index_add_(0, t_idx, y * w[t_idx, slot].float()[:, None])
    return out


# --------------------------------------------------------------------------
# greedy over a vocab-sharded head
# --------------------------------------------------------------------------
def sharded_greedy(local_logits: list[torch.Tensor]) -> torch.Tensor:
    """Global argmax across vocab shards with the lowest-id tie break
    (``static_decode_35b.py:1549-1560``)."""
    full = torch.cat([l.float() for l in local_logits], dim=-1)
    m = full.max(-1, keepdim=True).values
    ids = torch.arange(full.shape[-1], device=full.device)
    cand = torch.where(full == m, ids, torch.full_like(ids, full.shape[-1]))
    return cand.min(-1).values


# --------------------------------------------------------------------------
# DeepSeek V4: hyper-connections and single-KV-head attention
# --------------------------------------------------------------------------
def hc_pre(x, fn, scale, base, iters: int = 20, eps: float = 1e-6, norm_eps: float = 1e-6):
    """Hyper-Connection pre-mix (``run_deepseek_v4_tp.py:179-217``) on
    ``x [T, hc, dim]``; ``fn.shape[0] == hc`` selects the head variant (``:230-243``)."""
    T, hc, dim = x.shape
    xf = x.reshape(T, hc * dim).float()
    rs = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + norm_eps)
    mixes = (xf @ fn.float().t()) * rs
    if fn.shape[0] == hc:
        pre = torch.sigmoid(mixes * scale.float()[0] + base.float()) + eps
        y = (pre.unsqueeze(-1) * x.float()).sum(1)
        return y.to(x.dtype), None, None
    s, b = scale.float(), base.float()
    pre = torch.sigmoid(mixes[:, :hc] * s[0] + b[:hc]) + eps
    post = torch.sigmoid(mixes[:, hc:2 * hc] * s[1] + b[hc:2 * hc]) + eps
    m = torch.exp((mixes[:, 2 * hc:] * s[2] + b[2 * hc:]).view(T, hc, hc))
    for _ in range(iters):
        m = m / (m.sum(-1, keepdim=True) + eps)
        m = m / (m.sum(-2, keepdim=True) + eps)
    y = (pre.unsqueeze(-1) * x.float()).sum(1)
    return y.to(x.dtype), post, m


def hc_post(x, resid, post, comb):
    """``out[j] = post[j] x + sum_i comb[i][j] resid[i]`` (``:221-227``)."""
    out = post.unsqueeze(-1) * x.float().unsqueeze(-2) + (comb.unsqueeze(-1) * resid.float().unsqueeze(-2)).sum(1)
    return out.to(x.dtype)


def mqa_attn(q, kv, visible, q_per_seq: int, scale: float):
    rows, H, D = q.shape
    out = torch.empty(rows, H, D, dtype=torch.float32, device=q.device)
    for r in range(rows):
        b = r // q_per_seq
        L = int(visible[r])
        k = kv[b, :L].float()
        sc = (q[r].float() @ k.t()) * scale
        out[r] = sc.softmax(-1) @ k
    return out.to(q.dtype)


def deltanet_verify(qkv, z, a, b, stash_qkv, stash_ab, vstep, conv_ring, state, positions, pending, conv_w,
                    A_log, dt_bias, norm_w, k_heads: int, n_tok: int, eps: float = 1e-6) -> torch.Tensor:
    """Multi-token DeltaNet verify with deferred commit (oracle of
    ``deltanet_verify.cu``): commit the ``pending[b]`` stashed tokens of the last
    step into ``state``/``conv_ring``, run the ``n_tok`` new tokens per sequence
    on copies (outputs only), stash their raw rows under the other parity.
    Rows are ``[B*n_tok, *]``; returns ``[B*n_tok, VH*Dv]``."""
    B, VH, Dk, Dv = state.shape
    N = n_tok
    assert N <= stash_qkv.shape[2]
    par = int(vstep.reshape(-1)[0]) & 1
    out = torch.zeros(B * N, VH * Dv, dtype=qkv.dtype, device=qkv.device)
    for bi in range(B):
        p = int(positions[bi])
        if p < 0:
            continue
        na = int(pending[bi])
        for j in range(na):
            ab = stash_ab[par, bi, j]
            deltanet_decode(stash_qkv[par, bi, j][None], ab[None, :VH], ab[None, VH:],
                            torch.zeros(1, VH * Dv, dtype=qkv.dtype, device=qkv.device),
                            conv_ring[bi:bi + 1], state[bi:bi + 1], torch.tensor([p - na + j]), conv_w, A_log,
                            dt_bias, norm_w, k_heads, Dk, Dv, eps)
        ring_c, st_c = conv_ring[bi:bi + 1].clone(), state[bi:bi + 1].clone()
        for i in range(N):
            r = bi * N + i
            out[r] = deltanet_decode(qkv[r][None], a[r][None], b[r][None], z[r][None], ring_c, st_c,
                                     torch.tensor([p + i]), conv_w, A_log, dt_bias, norm_w, k_heads, Dk, Dv,
                                     eps)[0].to(out.dtype)
            stash_qkv[par ^ 1, bi, i] = qkv[r].to(stash_qkv.dtype)
            stash_ab[par ^ 1, bi, i, :VH] = a[r].to(stash_ab.dtype)
            stash_ab[par ^ 1, bi, i, VH:] = b[r].to(stash_ab.dtype)
    return out
