"""Qwen3.6 hybrid model (gated DeltaNet + gated GQA; dense SwiGLU or routed MoE).

One implementation serves Qwen3.6-27B (dense, ``StaticDecodeModule``,
``contrib/qwen3.6-27b/static_decode.py:374-963``) and Qwen3.6-35B-A3B (MoE,
``StaticDecode35B``, ``contrib/qwen3.6-35b-a3b/static_decode_35b.py:836-2449``).

Execution model (B200): one process per GPU, tensor-parallel over a process
group.  The decode step is a fixed-shape function of static buffers
(:class:`Qwen36State`) so it can be captured once as a CUDA graph
(:mod:`bwn.runtime.static_decode`), the analogue of the reference's
``torch.compile(backend="neuron", fullgraph=True)`` NEFF.  Every hot op is a
``torch.ops.bwn`` kernel:

* per DeltaNet layer: 1 fused in-projection GEMM ``[qkv|z|b|a]``, the fused
  recurrent kernel, the out-projection GEMM;
* per GQA layer: 1 fused ``[q/gate|k|v]`` GEMM, the fused decode-attention
  kernel (norms, RoPE, KV append, softmax, gate), ``o_proj``;
* SwiGLU MLP: gate/up GEMM with the SwiGLU epilogue, ``down`` GEMM;
* between sub-blocks: all-reduce (NCCL baseline or the fused NVLink kernels of
  :mod:`bwn.parallel.fused`), then the fused residual add + RMSNorm.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable

import torch
import torch.nn as nn

from .. import ops as O
from ..config import Qwen36Config, tp_dims
from ..io import qwen36_weights as W
from ..ops import reference as R
from ..parallel.comm import Comm


@dataclass
class Qwen36State:
    """Static per-sequence decode state (one writer per buffer per step)."""

    conv: torch.Tensor       # [L_dn, B, R, C]  conv ring (slot = position % R; R = 4, or 8 for verify)
    ssm: torch.Tensor        # [L_dn, B, VH, 128, 128]  recurrent state
    k_cache: torch.Tensor    # [L_gqa, B, KVH, S_max, D]
    v_cache: torch.Tensor
    positions: torch.Tensor  # [B] int32: position of the next token

    @property
    def batch(self) -> int:
        return self.positions.shape[0]

    def reset(self, rows=None) -> None:
        if rows is None:
            self.conv.zero_()
            self.ssm.zero_()
            self.positions.zero_()
        else:
            self.conv[:, rows] = 0
            self.ssm[:, rows] = 0
            self.positions[rows] = 0

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.conv, self.ssm, self.k_cache, self.v_cache))


@dataclass
class SpecBuffers:
    """Per-sequence buffers of speculative verification (deferred DeltaNet commit)."""

    n_tok: int               # tokens verified per step (drafts + 1)
    stash_qkv: torch.Tensor  # [L_dn, 2, B, n_tok, C] raw rows of the last verify, by step parity
    stash_ab: torch.Tensor   # [L_dn, 2, B, n_tok, 2*VH]
    pending: torch.Tensor    # [B] accepted tokens of the last verify not yet committed
    vstep: torch.Tensor      # [1] verify step counter (selects the stash parity)


class Qwen36Model(nn.Module):
    """Rank-local Qwen3.6 model.  Parameters hold this rank's shards only."""

    def __init__(self, cfg: Qwen36Config, comm: Comm | None = None, device="cpu", dtype=torch.bfloat16,
                 moe_sharding: str | None = None):
        super().__init__()
        from ..utils import env
        self.cfg = cfg
        self.comm = comm or Comm.single()
        self.tp = self.comm.size
        self.rank = self.comm.rank
        self.moe_sharding = moe_sharding or env.get("BWN_MOE_SHARDING")
        self.moe_shared_only = bool(env.get("BWN_MOE_SHARED_ONLY"))
        # vocab-parallel embedding (the reference's PREFILL_SHARDED_EMBED): each rank
        # keeps vocab/tp rows, ids outside its range read zeros, one sum all-reduce
        self.shard_embed = bool(env.get("BWN_SHARD_EMBED")) and self.comm.size > 1
        self.d = tp_dims(cfg, self.tp, self.rank, self.moe_sharding)
        if (cfg.is_moe and self.moe_sharding == "tp" and torch.device(device).type == "cuda"
                and (2 * cfg.moe_inter // self.tp) % 128):
            raise ValueError(f"moe_sharding='tp' at TP={self.tp}: each rank's gate/up slice has "
                             f"{2 * cfg.moe_inter // self.tp} rows; the grouped expert GEMM needs a multiple of 128")
        self.device = torch.device(device)
        self.dtype = dtype
        self.layers: list[dict[str, torch.Tensor]] = []
        self.g: dict[str, torch.Tensor] = {}
        cos, sin = R.rope_table(1, cfg.rope_dim, cfg.rope_theta, device=self.device)
        self.rope_cos, self.rope_sin = cos, sin
        self.fused_comm = None  # set by parallel.fused when the NVLink kernels are enabled

    # ------------------------------------------------------------------ load
    def load_hf(self, get: Callable[[str], torch.Tensor], fp8_experts: Callable | None = None) -> "Qwen36Model":
        """``fp8_experts(layer, e0, e1, c0, width)``, when given, supplies each MoE
        layer's routed experts as fp8 (see :meth:`bwn.io.checkpoint.Checkpoint.fp8_experts`)."""
        cfg, d = self.cfg, self.d
        self.layers = []
        for i in range(cfg.num_layers):
            ex = None
            if fp8_experts is not None and cfg.is_moe:
                tp_slice = d.moe_sharding == "tp"
                ex = fp8_experts(i, d.expert_offset, d.expert_offset + d.experts,
                                 self.rank * d.moe_inter if tp_slice else 0, d.moe_inter if tp_slice else None)
            t = W.fuse_layer(cfg, i, get, self.tp, self.rank, self.dtype, self.moe_sharding, experts=ex)
            self.layers.append({k: v.to(self.device) for k, v in t.items()})
        self.g = {k: v.to(self.device) for k, v in W.fuse_globals(cfg, get, self.tp, self.rank, self.dtype).items()}
        self._shard_embed_table()
        self._prepare_moe_decode()
        return self

    def embed(self, tokens: torch.Tensor) -> torch.Tensor:
        """Token embeddings ``[T, H]`` (the residual stream's start)."""
        if not self.shard_embed:
            return O.embedding(tokens.int(), self.g["embed"], 0)
        e = O.embedding(tokens.int(), self.g["embed"], self.d.vocab_offset)
        return self.comm.all_reduce_(e)

    def init_random(self, seed: int = 0, gen_device=None) -> "Qwen36Model":
        """Random-init weights from a seed (same model for every TP degree)."""
        cfg = self.cfg
        gd = gen_device or self.device
        self.layers = []
        for i in range(cfg.num_layers):
            hf = W.synthetic_hf_layer(cfg, i, seed, gd)
            t = W.fuse_layer(cfg, i, hf.__getitem__, self.tp, self.rank, self.dtype, self.moe_sharding)
            self.layers.append({k: v.to(self.device) for k, v in t.items()})
            del hf
        glob = W.synthetic_hf_globals(cfg, seed, gd)
        self.g = {k: v.to(self.device) for k, v in W.fuse_globals(cfg, glob.__getitem__, self.tp, self.rank,
                                                                   self.dtype).items()}
        self._shard_embed_table()
        self._prepare_moe_decode()
        return self

    def _shard_embed_table(self) -> None:
        if self.shard_embed:
            d = self.d
            self.g["embed"] = self.g["embed"][d.vocab_offset:d.vocab_offset + d.vocab].contiguous()

    def _prepare_moe_decode(self) -> None:
        """Tensors of the decode-sized MoE path (``_moe_decode``): the router with
        the shared-expert gate as one more row, and the routed experts with the
        shared expert appended as one more expert (``*_x``; the routed-only
        tensors become views of them, so nothing is stored twice).  With experts
        partitioned across ranks each rank appends the whole shared expert and
        computes it for its own slice of the tokens; with every expert sliced
        across ranks it appends its slice and computes it for all tokens."""
        cfg, d = self.cfg, self.d
        if not cfg.is_moe:
            return
        full = d.moe_sharding != "tp" and self.tp > 1
        for L in self.layers:
            L["router_x"] = torch.cat([L["router"], L["shared_gate"]], 0).contiguous()
            gu, dn = L["experts_gate_up"], L["experts_down"]
            sgu, sdn = L["shared_gate_up"], L["shared_down"]
            if full:  # every rank's slice, gathered (16-row interleave blocks stay whole)
                sgu = self.comm.all_gather_first(sgu.contiguous())
                sdn = self.comm.all_gather_last(sdn.contiguous()).contiguous()
            if not torch.is_tensor(gu) or sgu.shape[0] != gu.shape[1] or sdn.shape != dn.shape[1:]:
                continue  # fp8 experts or a shared expert of another width: kept on its own GEMMs
            gux = torch.cat([gu, sgu[None].to(gu.dtype)], 0)
            dnx = torch.cat([dn, sdn[None].to(dn.dtype)], 0)
            L["experts_gate_up_x"], L["experts_down_x"] = gux, dnx
            L["experts_gate_up"], L["experts_down"] = gux[:-1], dnx[:-1]

    FP8_KEYS = ("in_proj", "out_proj", "qkv_proj", "o_proj", "gate_up", "down", "shared_gate_up", "shared_down")

    def quantize_fp8(self, include_head: bool = True, experts: bool = False, dense: bool = True) -> "Qwen36Model":
        """Convert the projection weights to 128x128 block-scaled E4M3 (W8A16):
        the fp8 variant of the reference's ``--fp8-weights``
        (``contrib/qwen3.6-27b/static_decode.py:283-319``).  ``experts``: the
        routed experts too (:class:`~bwn.io.fp8.FP8Experts`, fp8 grouped GEMM;
        the reference's block-scaled FP8 MoE, ``moe_fused_w8_35b.py``)."""
        from ..io.fp8 import FP8Experts, FP8Weight
        for L in self.layers:
            for k in self.FP8_KEYS if dense else ():
                if k in L and torch.is_tensor(L[k]) and L[k].dim() == 2 and L[k].shape[1] % 16 == 0:
                    L[k] = FP8Weight.from_dense(L[k])
            if experts and torch.is_tensor(L.get("experts_gate_up_x")):
                # the shared expert rides along as the last expert, block-scaled like
                # the routed ones (as the official FP8 checkpoints store it)
                n = L["experts_gate_up_x"].shape[0] - 1
                gx = FP8Experts.from_interleaved(L["experts_gate_up_x"])
                dx = FP8Experts.quantize(L["experts_down_x"])
                L["experts_gate_up_x"], L["experts_down_x"] = gx, dx
                L["experts_gate_up"], L["experts_down"] = gx.select(0, n), dx.select(0, n)
            elif experts and torch.is_tensor(L.get("experts_gate_up")):
                L["experts_gate_up"] = FP8Experts.from_interleaved(L["experts_gate_up"])
                L["experts_down"] = FP8Experts.quantize(L["experts_down"])
        if include_head:
            self.g["lm_head"] = FP8Weight.from_dense(self.g["lm_head"])
        return self

    def weight_bytes(self) -> int:
        """Bytes of weights held on this rank, each storage counted once (the
        routed experts and the router are views of the decode path's stacks)."""
        seen: dict[int, int] = {}

        def add(t):
            if torch.is_tensor(t):
                st = t.untyped_storage()
                seen[st.data_ptr()] = max(seen.get(st.data_ptr(), 0), st.nbytes())
            elif t is not None and not isinstance(t, (int, float, str, bool)):
                for v in vars(t).values() if hasattr(t, "__dict__") else ():
                    if torch.is_tensor(v):
                        add(v)

        for L in self.layers:
            for v in L.values():
                add(v)
        for v in self.g.values():
            add(v)
        return sum(seen.values())

    # ----------------------------------------------------------------- state
    def new_state(self, batch: int, max_seq: int, ssm_dtype=torch.float32, ring_slots: int | None = None) -> Qwen36State:
        """Static decode buffers.  ``ring_slots`` (default the conv kernel size) is
        the position-addressed conv ring; speculative verify needs 8."""
        cfg, d = self.cfg, self.d
        dev = self.device
        R = ring_slots or cfg.conv_kernel
        st = Qwen36State(
            conv=torch.zeros(cfg.num_deltanet, batch, R, d.dn_qkv_dim, dtype=self.dtype, device=dev),
            ssm=torch.zeros(cfg.num_deltanet, batch, d.dn_v_heads, cfg.dn_k_dim, cfg.dn_v_dim, dtype=ssm_dtype,
                            device=dev),
            k_cache=torch.zeros(cfg.num_gqa, batch, d.kv_heads, max_seq, cfg.head_dim, dtype=self.dtype, device=dev),
            v_cache=torch.zeros(cfg.num_gqa, batch, d.kv_heads, max_seq, cfg.head_dim, dtype=self.dtype, device=dev),
            positions=torch.zeros(batch, dtype=torch.int32, device=dev),
        )
        self.ensure_rope(max_seq)
        return st

    def ensure_rope(self, max_seq: int) -> None:
        if self.rope_cos.shape[0] < max_seq:
            self.rope_cos, self.rope_sin = R.rope_table(max_seq, self.cfg.rope_dim, self.cfg.rope_theta,
                                                        device=self.device)

    # ---------------------------------------------------------------- decode
    def _reduce_add_norm(self, part: torch.Tensor, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """``x += all_reduce(part)``; return ``rmsnorm(x) * (1+w)``."""
        fc = self.fused_comm
        if fc is not None and fc.fits(part.shape[0]):
            return fc.allreduce_add_norm(part, x, w, self.cfg.rms_eps)
        if self.tp > 1:
            self.comm.all_reduce_(part)
        return O.add_rms_norm(part, x, w, self.cfg.rms_eps)

    def _row_parallel(self, a: torch.Tensor, w: torch.Tensor, x: torch.Tensor, norm_w: torch.Tensor) -> torch.Tensor:
        """Row-parallel projection + all-reduce + residual add + RMSNorm.  With the
        fused NVLink path this is one kernel (GEMM epilogue -> peer reduce)."""
        fc = self.fused_comm
        if fc is not None and fc.fits(a.shape[0]):
            return fc.gemm_allreduce_add_norm(a, w, x, norm_w, self.cfg.rms_eps)
        return self._reduce_add_norm(O.linear(a, w), x, norm_w)

    def _deltanet_decode(self, i: int, h: torch.Tensor, st: Qwen36State, di: int) -> torch.Tensor:
        L, d = self.layers[i], self.d
        C, Z, VH = d.dn_qkv_dim, d.dn_value_dim, d.dn_v_heads
        proj = O.linear(h, L["in_proj"])  # [B, C + Z + 2VH]
        qkv, z = proj[:, :C], proj[:, C:C + Z]
        b, a = proj[:, C + Z:C + Z + VH], proj[:, C + Z + VH:]
        return O.deltanet_decode(qkv, z, a, b, st.conv[di], st.ssm[di], st.positions, L["conv_w"], L["A_log"],
                                 L["dt_bias"], L["norm_w"], d.dn_k_heads, self.cfg.rms_eps)

    def _gqa_decode(self, i: int, h: torch.Tensor, st: Qwen36State, gi: int) -> torch.Tensor:
        L, d, cfg = self.layers[i], self.d, self.cfg
        B = h.shape[0]
        D, QH, KVH = cfg.head_dim, d.q_heads, d.kv_heads
        proj = O.linear(h, L["qkv_proj"])  # [B, QH*2D + 2*KVH*D]
        qg = proj[:, :QH * 2 * D].view(B, QH, 2 * D)
        k = proj[:, QH * 2 * D:QH * 2 * D + KVH * D].view(B, KVH, D)
        v = proj[:, QH * 2 * D + KVH * D:].view(B, KVH, D)
        return O.gqa_decode(qg, k, v, L["q_norm"], L["k_norm"], self.rope_cos, self.rope_sin, st.k_cache[gi],
                            st.v_cache[gi], st.positions, cfg.rms_eps)

    def _mlp(self, i: int, h: torch.Tensor) -> torch.Tensor:
        """Returns the (TP-partial) MLP / MoE output before the reduction."""
        L = self.layers[i]
        if self.cfg.is_moe:
            from .moe import qwen_moe_forward
            return qwen_moe_forward(self, L, h)
        return O.linear_swiglu(h, L["gate_up"])

    def moe_residual(self, i: int, h: torch.Tensor, x: torch.Tensor, nxt: torch.Tensor) -> torch.Tensor:
        """MoE sub-block with residual add + next RMSNorm.  With the expert-parallel
        all-to-all enabled (:func:`bwn.parallel.ep.enable_ep_all_to_all`) and enough
        tokens per rank, each rank routes its slice of the tokens through the
        NVLink all-to-all and the slices are all-gathered; otherwise each rank runs
        its experts over all tokens and the partials are all-reduced."""
        ep = getattr(self, "ep_a2a", None)
        T = h.shape[0]
        if self._moe_decode_ok(i, h) and (ep is None or T // self.tp < ep.min_tokens):
            return self._moe_decode(i, h, x, nxt)
        if ep is not None and T % self.tp == 0 and ep.min_tokens <= T // self.tp <= ep.T_max:
            from .moe import route
            L = self.layers[i]
            Ts = T // self.tp
            hs = h[self.rank * Ts:(self.rank + 1) * Ts]
            w, ids = route(self, L, hs)
            sy = O.linear(O.linear_swiglu(hs, L["shared_gate_up_full"]), L["shared_down_full"])
            sg = O.linear_f32(hs, L["shared_gate"])
            ys = ep.moe(hs, w, ids, L["experts_gate_up"], L["experts_down"], shared=(sy, sg))
            return O.add_rms_norm(self.comm.all_gather_first(ys), x, nxt, self.cfg.rms_eps)
        return self._reduce_add_norm(self._mlp(i, h), x, nxt)

    def _moe_decode_ok(self, i: int, h: torch.Tensor) -> bool:
        from ..utils import env
        cfg = self.cfg
        return (h.is_cuda and h.shape[0] <= 64 and "router_x" in self.layers[i]
                and cfg.hidden in (256, 512, 1024, 2048, 4096) and cfg.num_experts <= 512 and cfg.top_k <= 16
                and not self.moe_shared_only
                and bool(env.get("BWN_MOE_FUSED")))

    def _moe_decode(self, i: int, h: torch.Tensor, x: torch.Tensor, nxt: torch.Tensor) -> torch.Tensor:
        """Decode-sized MoE sub-block in four launches (``csrc/kernels/moe_decode.cu``):
        fused routing + gather, grouped gate/up, grouped down (the shared expert
        rides along as one more expert), then one combine kernel that also adds
        the residual and normalises (one GPU) or stores into the symmetric slot
        for the fused NVLink reduction (several GPUs)."""
        L, cfg, d = self.layers[i], self.cfg, self.d
        T = h.shape[0]
        o = O.ops()
        if "experts_gate_up_x" in L:
            if d.moe_sharding == "tp" or self.tp == 1:
                t_lo, t_hi = 0, T
            else:
                per = -(-T // self.tp)
                t_lo, t_hi = min(T, self.rank * per), min(T, (self.rank + 1) * per)
            gx, dx = L["experts_gate_up_x"], L["experts_down_x"]
            if hasattr(gx, "w8"):  # fp8 experts (shared expert folded in)
                args = (gx.w8, dx.w8, gx.scales16, dx.scales16)
            else:
                args = (gx, dx, None, None)
            y, w, pos_of, pos_sh, sg = o.moe_decode(h, L["router_x"], *args, d.expert_offset, cfg.num_experts,
                                                    cfg.top_k, cfg.norm_topk_prob, True, True, t_lo, t_hi, 0.0)
            shared_y = None
        else:  # fp8 experts; the bf16 shared expert on its own GEMMs, gated by the fused router's logit
            gu, dn = L["experts_gate_up"], L["experts_down"]
            y, w, pos_of, pos_sh, sg = o.moe_decode(h, L["router_x"], gu.w8, dn.w8, gu.scales16, dn.scales16,
                                                    d.expert_offset, cfg.num_experts, cfg.top_k, cfg.norm_topk_prob,
                                                    True, False, 0, 0, 0.0)
            shared_y = O.linear(O.linear_swiglu(h, L["shared_gate_up"]), L["shared_down"])
        shared_gate = sg if shared_y is not None else None
        if self.tp == 1:
            return o.moe_combine_ex(y, w, pos_of, pos_sh, sg, shared_y, shared_gate, 1, x, nxt, cfg.rms_eps)
        fc = self.fused_comm
        if fc is not None and fc.fits(T):
            if fc.one_kernel:  # combine, NVLS reduction, residual add and RMSNorm in one launch
                return o.moe_combine_symm_norm(y, w, pos_of, pos_sh, sg, shared_y, shared_gate, fc.local_ar, fc.mc_ar,
                                               fc.buf_elems, fc.peer_flags_ar, fc.peer_flags_ar[fc.rank], fc.state,
                                               fc.rank, x, nxt, cfg.rms_eps, fc.timeout_s)
            o.moe_combine_symm(y, w, pos_of, pos_sh, sg, shared_y, shared_gate, fc.local_ar, fc.buf_elems,
                               fc.peer_flags_ar, fc.state, fc.rank)
            return fc.reduce_add_norm(x, nxt, cfg.rms_eps)
        part = o.moe_combine_ex(y, w, pos_of, pos_sh, sg, shared_y, shared_gate, 0, None, None, 0.0)
        self.comm.all_reduce_(part)
        return O.add_rms_norm(part, x, nxt, cfg.rms_eps)

    def decode_hidden(self, tokens: torch.Tensor, st: Qwen36State, num_layers: int | None = None) -> torch.Tensor:
        """One decode step for ``tokens [B]`` at ``st.positions``; advances the
        positions and returns the final-normed hidden ``[B, H]``.  ``num_layers``
        (checks only) stops after that many layers and returns the hidden as
        normed for the next layer."""
        cfg = self.cfg
        x = self.embed(tokens)  # residual stream [B, H]
        h = O.rms_norm(x, self.layers[0]["in_norm"], cfg.rms_eps)
        di = gi = 0
        for i in range(cfg.num_layers if num_layers is None else num_layers):
            L = self.layers[i]
            if cfg.layer_type(i) == "deltanet":
                o = self._deltanet_decode(i, h, st, di)
                h = self._row_parallel(o, L["out_proj"], x, L["post_norm"])
                di += 1
            else:
                o = self._gqa_decode(i, h, st, gi)
                h = self._row_parallel(o, L["o_proj"], x, L["post_norm"])
                gi += 1
            nxt = self.layers[i + 1]["in_norm"] if i + 1 < cfg.num_layers else self.g["final_norm"]
            if cfg.is_moe:
                h = self.moe_residual(i, h, x, nxt)
            else:
                act = self._mlp(i, h)
                h = self._row_parallel(act, L["down"], x, nxt)
        st.positions.add_(1)
        return h

    # ------------------------------------------------------ speculative verify
    def new_spec_state(self, batch: int, n_tok: int) -> "SpecBuffers":
        """Stash / pending / step-counter buffers of multi-token verification
        (the decode state must come from ``new_state(..., ring_slots=8)``)."""
        d = self.d
        dev = self.device
        return SpecBuffers(
            n_tok=n_tok,
            stash_qkv=torch.zeros(self.cfg.num_deltanet, 2, batch, n_tok, d.dn_qkv_dim, dtype=self.dtype, device=dev),
            stash_ab=torch.zeros(self.cfg.num_deltanet, 2, batch, n_tok, 2 * d.dn_v_heads, dtype=self.dtype,
                                 device=dev),
            pending=torch.zeros(batch, dtype=torch.int32, device=dev),
            vstep=torch.zeros(1, dtype=torch.int32, device=dev),
        )

    def verify_hidden(self, tokens: torch.Tensor, st: Qwen36State, sp: "SpecBuffers",
                      feat_layers: tuple[int, ...] = ()) -> tuple[torch.Tensor, list[torch.Tensor]]:
        """Target forward over ``tokens [B, N]`` at positions ``st.positions + i``
        without committing them: DeltaNet layers first commit ``sp.pending`` tokens
        of the previous verify and only read the new ones; GQA layers write K/V at
        the new positions (overwritten later if rejected).  Positions are not
        advanced (the acceptance does it).  Returns the final-normed hidden
        ``[B*N, H]`` and the residual stream after each of ``feat_layers``."""
        cfg, d = self.cfg, self.d
        B, N = tokens.shape
        T = B * N
        pos_rows = (st.positions[:, None] + torch.arange(N, device=tokens.device, dtype=torch.int32)[None]).reshape(T)
        x = self.embed(tokens.reshape(T))
        h = O.rms_norm(x, self.layers[0]["in_norm"], cfg.rms_eps)
        feats = []
        di = gi = 0
        for i in range(cfg.num_layers):
            L = self.layers[i]
            if cfg.layer_type(i) == "deltanet":
                C, Z, VH = d.dn_qkv_dim, d.dn_value_dim, d.dn_v_heads
                proj = O.linear(h, L["in_proj"])
                o = O.deltanet_verify(proj[:, :C], proj[:, C:C + Z], proj[:, C + Z + VH:], proj[:, C + Z:C + Z + VH],
                                      sp.stash_qkv[di], sp.stash_ab[di], sp.vstep, st.conv[di], st.ssm[di],
                                      st.positions, sp.pending, L["conv_w"], L["A_log"], L["dt_bias"], L["norm_w"],
                                      d.dn_k_heads, N, cfg.rms_eps)
                h = self._row_parallel(o, L["out_proj"], x, L["post_norm"])
                di += 1
            else:
                D, QH, KVH = cfg.head_dim, d.q_heads, d.kv_heads
                proj = O.linear(h, L["qkv_proj"])
                qg = proj[:, :QH * 2 * D].view(T, QH, 2 * D)
                k = proj[:, QH * 2 * D:QH * 2 * D + KVH * D].view(T, KVH, D)
                v = proj[:, QH * 2 * D + KVH * D:].view(T, KVH, D)
                o = O.gqa_decode(qg, k, v, L["q_norm"], L["k_norm"], self.rope_cos, self.rope_sin, st.k_cache[gi],
                                 st.v_cache[gi], pos_rows, cfg.rms_eps, 0, N)
                h = self._row_parallel(o, L["o_proj"], x, L["post_norm"])
                gi += 1
            nxt = self.layers[i + 1]["in_norm"] if i + 1 < cfg.num_layers else self.g["final_norm"]
            if cfg.is_moe:
                h = self.moe_residual(i, h, x, nxt)
            else:
                h = self._row_parallel(self._mlp(i, h), L["down"], x, nxt)
            if i in feat_layers:
                feats.append((i, x.clone()))
        by_layer = dict(feats)
        return h, [by_layer[i] for i in feat_layers]

    def commit_pending(self, st: Qwen36State, sp: "SpecBuffers") -> None:
        """Fold the last verify's accepted tokens into the DeltaNet states (a
        verify with no new tokens); afterwards plain decode steps may follow."""
        cfg, d = self.cfg, self.d
        B = st.positions.shape[0]
        dev = st.positions.device
        C, VH = d.dn_qkv_dim, d.dn_v_heads
        empty = torch.zeros(0, C + d.dn_value_dim + 2 * VH, dtype=self.dtype, device=dev)
        di = 0
        for i in range(cfg.num_layers):
            if cfg.layer_type(i) != "deltanet":
                continue
            L = self.layers[i]
            O.deltanet_verify(empty[:, :C], empty[:, C:C + d.dn_value_dim], empty[:, :VH], empty[:, :VH],
                              sp.stash_qkv[di], sp.stash_ab[di], sp.vstep, st.conv[di], st.ssm[di], st.positions,
                              sp.pending, L["conv_w"], L["A_log"], L["dt_bias"], L["norm_w"], d.dn_k_heads, 0,
                              cfg.rms_eps)
            di += 1
        sp.pending.zero_()
        sp.vstep.add_(1)

    def greedy(self, h: torch.Tensor) -> torch.Tensor:
        """Vocab-sharded LM head + greedy with the lowest-id tie break
        (``static_decode_35b.py:1534-1564``) as a single int64 max all-reduce."""
        logits = O.linear(h, self.g["lm_head"])
        key = O.argmax_packed(logits, self.d.vocab_offset)
        fc = self.fused_comm
        if fc is not None and fc.fits(key.shape[0]):
            return fc.greedy(key)
        if self.tp > 1:
            self.comm.all_reduce_max_(key)
        return O.unpack_argmax(key)

    def sample(self, h: torch.Tensor, temperature: torch.Tensor, generator: torch.Generator | None = None
               ) -> torch.Tensor:
        """Temperature sampling on the vocab-sharded head by the Gumbel-max
        trick: ``argmax(logits / T + G)`` with iid standard Gumbel noise ``G`` is
        an exact sample of ``softmax(logits / T)``, so each rank perturbs only
        its own vocab shard and the same packed int64 max all-reduce as
        :meth:`greedy` picks the token.  ``temperature [B]`` (fp32, on the
        device; rows with T = 0 get exactly :meth:`greedy`'s token: the same
        head output, lowest id on ties)."""
        logits = O.linear(h, self.g["lm_head"]).float()
        t = temperature.float().reshape(-1, 1)
        u = torch.rand(logits.shape, device=logits.device, generator=generator).clamp_(1e-20, 1.0)
        noisy = torch.where(t > 0, logits / t.clamp_min(1e-6) - torch.log(-torch.log(u)), logits)
        key = O.argmax_packed(noisy, self.d.vocab_offset)
        fc = self.fused_comm
        if fc is not None and fc.fits(key.shape[0]):
            return fc.greedy(key)
        if self.tp > 1:
            self.comm.all_reduce_max_(key)
        return O.unpack_argmax(key)

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        """Full-vocab logits (gathered across vocab shards)."""
        local = O.linear_f32(h, self.g["lm_head"])
        return self.comm.all_gather_last(local)

    def decode_step(self, tokens: torch.Tensor, st: Qwen36State) -> torch.Tensor:
        return self.greedy(self.decode_hidden(tokens, st))

    # --------------------------------------------------------------- prefill
    def prefill_hidden(self, tokens: torch.Tensor, st: Qwen36State, valid_len: torch.Tensor | None = None,
                       chunk: int = 64, feat_layers: tuple[int, ...] = (), feats_out: list | None = None) -> torch.Tensor:
        """Process a prompt chunk ``tokens [B, S]`` starting at ``st.positions``
        (all rows share the start position, as in the reference's bucketed
        prefill, ``static_decode_35b.py:2497-2678``).  ``valid_len [B]`` marks
        real rows; pad rows leave every state untouched.  Returns the final-normed
        hidden of each row's last valid token ``[B, H]``."""
        from . import qwen36_prefill as P
        return P.prefill_hidden(self, tokens, st, valid_len, chunk, feat_layers, feats_out)

    def prefill(self, tokens: torch.Tensor, st: Qwen36State, valid_len=None, bucket: int = 0) -> torch.Tensor:
        """Bucketed prefill (``prefill_bucketed``): chunks of ``bucket`` tokens
        (whole prompt if 0); returns the greedy next token ids ``[B]``."""
        B, S = tokens.shape
        sp = getattr(self, "seq_parallel", None)
        if sp is not None and valid_len is None and (bucket == 0 or bucket >= S) and \
                (B * S) % (128 * self.tp) == 0 and B * S <= sp.T_max:
            from .qwen36_prefill import prefill_hidden_sp
            return self.greedy(prefill_hidden_sp(self, tokens, st, sp))
        bucket = bucket or S
        vl = valid_len if valid_len is not None else torch.full((B,), S, dtype=torch.int32, device=tokens.device)
        h = None
        for c0 in range(0, S, bucket):
            c1 = min(S, c0 + bucket)
            chunk_valid = (vl.to(tokens.device) - c0).clamp(0, c1 - c0).int()
            hc = self.prefill_hidden(tokens[:, c0:c1], st, chunk_valid)
            # keep the hidden of the last valid row seen so far per sequence
            h = hc if h is None else torch.where((chunk_valid > 0)[:, None], hc, h)
        return self.greedy(h)


def build_qwen36(cfg: Qwen36Config, comm: Comm | None = None, device="cpu", seed: int | None = 0,
                 hf_state: dict | None = None, dtype=torch.bfloat16, checkpoint: str | None = None,
                 moe_sharding: str | None = None, fp8_experts: bool = False) -> Qwen36Model:
    """A rank's model from an in-memory HF state dict, a safetensors checkpoint
    directory (HF layout, packed or per-expert MoE, official FP8 dequantized) or
    random init from ``seed``.  ``moe_sharding``: ``"ep"`` (experts partitioned
    across ranks) or ``"tp"`` (every expert sliced across ranks); default from
    ``BWN_MOE_SHARDING``.  ``fp8_experts``: an official FP8 checkpoint's routed
    experts stay fp8 (the fp8 grouped GEMM) instead of being dequantized."""
    m = Qwen36Model(cfg, comm, device, dtype, moe_sharding)
    if checkpoint is not None:
        from ..io.checkpoint import Checkpoint
        ck = Checkpoint(checkpoint)
        src = (lambda i, e0, e1, c0, w: ck.fp8_experts(f"layers.{i}.", e0, e1, c0, w)) if fp8_experts else None
        m.load_hf(ck.getter(), fp8_experts=src)
        ck.close()
    elif hf_state is not None:
        m.load_hf(W.hf_getter(hf_state))
    elif seed is not None:
        m.init_random(seed)
    return m


def from_pretrained(path: str, comm: Comm | None = None, device="cpu", dtype=torch.bfloat16,
                    fp8_experts: bool = False) -> Qwen36Model:
    """Config from ``config.json`` plus weights from the safetensors beside it."""
    from ..config import qwen36_from_hf
    return build_qwen36(qwen36_from_hf(path), comm, device, None, None, dtype, checkpoint=path,
                        fp8_experts=fp8_experts)


def param_gb(cfg: Qwen36Config) -> float:
    return cfg.param_count() * 2 / 1e9


def attn_scale(cfg: Qwen36Config) -> float:
    return 1.0 / math.sqrt(cfg.head_dim)
