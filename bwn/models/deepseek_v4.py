"""DeepSeek V4 Flash (MLA-style single-KV-head attention, Hyper-Connections,
256-expert MoE) -- the reference's TP/EP model
(``contrib/deepseek-v4-flash/run_deepseek_v4_tp.py:261-650``).

Parameter names follow the reference module (its state dict is the checkpoint
layout the pre-sharding script writes, ``preprocess_weights.py:80-121``).
Per rank:

* attention: ``wq_a``/``q_norm``/``wkv``/``kv_norm`` replicated, ``wq_b``
  column-parallel by heads, ``wo_a`` restricted to this rank's head groups,
  ``wo_b`` row-parallel over the matching o_lora slices -> all-reduce;
* MoE: gate (+ selection bias after the hash layers) replicated, experts
  partitioned (EP), shared expert tensor-parallel; partials all-reduced;
* Hyper-Connections: ``hc_mult`` residual streams, fused pre-mix (GEMV +
  Sinkhorn + contraction) and post-mix kernels.

On CUDA every op is a bwn kernel (tcgen05 GEMMs, grouped MoE GEMMs, hc_pre /
hc_post, interleaved RoPE, single-KV-head attention); on CPU the same code runs
the fp32 references.
"""
from __future__ import annotations

import math

import torch

from .. import ops as O
from ..config import DeepSeekV4Config
from ..io.qwen36_weights import seeded_tensor
from ..parallel.comm import Comm


class DeepSeekV4State:
    def __init__(self, cfg: DeepSeekV4Config, batch: int, max_seq: int, device, dtype=torch.bfloat16):
        self.kv = torch.zeros(cfg.num_layers, batch, max_seq, cfg.head_dim, dtype=dtype, device=device)
        self.positions = torch.zeros(batch, dtype=torch.int32, device=device)


def synthetic_checkpoint(cfg: DeepSeekV4Config, seed: int, device="cpu") -> dict:
    """Random-init weights in the reference's state-dict layout."""
    sd = {}
    d, hd, E, I = cfg.dim, cfg.head_dim, cfg.n_routed_experts, cfg.moe_inter
    mix = (2 + cfg.hc_mult) * cfg.hc_mult

    def t(name, shape, kind="normal", std=0.02, dtype=torch.bfloat16):
        sd[name] = seeded_tensor(name, shape, seed, device, kind, std, dtype)

    t("embed.weight", (cfg.vocab, d), std=1.0)
    t("head.weight", (cfg.vocab, d))
    t("norm.weight", (d,), "ones", dtype=torch.float32)
    t("hc_head_fn", (cfg.hc_mult, cfg.hc_mult * d), std=0.02, dtype=torch.float32)
    t("hc_head_base", (cfg.hc_mult,), "zeros", dtype=torch.float32)
    t("hc_head_scale", (1,), "ones", dtype=torch.float32)
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        t(p + "attn_norm.weight", (d,), "ones", dtype=torch.float32)
        t(p + "ffn_norm.weight", (d,), "ones", dtype=torch.float32)
        for w in ("attn", "ffn"):
            t(p + f"hc_{w}_fn", (mix, cfg.hc_mult * d), std=0.02, dtype=torch.float32)
            t(p + f"hc_{w}_base", (mix,), "normal", 0.1, dtype=torch.float32)
            t(p + f"hc_{w}_scale", (3,), "ones", dtype=torch.float32)
        a = p + "attn."
        t(a + "wq_a.weight", (cfg.q_lora_rank, d))
        t(a + "q_norm.weight", (cfg.q_lora_rank,), "ones", dtype=torch.float32)
        t(a + "wq_b.weight", (cfg.n_heads * hd, cfg.q_lora_rank))
        t(a + "wkv.weight", (hd, d))
        t(a + "kv_norm.weight", (hd,), "ones", dtype=torch.float32)
        t(a + "wo_a.weight", (cfg.o_groups * cfg.o_lora_rank, cfg.n_heads * hd // cfg.o_groups))
        t(a + "wo_b.weight", (d, cfg.o_groups * cfg.o_lora_rank))
        f = p + "ffn."
        t(f + "gate.weight", (E, d))
        if i >= cfg.n_hash_layers:
            t(f + "gate.bias", (E,), "normal", 0.01, dtype=torch.float32)
        t(f + "experts_w1", (E, I, d))
        t(f + "experts_w3", (E, I, d))
        t(f + "experts_w2", (E, d, I))
        t(f + "shared_experts.w1.weight", (I, d))
        t(f + "shared_experts.w3.weight", (I, d))
        t(f + "shared_experts.w2.weight", (d, I))
    return sd


def _expert_stack(sd, f, name, e0, e1):
    """Experts ``[e0, e1)`` as one tensor, from either the stacked or the
    per-expert (``experts.{e}.wN.weight``) layout."""
    if f + f"experts_{name}" in sd:
        return sd[f + f"experts_{name}"][e0:e1]
    return torch.stack([sd[f + f"experts.{e}.{name}.weight"] for e in range(e0, e1)])


def _unshard_view(sd: dict, cfg: DeepSeekV4Config, tp: int, rank: int) -> dict:
    """Present a pre-sharded rank file under the full-checkpoint names the loader
    slices: local experts move to their global ids, ``wq_b`` / ``wo_b`` /
    shared-expert slices are placed in zero-padded full tensors at this rank's
    offsets (only that window is read back)."""
    out = dict(sd)
    per = cfg.n_routed_experts // tp
    for k in list(sd):
        parts = k.split(".")
        if "experts" in parts and ".shared_experts." not in k:
            i = parts.index("experts")
            if i + 1 < len(parts) and parts[i + 1].isdigit():
                parts[i + 1] = str(rank * per + int(parts[i + 1]))
                out.pop(k)
                out[".".join(parts)] = sd[k]
        elif k.endswith(".wq_b.weight"):
            t = sd[k]
            full = t.new_zeros(t.shape[0] * tp, t.shape[1])
            full[rank * t.shape[0]:(rank + 1) * t.shape[0]] = t
            out[k] = full
        elif k.endswith(".wo_b.weight"):
            t = sd[k]
            full = t.new_zeros(t.shape[0], t.shape[1] * tp)
            full[:, rank * t.shape[1]:(rank + 1) * t.shape[1]] = t
            out[k] = full
    return out


class DeepSeekV4Model:
    """``comm`` is the tensor-parallel group of the attention.  ``ep_comm``
    (optional) is a separate expert-parallel group: the hybrid layout of the
    reference (``run_deepseek_v4_hybrid.py:36-37, 437-460, 516-585, 760-763``),
    where TP groups are consecutive ranks and EP groups are strided by the TP
    size; routed experts and the shared expert are then split over the EP group
    and the MoE partials all-reduced there.  Without it, one group does both."""

    def __init__(self, cfg: DeepSeekV4Config, comm: Comm | None = None, device="cpu", dtype=torch.bfloat16,
                 ep_comm: Comm | None = None):
        self.cfg = cfg
        self.comm = comm or Comm.single()
        self.ep_comm = ep_comm or self.comm
        self.tp, self.rank = self.comm.size, self.comm.rank
        self.ep, self.ep_rank = self.ep_comm.size, self.ep_comm.rank
        if cfg.n_heads % self.tp or cfg.o_groups % self.tp or cfg.n_routed_experts % self.ep:
            raise ValueError("tp must divide n_heads and o_groups, ep must divide n_routed_experts")
        self.device = torch.device(device)
        self.dtype = dtype
        self.heads = cfg.n_heads // self.tp
        self.groups = cfg.o_groups // self.tp
        self.e_local = cfg.n_routed_experts // self.ep
        self.e0 = self.ep_rank * self.e_local
        half = cfg.rope_head_dim // 2
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, cfg.rope_head_dim, 2, dtype=torch.float32) / cfg.rope_head_dim))
        f = torch.outer(torch.arange(cfg.max_seq_len, dtype=torch.float32), inv)
        self.cos, self.sin = f.cos().to(self.device), f.sin().to(self.device)
        assert self.cos.shape[1] == half
        self.L: list[dict] = []
        self.g: dict = {}
        self.ones_hd = torch.ones(cfg.head_dim, device=self.device)
        self.fused_comm = None  # set by bwn.parallel.fused.enable_fused_comm

    # ------------------------------------------------------------------ load
    def load(self, sd: dict, presharded: bool = False) -> "DeepSeekV4Model":
        """Load a full state dict (sliced here per rank) or, with ``presharded``,
        this rank's file from :func:`bwn.io.deepseek_weights.preprocess`
        (experts renumbered from 0, ``wq_b``/``wo_b`` already split)."""
        cfg, dt, dev = self.cfg, self.dtype, self.device
        hd, r = cfg.head_dim, self.rank
        h0, h1 = r * self.heads, (r + 1) * self.heads
        g0, g1 = r * self.groups, (r + 1) * self.groups
        olr = cfg.o_lora_rank
        E, I = cfg.n_routed_experts, cfg.moe_inter
        Is = I // self.ep
        re = self.ep_rank
        if presharded:
            sd = _unshard_view(sd, cfg, self.tp, r)
        self.L = []
        for i in range(cfg.num_layers):
            p, a, f = f"layers.{i}.", f"layers.{i}.attn.", f"layers.{i}.ffn."
            L = {
                "attn_norm": sd[p + "attn_norm.weight"].float(),
                "ffn_norm": sd[p + "ffn_norm.weight"].float(),
                "hc_attn": (sd[p + "hc_attn_fn"].float(), sd[p + "hc_attn_scale"].float(), sd[p + "hc_attn_base"].float()),
                "hc_ffn": (sd[p + "hc_ffn_fn"].float(), sd[p + "hc_ffn_scale"].float(), sd[p + "hc_ffn_base"].float()),
                "wq_a": sd[a + "wq_a.weight"].to(dt),
                "q_norm": sd[a + "q_norm.weight"].float(),
                "wq_b": sd[a + "wq_b.weight"][h0 * hd:h1 * hd].to(dt),
                "wkv": sd[a + "wkv.weight"].to(dt),
                "kv_norm": sd[a + "kv_norm.weight"].float(),
                "wo_a": sd[a + "wo_a.weight"].view(cfg.o_groups, olr, -1)[g0:g1].to(dt),
                "wo_b": sd[a + "wo_b.weight"][:, g0 * olr:g1 * olr].to(dt),
                "gate": sd[f + "gate.weight"].to(dt),
                "gate_bias": sd[f + "gate.bias"].float() if (f + "gate.bias") in sd else None,
            }
            w1 = _expert_stack(sd, f, "w1", self.e0, self.e0 + self.e_local)
            w3 = _expert_stack(sd, f, "w3", self.e0, self.e0 + self.e_local)
            L["experts_gate_up"] = torch.stack([O.interleave_gate_up(w1[e], w3[e]) for e in range(self.e_local)]).to(dt)
            L["experts_down"] = _expert_stack(sd, f, "w2", self.e0, self.e0 + self.e_local).to(dt)
            L["shared_gate_up"] = O.interleave_gate_up(sd[f + "shared_experts.w1.weight"][re * Is:(re + 1) * Is],
                                                       sd[f + "shared_experts.w3.weight"][re * Is:(re + 1) * Is]).to(dt)
            L["shared_down"] = sd[f + "shared_experts.w2.weight"][:, re * Is:(re + 1) * Is].to(dt)
            self.L.append({k: (tuple(x.to(dev) for x in v) if isinstance(v, tuple) else
                               (v.to(dev).contiguous() if v is not None else None)) for k, v in L.items()})
        self.g = {
            "embed": sd["embed.weight"].to(dt).to(dev),
            "head": sd["head.weight"].to(dt).to(dev),
            "norm": sd["norm.weight"].float().to(dev),
            "hc_head": tuple(sd[k].float().to(dev) for k in ("hc_head_fn", "hc_head_scale", "hc_head_base")),
        }
        return self

    def load_checkpoint(self, path: str, presharded: bool | None = None) -> "DeepSeekV4Model":
        """Load safetensors: a per-rank preprocessed file (``rank{r}.safetensors``
        in ``path``) or a full checkpoint in the reference's state-dict layout.
        FP8 pairs (``w`` + ``w_scale_inv``) are dequantized to the model dtype."""
        import os
        from ..io.checkpoint import Checkpoint
        from ..io.fp8 import dequantize_block
        rank_file = os.path.join(path, f"rank{self.rank}.safetensors")
        if presharded is None:
            presharded = os.path.isfile(rank_file)
        ck = Checkpoint(rank_file if presharded else path, prefix="")
        sd = {}
        for k in ck.wm:
            if k.endswith("_scale_inv"):
                continue
            t = ck.raw(k)
            if (k + "_scale_inv") in ck.wm:
                t = dequantize_block(t, ck.raw(k + "_scale_inv").float()).to(self.dtype)
            sd[k] = t
        self.load(sd, presharded=presharded)
        ck.close()
        return self

    FP8_KEYS = ("wq_a", "wq_b", "wkv", "wo_b", "shared_gate_up", "shared_down")

    def quantize_fp8(self, include_head: bool = True, experts: bool = False) -> "DeepSeekV4Model":
        """Dense projections (and the LM head) as 128x128 block-scaled E4M3
        (W8A16), the layout of the checkpoint's FP8 dense weights; with
        ``experts`` the routed experts too (:class:`~bwn.io.fp8.FP8Experts` on
        the fp8 grouped GEMM, clamped SwiGLU in its epilogue)."""
        from ..io.fp8 import FP8Experts, FP8Weight
        for L in self.L:
            for k in self.FP8_KEYS:
                w = L.get(k)
                if torch.is_tensor(w) and w.dim() == 2 and w.shape[1] % 16 == 0:
                    L[k] = FP8Weight.from_dense(w)
            if experts and torch.is_tensor(L.get("experts_gate_up")):
                L["experts_gate_up"] = FP8Experts.from_interleaved(L["experts_gate_up"])
                L["experts_down"] = FP8Experts.quantize(L["experts_down"])
        if include_head:
            self.g["head"] = FP8Weight.from_dense(self.g["head"])
        return self

    def init_random_local(self, seed: int = 0) -> "DeepSeekV4Model":
        """Random-init only this rank's shards, directly on the device (full-size
        models: the whole synthetic state dict would not fit in host memory).
        The weights differ between tensor-parallel degrees; for benchmarks."""
        cfg, dt, dev = self.cfg, self.dtype, self.device
        hd, olr, I = cfg.head_dim, cfg.o_lora_rank, cfg.moe_inter
        Is = I // self.ep
        mix = (2 + cfg.hc_mult) * cfg.hc_mult
        g = torch.Generator(device=dev).manual_seed(seed * 1000 + self.rank)

        def rn(*shape, std=0.02, dtype=dt):
            return (torch.randn(*shape, device=dev, generator=g, dtype=torch.float32) * std).to(dtype)

        def ones(n):
            return torch.ones(n, device=dev)

        self.L = []
        for i in range(cfg.num_layers):
            L = {
                "attn_norm": ones(cfg.dim), "ffn_norm": ones(cfg.dim),
                "hc_attn": (rn(mix, cfg.hc_mult * cfg.dim, dtype=torch.float32), ones(3),
                            rn(mix, std=0.1, dtype=torch.float32)),
                "hc_ffn": (rn(mix, cfg.hc_mult * cfg.dim, dtype=torch.float32), ones(3),
                           rn(mix, std=0.1, dtype=torch.float32)),
                "wq_a": rn(cfg.q_lora_rank, cfg.dim), "q_norm": ones(cfg.q_lora_rank),
                "wq_b": rn(self.heads * hd, cfg.q_lora_rank), "wkv": rn(hd, cfg.dim), "kv_norm": ones(hd),
                "wo_a": rn(self.groups, olr, cfg.n_heads * hd // cfg.o_groups),
                "wo_b": rn(cfg.dim, self.groups * olr),
                "gate": rn(cfg.n_routed_experts, cfg.dim),
                "gate_bias": rn(cfg.n_routed_experts, std=0.01, dtype=torch.float32)
                if i >= cfg.n_hash_layers else None,
                "experts_gate_up": rn(self.e_local, 2 * I, cfg.dim),
                "experts_down": rn(self.e_local, cfg.dim, I),
                "shared_gate_up": rn(2 * Is, cfg.dim), "shared_down": rn(cfg.dim, Is),
            }
            self.L.append(L)
        self.g = {"embed": rn(cfg.vocab, cfg.dim, std=1.0), "head": rn(cfg.vocab, cfg.dim), "norm": ones(cfg.dim),
                  "hc_head": (rn(cfg.hc_mult, cfg.hc_mult * cfg.dim, dtype=torch.float32), ones(1),
                              torch.zeros(cfg.hc_mult, device=dev))}
        return self

    def init_random(self, seed: int = 0) -> "DeepSeekV4Model":
        return self.load(synthetic_checkpoint(self.cfg, seed, "cpu"))

    def new_state(self, batch: int, max_seq: int) -> DeepSeekV4State:
        return DeepSeekV4State(self.cfg, batch, max_seq, self.device, self.dtype)

    # --------------------------------------------------------------- blocks
    def _allreduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.tp > 1:
            self.comm.all_reduce_(x)
        return x

    def _attn(self, L, x, st: DeepSeekV4State, li: int, pos: torch.Tensor, bidx: torch.Tensor, q_per_seq: int,
              mix):
        """Attention sub-block; returns the new residual streams
        ``hc_post(all_reduce(out), *mix)`` with ``mix = (h, post, comb)``."""
        cfg = self.cfg
        T, hd, rd = x.shape[0], cfg.head_dim, cfg.rope_head_dim
        eps = cfg.norm_eps
        q = O.linear(O.rms_norm(O.linear(x, L["wq_a"]), L["q_norm"], eps, one_plus=False), L["wq_b"])
        q = O.rms_norm(q.view(T * self.heads, hd), self.ones_hd, 1e-6, one_plus=False).view(T, self.heads, hd)
        kv = O.rms_norm(O.linear(x, L["wkv"]), L["kv_norm"], eps, one_plus=False).view(T, 1, hd)
        if rd > 0:
            O.rope_interleaved_(q, self.cos, self.sin, pos)
            O.rope_interleaved_(kv, self.cos, self.sin, pos)
        cache = st.kv[li]  # [B, S, hd]
        S = cache.shape[1]
        cache.view(-1, hd).index_copy_(0, (bidx.long() * S + pos.long()), kv.view(T, hd))
        o = O.mqa_attn(q, cache, pos + 1, q_per_seq, 1.0 / math.sqrt(hd))  # [T, H, hd]
        hpg = cfg.n_heads // cfg.o_groups
        og = o.view(T, self.groups, hpg * hd)
        olr = cfg.o_lora_rank
        lora = torch.empty(T, self.groups * olr, dtype=x.dtype, device=x.device)
        for g in range(self.groups):  # grouped low-rank projection straight into its column slice
            O.linear_into(og[:, g], L["wo_a"][g], lora[:, g * olr:(g + 1) * olr])
        fc = self.fused_comm
        if fc is not None and fc.fits(T):  # row-parallel GEMM -> NVLS all-reduce + hc_post (fused path F1)
            return fc.gemm_allreduce_hc_post(lora, L["wo_b"], *mix)
        return O.hc_post(self._allreduce(O.linear(lora, L["wo_b"])), *mix)

    def _moe(self, L, x, li: int, mix):
        """MoE sub-block (routed + shared experts); returns ``hc_post(y, *mix)``."""
        cfg = self.cfg
        logits = O.linear_f32(x, L["gate"])
        w, ids = O.moe_topk_deepseek(logits, L["gate_bias"], cfg.n_activated_experts, cfg.score_func, cfg.route_scale)
        routed = O.moe_experts(x, w, ids, L["experts_gate_up"], L["experts_down"], self.e0,
                               swiglu_limit=cfg.swiglu_limit)
        shared = O.linear(O.linear_swiglu(x, L["shared_gate_up"]), L["shared_down"])
        y = (routed.float() + shared.float()).to(x.dtype)
        if self.ep > 1:
            fc = self.fused_comm
            if fc is not None and self.ep_comm is self.comm and fc.fits(y.shape[0]):
                return fc.allreduce_hc_post(y, *mix)
            self.ep_comm.all_reduce_(y)
        return O.hc_post(y, *mix)

    def forward_tokens(self, tokens: torch.Tensor, pos: torch.Tensor, bidx: torch.Tensor, st: DeepSeekV4State,
                       q_per_seq: int) -> torch.Tensor:
        """Run flattened tokens ``[T]`` (positions ``pos``, sequence ``bidx``)
        through every layer, writing their K/V rows; returns final hidden ``[T, dim]``."""
        cfg = self.cfg
        hc = cfg.hc_mult
        x0 = O.embedding(tokens.int(), self.g["embed"], 0)
        h = x0.unsqueeze(1).expand(-1, hc, -1).contiguous()  # [T, hc, dim]
        for li, L in enumerate(self.L):
            fn, sc, bs = L["hc_attn"]
            x, post, comb = O.hc_pre(h, fn, sc, bs, cfg.hc_sinkhorn_iters, cfg.hc_eps, cfg.norm_eps)
            h = self._attn(L, O.rms_norm(x, L["attn_norm"], cfg.norm_eps, one_plus=False), st, li, pos, bidx,
                           q_per_seq, (h, post, comb))
            fn, sc, bs = L["hc_ffn"]
            x, post, comb = O.hc_pre(h, fn, sc, bs, cfg.hc_sinkhorn_iters, cfg.hc_eps, cfg.norm_eps)
            h = self._moe(L, O.rms_norm(x, L["ffn_norm"], cfg.norm_eps, one_plus=False), li, (h, post, comb))
        fn, sc, bs = self.g["hc_head"]
        y, _, _ = O.hc_pre(h, fn, sc, bs, cfg.hc_sinkhorn_iters, cfg.hc_eps, cfg.norm_eps)
        return O.rms_norm(y, self.g["norm"], cfg.norm_eps, one_plus=False)

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return O.linear_f32(hidden, self.g["head"])

    def prefill(self, tokens: torch.Tensor, st: DeepSeekV4State) -> torch.Tensor:
        """``tokens [B, S]`` from position 0; returns next ids ``[B]``."""
        B, S = tokens.shape
        dev = self.device
        pos = torch.arange(S, device=dev, dtype=torch.int32).repeat(B)
        bidx = torch.arange(B, device=dev, dtype=torch.int32).repeat_interleave(S)
        h = self.forward_tokens(tokens.reshape(-1).to(dev), pos, bidx, st, S)
        st.positions.fill_(S)
        last = h.view(B, S, -1)[:, -1]
        return self.logits(last).argmax(-1).int()

    def decode_step(self, tokens: torch.Tensor, st: DeepSeekV4State) -> torch.Tensor:
        B = tokens.shape[0]
        bidx = torch.arange(B, device=self.device, dtype=torch.int32)
        h = self.forward_tokens(tokens.to(self.device), st.positions, bidx, st, 1)
        st.positions.add_(1)
        return self.logits(h).argmax(-1).int()


def main(argv=None) -> None:
    """The runner command (``contrib/deepseek-v4-flash/run_deepseek_v4_tp.py:730-907``
    and its hybrid / tiny twins): load a checkpoint (HF-layout safetensors, or
    the per-rank files of :func:`bwn.io.deepseek_weights.preprocess`) or a
    random tiny model, prefill a prompt, greedy-decode ``--max-new`` tokens;
    prints TTFT, decode tok/s, the ids and a NaN check.  One process per GPU
    under torchrun; ``--hybrid-tp N`` splits the world into TP groups of N and
    EP groups strided by N.

        torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m bwn.models.deepseek_v4 --checkpoint DIR
        python -m bwn.models.deepseek_v4 --tiny --cpu --max-new 8
    """
    import argparse
    import json
    import time

    import torch.distributed as dist

    from ..config import deepseek_v4_from_hf, tiny_deepseek_v4
    from ..ops import check_status
    from ..parallel.comm import hybrid_groups, init_distributed

    ap = argparse.ArgumentParser(description="DeepSeek V4 greedy generation")
    ap.add_argument("--checkpoint", "--model-path", default="",
                    help="checkpoint directory (config.json beside the weights), or the per-rank files of "
                         "bwn.io.deepseek_weights (detected)")
    ap.add_argument("--presharded", action="store_true", help="per-rank files from bwn.io.deepseek_weights")
    ap.add_argument("--tiny", action="store_true", help="random tiny model instead of a checkpoint")
    ap.add_argument("--prompt-ids", default="", help="comma-separated prompt ids (random when empty)")
    ap.add_argument("--prompt-len", type=int, default=32)
    ap.add_argument("--max-new", type=int, default=8)
    ap.add_argument("--max-cache", type=int, default=128)
    ap.add_argument("--hybrid-tp", type=int, default=0)
    ap.add_argument("--fp8", action="store_true")
    ap.add_argument("--cpu", action="store_true")
    a = ap.parse_args(argv)

    cpu = a.cpu or not torch.cuda.is_available()
    comm = init_distributed("gloo" if cpu else "nccl")
    dev = torch.device("cpu") if cpu else torch.device("cuda", torch.cuda.current_device())
    dtype = torch.float32 if cpu else torch.bfloat16
    ep_comm = None
    if a.hybrid_tp and comm.size > 1:
        comm, ep_comm = hybrid_groups(a.hybrid_tp)
    if a.checkpoint and not a.tiny:
        cfg = deepseek_v4_from_hf(a.checkpoint)
        model = DeepSeekV4Model(cfg, comm, dev, dtype, ep_comm=ep_comm)
        model.load_checkpoint(a.checkpoint, a.presharded or None)
    else:
        cfg = tiny_deepseek_v4()
        model = DeepSeekV4Model(cfg, comm, dev, dtype, ep_comm=ep_comm).init_random(0)
    if a.fp8:
        model.quantize_fp8()
    if a.prompt_ids:
        prompt = torch.tensor([[int(t) for t in a.prompt_ids.split(",") if t.strip()]])
    else:
        prompt = torch.randint(0, cfg.vocab, (1, a.prompt_len), generator=torch.Generator().manual_seed(0))
    S = prompt.shape[1]
    max_gen = min(a.max_new, a.max_cache - S)
    st = model.new_state(1, a.max_cache)

    def sync():
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)

    sync()
    t0 = time.perf_counter()
    nxt = model.prefill(prompt.to(dev), st)
    sync()
    ttft = time.perf_counter() - t0
    ids = [int(nxt[0])]
    t1 = time.perf_counter()
    for _ in range(max_gen - 1):
        nxt = model.decode_step(nxt, st)
        ids.append(int(nxt[0]))
    sync()
    dt = time.perf_counter() - t1
    check_status("deepseek generate")
    h = model.forward_tokens(nxt.to(dev), st.positions, torch.zeros(1, dtype=torch.int32, device=dev), st, 1)
    finite = bool(torch.isfinite(model.logits(h)).all())
    multi = dist.is_available() and dist.is_initialized()
    if (dist.get_rank() if multi else 0) == 0:
        print(json.dumps({"model": cfg.name, "world": dist.get_world_size() if multi else 1,
                          "tp": model.tp, "ep": model.ep, "prompt_len": S, "generated": ids,
                          "ttft_s": round(ttft, 3),
                          "decode_tok_s": round((len(ids) - 1) / dt, 2) if len(ids) > 1 and dt > 0 else None,
                          "finite": finite}))
    if multi:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
