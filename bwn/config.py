"""Typed model configurations and tensor-parallel dimension helpers.

One dataclass per model family replaces the reference's module-level constant
blocks and import-time env reads:

* Qwen3.6 hybrid (dense 27B and MoE 35B-A3B) -- constants in
  ``contrib/qwen3.6-27b/static_decode.py:101-130`` and
  ``contrib/qwen3.6-35b-a3b/model_dims.py:20-78``; per-rank split in
  ``contrib/qwen3.6-35b-a3b/model_dims.py:99-127`` (``tp_dims``) and HF
  ``config.json`` override in ``model_dims.py:130-179`` (``load_from_config``).
* DeepSeek V4 Flash -- ``contrib/deepseek-v4-flash/run_deepseek_v4_tp.py:40-119``.
* ESM-2 -- the HF ``facebook/esm2_t*`` family used by ``contrib/esm2/train_esm.py``.

Kernel shape parameters are passed as launch arguments derived from these
objects, never read from the environment.
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, replace
from typing import Any


@dataclass(frozen=True)
class Qwen36Config:
    """Qwen3.6 hybrid backbone: ``[DeltaNet x3, GQA x1]`` repeated.

    ``intermediate > 0`` selects a dense SwiGLU MLP on every layer (27B);
    ``num_experts > 0`` selects the routed MoE with a sigmoid-gated shared
    expert on every layer (35B-A3B).
    """

    name: str = "qwen3.6-27b"
    num_layers: int = 64
    hidden: int = 5120
    vocab: int = 248320
    rms_eps: float = 1e-6
    full_attn_interval: int = 4
    # gated DeltaNet (linear attention)
    dn_k_heads: int = 16
    dn_v_heads: int = 48
    dn_k_dim: int = 128
    dn_v_dim: int = 128
    conv_kernel: int = 4
    # gated GQA (full attention)
    q_heads: int = 24
    kv_heads: int = 4
    head_dim: int = 256
    partial_rotary: float = 0.25
    rope_theta: float = 1e7
    # dense MLP
    intermediate: int = 17408
    # MoE
    num_experts: int = 0
    top_k: int = 0
    moe_inter: int = 0
    shared_inter: int = 0
    norm_topk_prob: bool = True
    tie_embeddings: bool = False

    # ---- derived -----------------------------------------------------------
    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def rope_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary)

    @property
    def dn_key_dim(self) -> int:
        return self.dn_k_heads * self.dn_k_dim

    @property
    def dn_value_dim(self) -> int:
        return self.dn_v_heads * self.dn_v_dim

    @property
    def dn_qkv_dim(self) -> int:
        return 2 * self.dn_key_dim + self.dn_value_dim

    def layer_type(self, i: int) -> str:
        """``gqa`` iff ``i % interval == interval-1`` (``static_decode.py:133-135``)."""
        return "gqa" if i % self.full_attn_interval == self.full_attn_interval - 1 else "deltanet"

    @property
    def num_gqa(self) -> int:
        return sum(1 for i in range(self.num_layers) if self.layer_type(i) == "gqa")

    @property
    def num_deltanet(self) -> int:
        return self.num_layers - self.num_gqa

    def deltanet_index(self, i: int) -> int:
        return sum(1 for j in range(i) if self.layer_type(j) == "deltanet")

    def gqa_index(self, i: int) -> int:
        return sum(1 for j in range(i) if self.layer_type(j) == "gqa")

    def param_count(self) -> int:
        h = self.hidden
        dn = h * (self.dn_qkv_dim + self.dn_value_dim + 2 * self.dn_v_heads) + self.dn_value_dim * h
        dn += self.dn_qkv_dim * self.conv_kernel + 2 * self.dn_v_heads + self.dn_v_dim
        gqa = h * (self.q_heads * self.head_dim * 2 + 2 * self.kv_heads * self.head_dim)
        gqa += self.q_heads * self.head_dim * h + 2 * self.head_dim
        if self.is_moe:
            mlp = self.num_experts * 3 * h * self.moe_inter + self.num_experts * h
            mlp += 3 * h * self.shared_inter + h
        else:
            mlp = 3 * h * self.intermediate
        per = [dn if self.layer_type(i) == "deltanet" else gqa for i in range(self.num_layers)]
        total = sum(per) + self.num_layers * (mlp + 2 * h)
        total += self.vocab * h * (1 if self.tie_embeddings else 2) + h
        return total

    def scaled(self, **kw: Any) -> "Qwen36Config":
        return replace(self, **kw)


QWEN36_27B = Qwen36Config()

QWEN36_35B_A3B = Qwen36Config(
    name="qwen3.6-35b-a3b",
    num_layers=40,
    hidden=2048,
    vocab=248320,
    dn_k_heads=16,
    dn_v_heads=32,
    q_heads=16,
    kv_heads=2,
    intermediate=0,
    num_experts=256,
    top_k=8,
    moe_inter=512,
    shared_inter=512,
)


def tiny_qwen36(moe: bool = False, layers: int = 4) -> Qwen36Config:
    """Small shape-faithful variant for CPU tests (same head dims as production)."""
    base = QWEN36_35B_A3B if moe else QWEN36_27B
    kw = dict(
        name=base.name + "-tiny",
        num_layers=layers,
        hidden=256,
        vocab=512,
        dn_k_heads=2,
        dn_v_heads=4,
        q_heads=4,
        kv_heads=2,
        head_dim=256,
        dn_k_dim=128,
        dn_v_dim=128,
    )
    if moe:
        kw.update(num_experts=16, top_k=4, moe_inter=64, shared_inter=64)
    else:
        kw.update(intermediate=512)
    return replace(base, **kw)


@dataclass(frozen=True)
class TPDims:
    """Per-rank dimensions of a Qwen3.6 model under tensor/expert parallelism.

    Mirrors ``model_dims.tp_dims`` (``contrib/qwen3.6-35b-a3b/model_dims.py:99-127``):
    DeltaNet K/V heads and attention Q heads split evenly; KV heads are
    replicated when ``tp > kv_heads``; experts are partitioned ``E/tp`` per rank
    (``moe_sharding="ep"``), or every rank holds every expert with a ``1/tp``
    slice of its intermediate width (``"tp"``, the reference's MOE_DECODE_TP,
    ``static_decode_35b.py:746-768``: the routed work is balanced across ranks
    whatever the routing).
    """

    tp: int
    rank: int
    dn_k_heads: int
    dn_v_heads: int
    dn_qkv_dim: int
    dn_value_dim: int
    q_heads: int
    kv_heads: int  # KV heads held locally (>= 1; replicated when tp > kv_heads)
    kv_head_offset: int  # first global KV head held by this rank
    kv_replication: int
    intermediate: int
    experts: int
    expert_offset: int
    vocab: int
    vocab_offset: int
    moe_sharding: str = "ep"
    moe_inter: int = 0  # intermediate width of each held expert


MOE_SHARDINGS = ("ep", "tp")


def tp_dims(cfg: Qwen36Config, tp: int, rank: int = 0, moe_sharding: str = "ep") -> TPDims:
    if cfg.dn_k_heads % tp or cfg.dn_v_heads % tp:
        raise ValueError(f"DeltaNet heads ({cfg.dn_k_heads}/{cfg.dn_v_heads}) must divide tp={tp}")
    if cfg.q_heads % tp:
        raise ValueError(f"q_heads={cfg.q_heads} must divide tp={tp}")
    if moe_sharding not in MOE_SHARDINGS:
        raise ValueError(f"moe_sharding={moe_sharding!r}: expected one of {MOE_SHARDINGS}")
    expert_tp = cfg.is_moe and moe_sharding == "tp"
    if cfg.is_moe and not expert_tp and cfg.num_experts % tp:
        raise ValueError(f"num_experts={cfg.num_experts} must divide tp={tp}")
    if expert_tp and (cfg.moe_inter % tp or (cfg.moe_inter // tp) % 16):
        raise ValueError(f"moe_inter={cfg.moe_inter} must split over tp={tp} into multiples of 16")
    if not cfg.is_moe and cfg.intermediate % tp:
        raise ValueError(f"intermediate={cfg.intermediate} must divide tp={tp}")
    if cfg.vocab % tp:
        raise ValueError(f"vocab={cfg.vocab} must divide tp={tp}")
    qh = cfg.q_heads // tp
    if tp >= cfg.kv_heads:
        if tp % cfg.kv_heads:
            raise ValueError("tp must be a multiple of kv_heads when tp > kv_heads")
        rep = tp // cfg.kv_heads
        kvh, kv_off = 1, rank // rep
    else:
        if cfg.kv_heads % tp:
            raise ValueError("kv_heads must divide tp")
        rep = 1
        kvh = cfg.kv_heads // tp
        kv_off = rank * kvh
    dk, dv = cfg.dn_k_heads // tp, cfg.dn_v_heads // tp
    return TPDims(
        tp=tp,
        rank=rank,
        dn_k_heads=dk,
        dn_v_heads=dv,
        dn_qkv_dim=(2 * dk * cfg.dn_k_dim + dv * cfg.dn_v_dim),
        dn_value_dim=dv * cfg.dn_v_dim,
        q_heads=qh,
        kv_heads=kvh,
        kv_head_offset=kv_off,
        kv_replication=rep,
        intermediate=(cfg.intermediate // tp) if not cfg.is_moe else 0,
        experts=(cfg.num_experts if expert_tp else cfg.num_experts // tp) if cfg.is_moe else 0,
        expert_offset=(0 if expert_tp else rank * (cfg.num_experts // tp)) if cfg.is_moe else 0,
        vocab=cfg.vocab // tp,
        vocab_offset=rank * (cfg.vocab // tp),
        moe_sharding=moe_sharding if cfg.is_moe else "ep",
        moe_inter=(cfg.moe_inter // tp if expert_tp else cfg.moe_inter) if cfg.is_moe else 0,
    )


def qwen36_from_hf(path_or_dict: str | dict) -> Qwen36Config:
    """Build a config from an HF ``config.json`` (``model_dims.py:130-179``)."""
    if isinstance(path_or_dict, str):
        p = path_or_dict
        if os.path.isdir(p):
            p = os.path.join(p, "config.json")
        with open(p) as f:
            d = json.load(f)
    else:
        d = dict(path_or_dict)
    d = d.get("text_config", d)
    rope = d.get("rope_parameters") or d.get("rope_scaling") or {}
    kw = dict(
        name=d.get("model_type", "qwen3.6"),
        num_layers=d["num_hidden_layers"],
        hidden=d["hidden_size"],
        vocab=d["vocab_size"],
        rms_eps=d.get("rms_norm_eps", 1e-6),
        full_attn_interval=d.get("full_attention_interval", 4),
        dn_k_heads=d["linear_num_key_heads"],
        dn_v_heads=d["linear_num_value_heads"],
        dn_k_dim=d["linear_key_head_dim"],
        dn_v_dim=d["linear_value_head_dim"],
        conv_kernel=d.get("linear_conv_kernel_dim", 4),
        q_heads=d["num_attention_heads"],
        kv_heads=d["num_key_value_heads"],
        head_dim=d.get("head_dim", 256),
        partial_rotary=rope.get("partial_rotary_factor", d.get("partial_rotary_factor", 0.25)),
        rope_theta=rope.get("rope_theta", d.get("rope_theta", 1e7)),
        intermediate=d.get("intermediate_size", 0) if not d.get("num_experts") else 0,
        num_experts=d.get("num_experts", 0) or 0,
        top_k=d.get("num_experts_per_tok", 0) or 0,
        moe_inter=d.get("moe_intermediate_size", 0) or 0,
        shared_inter=d.get("shared_expert_intermediate_size", 0) or 0,
        norm_topk_prob=d.get("norm_topk_prob", True),
        tie_embeddings=d.get("tie_word_embeddings", False),
    )
    return Qwen36Config(**kw)


def qwen36_to_hf(cfg: Qwen36Config) -> dict:
    """The HF ``config.json`` fields :func:`qwen36_from_hf` reads (for writing
    checkpoints this framework can load back)."""
    d = {
        "model_type": cfg.name, "num_hidden_layers": cfg.num_layers, "hidden_size": cfg.hidden,
        "vocab_size": cfg.vocab, "rms_norm_eps": cfg.rms_eps, "full_attention_interval": cfg.full_attn_interval,
        "linear_num_key_heads": cfg.dn_k_heads, "linear_num_value_heads": cfg.dn_v_heads,
        "linear_key_head_dim": cfg.dn_k_dim, "linear_value_head_dim": cfg.dn_v_dim,
        "linear_conv_kernel_dim": cfg.conv_kernel, "num_attention_heads": cfg.q_heads,
        "num_key_value_heads": cfg.kv_heads, "head_dim": cfg.head_dim,
        "rope_parameters": {"rope_type": "default", "rope_theta": cfg.rope_theta,
                            "partial_rotary_factor": cfg.partial_rotary},
        "tie_word_embeddings": cfg.tie_embeddings, "norm_topk_prob": cfg.norm_topk_prob,
    }
    if cfg.num_experts:
        d.update(num_experts=cfg.num_experts, num_experts_per_tok=cfg.top_k, moe_intermediate_size=cfg.moe_inter,
                 shared_expert_intermediate_size=cfg.shared_inter)
    else:
        d["intermediate_size"] = cfg.intermediate
    return d


@dataclass(frozen=True)
class DeepSeekV4Config:
    """DeepSeek V4 Flash dims (``run_deepseek_v4_tp.py:40-81``).

    The reference reads hidden/head dims/ranks from the HF ``config.json``
    (``:84-119``); the defaults here follow the public V4-Flash config
    (284B total, 13B active, 43 layers, vocab 129280, 256 routed experts).
    """

    name: str = "deepseek-v4-flash"
    vocab: int = 129280
    dim: int = 4096
    num_layers: int = 43
    n_heads: int = 64
    head_dim: int = 512
    rope_head_dim: int = 64
    q_lora_rank: int = 1024
    o_lora_rank: int = 1024
    o_groups: int = 8
    n_routed_experts: int = 256
    n_shared_experts: int = 1
    n_activated_experts: int = 6
    moe_inter: int = 2048
    n_hash_layers: int = 3
    score_func: str = "sqrtsoftplus"
    route_scale: float = 1.5
    swiglu_limit: float = 10.0
    hc_mult: int = 4
    hc_sinkhorn_iters: int = 20
    hc_eps: float = 1e-6
    norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    max_seq_len: int = 8192
    window_size: int = 128
    compress_ratios: tuple = ()

    def scaled(self, **kw: Any) -> "DeepSeekV4Config":
        return replace(self, **kw)

    def param_count(self) -> int:
        d, h, hd = self.dim, self.n_heads, self.head_dim
        attn = d * self.q_lora_rank + self.q_lora_rank * h * hd + d * hd
        attn += (h * hd // self.o_groups) * self.o_lora_rank * self.o_groups + self.o_groups * self.o_lora_rank * d
        moe = (self.n_routed_experts + self.n_shared_experts) * 3 * d * self.moe_inter + self.n_routed_experts * d
        hc = 2 * (2 + self.hc_mult) * self.hc_mult * self.hc_mult * d
        return self.num_layers * (attn + moe + hc) + 2 * self.vocab * d


def tiny_deepseek_v4() -> DeepSeekV4Config:
    return DeepSeekV4Config(
        name="deepseek-v4-tiny", vocab=512, dim=128, num_layers=3, n_heads=8, head_dim=64,
        rope_head_dim=16, q_lora_rank=64, o_lora_rank=64, o_groups=2, n_routed_experts=16,
        n_activated_experts=4, moe_inter=64, n_hash_layers=1, max_seq_len=256,
    )


def deepseek_v4_from_hf(path_or_dict: str | dict) -> DeepSeekV4Config:
    """Map an HF DeepSeek-V4 ``config.json`` onto :class:`DeepSeekV4Config`
    (``run_deepseek_v4_tp.py:84-119``)."""
    if isinstance(path_or_dict, str):
        p = os.path.join(path_or_dict, "config.json") if os.path.isdir(path_or_dict) else path_or_dict
        with open(p) as f:
            d = json.load(f)
    else:
        d = dict(path_or_dict)
    m = {
        "vocab_size": "vocab", "hidden_size": "dim", "num_hidden_layers": "num_layers",
        "num_attention_heads": "n_heads", "head_dim": "head_dim", "qk_rope_head_dim": "rope_head_dim",
        "q_lora_rank": "q_lora_rank", "o_lora_rank": "o_lora_rank", "o_groups": "o_groups",
        "n_routed_experts": "n_routed_experts", "n_shared_experts": "n_shared_experts",
        "num_experts_per_tok": "n_activated_experts", "moe_intermediate_size": "moe_inter",
        "num_hash_layers": "n_hash_layers", "scoring_func": "score_func",
        "routed_scaling_factor": "route_scale", "swiglu_limit": "swiglu_limit",
        "hc_mult": "hc_mult", "hc_sinkhorn_iters": "hc_sinkhorn_iters", "rms_norm_eps": "norm_eps",
        "rope_theta": "rope_theta", "sliding_window": "window_size",
    }
    kw = {v: d[k] for k, v in m.items() if k in d}
    if "compress_ratios" in d:
        kw["compress_ratios"] = tuple(d["compress_ratios"])
    return DeepSeekV4Config(**kw)


@dataclass(frozen=True)
class ESM2Config:
    """ESM-2 (HF ``EsmForMaskedLM``): pre-LN BERT with rotary embeddings, GELU FFN."""

    name: str = "esm2_t6_8M"
    num_layers: int = 6
    hidden: int = 320
    heads: int = 20
    ffn: int = 1280
    vocab: int = 33
    max_positions: int = 1026
    layer_norm_eps: float = 1e-5
    mask_token_id: int = 32
    pad_token_id: int = 1
    cls_token_id: int = 0
    eos_token_id: int = 2
    token_dropout: bool = True

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    def param_count(self) -> int:
        h = self.hidden
        layer = 4 * h * h + 4 * h + 2 * h * self.ffn + self.ffn + h + 4 * h
        return self.num_layers * layer + self.vocab * h + h * h + 4 * h + self.vocab


ESM2_SIZES = {
    "8M": ESM2Config(),
    "35M": ESM2Config(name="esm2_t12_35M", num_layers=12, hidden=480, heads=20, ffn=1920),
    "150M": ESM2Config(name="esm2_t30_150M", num_layers=30, hidden=640, heads=20, ffn=2560),
    "650M": ESM2Config(name="esm2_t33_650M", num_layers=33, hidden=1280, heads=20, ffn=5120),
    "3B": ESM2Config(name="esm2_t36_3B", num_layers=36, hidden=2560, heads=40, ffn=10240),
    "15B": ESM2Config(name="esm2_t48_15B", num_layers=48, hidden=5120, heads=40, ffn=20480),
}

# ESM-2 alphabet (the order HF's EsmTokenizer vocab file uses).
ESM_ALPHABET = [
    "<cls>", "<pad>", "<eos>", "<unk>", "L", "A", "G", "V", "S", "E", "R", "T", "I", "D", "P",
    "K", "Q", "N", "F", "Y", "M", "H", "W", "C", "X", "B", "U", "Z", "O", ".", "-", "<null_1>",
    "<mask>",
]
ESM_STANDARD_AA = list("LAGVSERTIDPKQNFYMHWC")


def to_dict(cfg) -> dict:
    return dataclasses.asdict(cfg)
