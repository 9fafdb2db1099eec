"""HF Qwen3.5/3.6 checkpoint layout -> per-rank fused weights.

The reference slices HF tensors per TP rank by hand
(``contrib/qwen3.6-27b/static_decode.py:968-1055`` ``shard_*``;
``contrib/qwen3.6-35b-a3b/static_decode_35b.py:2682-2964``
``load_sharded_weights``: group-aware qkv/conv slices ``:2889-2912``, KV
replication ``:2916-2928``, experts per rank, vocab-sharded head).  This module
does the same slicing and then fuses what the B200 kernels consume together:

* DeltaNet ``in_proj = [qkv | z | b | a]`` (one GEMM per layer);
* GQA ``qkv_proj = [q/gate (HF per-head interleave) | k | v]``;
* SwiGLU ``gate_up`` interleaved in 16-row blocks (fused epilogue);
* norms and gate parameters kept fp32.

Random init (``synthetic_hf_layer``) generates the full HF-layout tensors from a
seed per parameter name, so the model is identical for every TP degree.
"""
from __future__ import annotations

import hashlib
import math
from typing import Callable

import torch

from ..config import Qwen36Config, tp_dims
from ..ops import interleave_gate_up

HF_PREFIXES = ("model.language_model.", "model.", "language_model.model.", "")


def _seed_of(name: str, seed: int) -> int:
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 63) - 1)


def seeded_tensor(name: str, shape, seed: int, device, kind: str = "normal", std: float = 0.02,
                  dtype=torch.bfloat16) -> torch.Tensor:
    """Deterministic tensor for ``name``: the same values on every rank and TP
    degree for a given generation device type (CPU and CUDA generators differ)."""
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(_seed_of(name, seed))
    if kind == "normal":
        t = torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * std
    elif kind == "uniform":
        lo, hi = std
        t = torch.rand(shape, generator=g, device=dev, dtype=torch.float32) * (hi - lo) + lo
    elif kind == "zeros":
        t = torch.zeros(shape, device=dev)
    elif kind == "ones":
        t = torch.ones(shape, device=dev)
    else:
        raise ValueError(kind)
    return t.to(dtype)


def synthetic_hf_layer(cfg: Qwen36Config, i: int, seed: int, device) -> dict[str, torch.Tensor]:
    """HF-layout tensors of layer ``i`` with random-init values (names without prefix)."""
    H = cfg.hidden
    p = f"layers.{i}."
    out: dict[str, torch.Tensor] = {}
    std = 0.02
    out[p + "input_layernorm.weight"] = seeded_tensor(p + "in_norm", (H,), seed, device, "normal", 0.05, torch.float32)
    out[p + "post_attention_layernorm.weight"] = seeded_tensor(p + "post_norm", (H,), seed, device, "normal", 0.05,
                                                               torch.float32)
    if cfg.layer_type(i) == "deltanet":
        a = p + "linear_attn."
        C = cfg.dn_qkv_dim
        out[a + "in_proj_qkv.weight"] = seeded_tensor(a + "qkv", (C, H), seed, device, std=std)
        out[a + "in_proj_z.weight"] = seeded_tensor(a + "z", (cfg.dn_value_dim, H), seed, device, std=std)
        out[a + "in_proj_b.weight"] = seeded_tensor(a + "b", (cfg.dn_v_heads, H), seed, device, std=std)
        out[a + "in_proj_a.weight"] = seeded_tensor(a + "a", (cfg.dn_v_heads, H), seed, device, std=std)
        out[a + "conv1d.weight"] = seeded_tensor(a + "conv", (C, 1, cfg.conv_kernel), seed, device, "normal", 0.3,
                                                 torch.float32)
        out[a + "dt_bias"] = seeded_tensor(a + "dt", (cfg.dn_v_heads,), seed, device, "ones", dtype=torch.float32)
        out[a + "A_log"] = seeded_tensor(a + "A", (cfg.dn_v_heads,), seed, device, "uniform", (0.0, 2.7),
                                         torch.float32)
        out[a + "norm.weight"] = seeded_tensor(a + "norm", (cfg.dn_v_dim,), seed, device, "ones", dtype=torch.float32)
        out[a + "out_proj.weight"] = seeded_tensor(a + "out", (H, cfg.dn_value_dim), seed, device, std=std)
    else:
        a = p + "self_attn."
        D = cfg.head_dim
        out[a + "q_proj.weight"] = seeded_tensor(a + "q", (cfg.q_heads * D * 2, H), seed, device, std=std)
        out[a + "k_proj.weight"] = seeded_tensor(a + "k", (cfg.kv_heads * D, H), seed, device, std=std)
        out[a + "v_proj.weight"] = seeded_tensor(a + "v", (cfg.kv_heads * D, H), seed, device, std=std)
        out[a + "o_proj.weight"] = seeded_tensor(a + "o", (H, cfg.q_heads * D), seed, device, std=std)
        out[a + "q_norm.weight"] = seeded_tensor(a + "qn", (D,), seed, device, "normal", 0.05, torch.float32)
        out[a + "k_norm.weight"] = seeded_tensor(a + "kn", (D,), seed, device, "normal", 0.05, torch.float32)
    m = p + "mlp."
    if cfg.is_moe:
        E, I = cfg.num_experts, cfg.moe_inter
        out[m + "gate.weight"] = seeded_tensor(m + "router", (E, H), seed, device, std=std)
        out[m + "experts.gate_up_proj"] = seeded_tensor(m + "egu", (E, 2 * I, H), seed, device, std=std)
        out[m + "experts.down_proj"] = seeded_tensor(m + "ed", (E, H, I), seed, device, std=std)
        Is = cfg.shared_inter
        out[m + "shared_expert.gate_proj.weight"] = seeded_tensor(m + "sg", (Is, H), seed, device, std=std)
        out[m + "shared_expert.up_proj.weight"] = seeded_tensor(m + "su", (Is, H), seed, device, std=std)
        out[m + "shared_expert.down_proj.weight"] = seeded_tensor(m + "sd", (H, Is), seed, device, std=std)
        out[m + "shared_expert_gate.weight"] = seeded_tensor(m + "sgate", (1, H), seed, device, std=std)
    else:
        I = cfg.intermediate
        out[m + "gate_proj.weight"] = seeded_tensor(m + "g", (I, H), seed, device, std=std)
        out[m + "up_proj.weight"] = seeded_tensor(m + "u", (I, H), seed, device, std=std)
        out[m + "down_proj.weight"] = seeded_tensor(m + "d", (H, I), seed, device, std=std)
    return out


def synthetic_hf_global(cfg: Qwen36Config, name: str, seed: int, device) -> torch.Tensor:
    """One of the non-layer tensors (``embed_tokens.weight``, ``norm.weight``,
    ``lm_head.weight``) with its random-init values."""
    H, V = cfg.hidden, cfg.vocab
    if name == "embed_tokens.weight":
        return seeded_tensor("embed", (V, H), seed, device, std=1.0)
    if name == "norm.weight":
        return seeded_tensor("final_norm", (H,), seed, device, "normal", 0.05, torch.float32)
    if name == "lm_head.weight" and not cfg.tie_embeddings:
        return seeded_tensor("lm_head", (V, H), seed, device, std=0.02)
    raise KeyError(name)


def synthetic_hf_global_names(cfg: Qwen36Config) -> list[str]:
    return ["embed_tokens.weight", "norm.weight"] + ([] if cfg.tie_embeddings else ["lm_head.weight"])


def synthetic_hf_globals(cfg: Qwen36Config, seed: int, device) -> dict[str, torch.Tensor]:
    return {n: synthetic_hf_global(cfg, n, seed, device) for n in synthetic_hf_global_names(cfg)}


# --------------------------------------------------------------------------
# per-rank slicing + fusion
# --------------------------------------------------------------------------
def fuse_layer(cfg: Qwen36Config, i: int, get: Callable[[str], torch.Tensor], tp: int, rank: int,
               dtype=torch.bfloat16, moe_sharding: str = "ep", experts: tuple | None = None) -> dict[str, torch.Tensor]:
    """Build the rank-local fused tensors of layer ``i``; ``get(name)`` returns an
    HF-layout tensor (name without the ``model.`` prefix).  ``experts``: this
    rank's routed experts already built (e.g. fp8 ``(gate_up, down)`` straight
    from an official FP8 checkpoint); they are not read through ``get``."""
    d = tp_dims(cfg, tp, rank, moe_sharding)
    p = f"layers.{i}."
    out: dict[str, torch.Tensor] = {
        "in_norm": get(p + "input_layernorm.weight").float(),
        "post_norm": get(p + "post_attention_layernorm.weight").float(),
    }
    if cfg.layer_type(i) == "deltanet":
        a = p + "linear_attn."
        Dk, Dv, KD = cfg.dn_k_dim, cfg.dn_v_dim, cfg.dn_key_dim
        kh0, kh1 = rank * d.dn_k_heads, (rank + 1) * d.dn_k_heads
        vh0, vh1 = rank * d.dn_v_heads, (rank + 1) * d.dn_v_heads
        ch = torch.cat([
            torch.arange(kh0 * Dk, kh1 * Dk),
            torch.arange(KD + kh0 * Dk, KD + kh1 * Dk),
            torch.arange(2 * KD + vh0 * Dv, 2 * KD + vh1 * Dv),
        ])
        qkv = get(a + "in_proj_qkv.weight")
        qkv = qkv[ch.to(qkv.device)]
        z = get(a + "in_proj_z.weight")[vh0 * Dv:vh1 * Dv]
        b = get(a + "in_proj_b.weight")[vh0:vh1]
        aa = get(a + "in_proj_a.weight")[vh0:vh1]
        out["in_proj"] = torch.cat([qkv, z, b, aa], 0).to(dtype).contiguous()
        conv = get(a + "conv1d.weight")
        out["conv_w"] = conv.reshape(conv.shape[0], -1)[ch.to(conv.device)].float().contiguous()
        out["dt_bias"] = get(a + "dt_bias")[vh0:vh1].float().contiguous()
        out["A_log"] = get(a + "A_log")[vh0:vh1].float().contiguous()
        out["norm_w"] = get(a + "norm.weight").float().contiguous()
        out["out_proj"] = get(a + "out_proj.weight")[:, vh0 * Dv:vh1 * Dv].to(dtype).contiguous()
    else:
        a = p + "self_attn."
        D = cfg.head_dim
        q0, q1 = rank * d.q_heads, (rank + 1) * d.q_heads
        k0, k1 = d.kv_head_offset, d.kv_head_offset + d.kv_heads
        q = get(a + "q_proj.weight")[q0 * 2 * D:q1 * 2 * D]
        k = get(a + "k_proj.weight")[k0 * D:k1 * D]
        v = get(a + "v_proj.weight")[k0 * D:k1 * D]
        out["qkv_proj"] = torch.cat([q, k, v], 0).to(dtype).contiguous()
        out["q_norm"] = get(a + "q_norm.weight").float().contiguous()
        out["k_norm"] = get(a + "k_norm.weight").float().contiguous()
        out["o_proj"] = get(a + "o_proj.weight")[:, q0 * D:q1 * D].to(dtype).contiguous()
    m = p + "mlp."
    if cfg.is_moe:
        e0, e1 = d.expert_offset, d.expert_offset + d.experts
        out["router"] = get(m + "gate.weight").to(dtype).contiguous()
        if experts is not None:
            out["experts_gate_up"], out["experts_down"] = experts
        else:
            gu = get(m + "experts.gate_up_proj")[e0:e1]
            # intermediate columns held: all of them (expert parallel) or this
            # rank's slice of every expert (tensor parallel within the expert)
            I, Il = cfg.moe_inter, d.moe_inter
            c0 = rank * Il if d.moe_sharding == "tp" else 0
            out["experts_gate_up"] = torch.stack(
                [interleave_gate_up(gu[e, c0:c0 + Il], gu[e, I + c0:I + c0 + Il]) for e in range(gu.shape[0])]
            ).to(dtype).contiguous()
            out["experts_down"] = get(m + "experts.down_proj")[e0:e1, :, c0:c0 + Il].to(dtype).contiguous()
        # shared expert: tensor-parallel (colwise gate/up, rowwise down); each rank
        # scales its partial by the replicated sigmoid gate, so the EP/TP sum
        # reconstructs gate * shared(x) without a redundant copy per rank
        Is = cfg.shared_inter // tp
        s0, s1 = rank * Is, (rank + 1) * Is
        out["shared_gate_up"] = interleave_gate_up(get(m + "shared_expert.gate_proj.weight")[s0:s1],
                                                   get(m + "shared_expert.up_proj.weight")[s0:s1]).to(dtype).contiguous()
        out["shared_down"] = get(m + "shared_expert.down_proj.weight")[:, s0:s1].to(dtype).contiguous()
        out["shared_gate"] = get(m + "shared_expert_gate.weight").to(dtype).contiguous()
    else:
        I0, I1 = rank * d.intermediate, (rank + 1) * d.intermediate
        g = get(m + "gate_proj.weight")[I0:I1]
        u = get(m + "up_proj.weight")[I0:I1]
        out["gate_up"] = interleave_gate_up(g, u).to(dtype).contiguous()
        out["down"] = get(m + "down_proj.weight")[:, I0:I1].to(dtype).contiguous()
    return out


def fuse_globals(cfg: Qwen36Config, get: Callable[[str], torch.Tensor], tp: int, rank: int,
                 dtype=torch.bfloat16) -> dict[str, torch.Tensor]:
    d = tp_dims(cfg, tp, rank)
    emb = get("embed_tokens.weight")
    head = emb if cfg.tie_embeddings else get("lm_head.weight")
    return {
        "embed": emb.to(dtype).contiguous(),  # replicated: no all-reduce on the embed path
        "lm_head": head[d.vocab_offset:d.vocab_offset + d.vocab].to(dtype).contiguous(),
        "final_norm": get("norm.weight").float().contiguous(),
    }


def hf_getter(state: dict[str, torch.Tensor]) -> Callable[[str], torch.Tensor]:
    """Name lookup over an HF state dict that tolerates the known prefixes."""

    def get(name: str) -> torch.Tensor:
        if name == "lm_head.weight":
            for k in ("lm_head.weight", "language_model.lm_head.weight"):
                if k in state:
                    return state[k]
        for pre in HF_PREFIXES:
            if pre + name in state:
                return state[pre + name]
        raise KeyError(name)

    return get


def init_std_check(cfg: Qwen36Config) -> float:
    return 1.0 / math.sqrt(cfg.hidden)
