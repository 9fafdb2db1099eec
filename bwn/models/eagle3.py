"""EAGLE3 draft model for speculative decoding of Qwen3.6 targets.

The reference serves EAGLE3 through an external vLLM fork (3 speculative
tokens, ``contrib/qwen3.6-27b/deploy/eagle3_config.yaml:7-10``); the draft
itself is not in its tree.  This is the EAGLE3 draft structure:

* feature fusion: ``fc`` maps the target's residual stream at three layers
  (low / middle / high, ``(2, L/2, L-3)``) ``[3H] -> [H]``;
* one decoder layer whose attention input is ``[norm(embed(next token)),
  norm(hidden)]`` (``2H`` wide), residual = the fused hidden;
* a reduced draft vocabulary with ``d2t`` offsets to target ids.

The attention block is the target's own gated-GQA block (q/k RMSNorm(1+w),
partial RoPE, sigmoid output gate) so the draft runs on the same fused
decode / multi-token / prefill attention kernels as the target.  The draft is
replicated on every tensor-parallel rank (it is one layer).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops as O
from ..config import Qwen36Config
from ..io.qwen36_weights import seeded_tensor
from ..ops import reference as R


@dataclass(frozen=True)
class Eagle3Config:
    hidden: int
    target_vocab: int
    draft_vocab: int
    q_heads: int
    kv_heads: int
    head_dim: int
    rope_dim: int
    rope_theta: float
    intermediate: int
    rms_eps: float
    feat_layers: tuple[int, int, int]


def eagle3_config(t: Qwen36Config, draft_vocab: int = 32000) -> Eagle3Config:
    L = t.num_layers
    return Eagle3Config(
        hidden=t.hidden, target_vocab=t.vocab, draft_vocab=min(draft_vocab, t.vocab), q_heads=t.q_heads,
        kv_heads=t.kv_heads, head_dim=t.head_dim, rope_dim=t.rope_dim, rope_theta=t.rope_theta,
        intermediate=t.intermediate if t.intermediate else 3 * t.hidden, rms_eps=t.rms_eps,
        feat_layers=(min(2, L - 1), L // 2, max(L - 3, 0)))


class DraftState:
    def __init__(self, cfg: Eagle3Config, batch: int, max_seq: int, device, dtype):
        self.k_cache = torch.zeros(batch, cfg.kv_heads, max_seq, cfg.head_dim, dtype=dtype, device=device)
        self.v_cache = torch.zeros_like(self.k_cache)


def synthetic_eagle3(cfg: Eagle3Config, seed: int, device="cpu") -> dict[str, torch.Tensor]:
    """Random-init weights in the HF EAGLE3 naming (query||gate q_proj rows)."""
    H, D, I = cfg.hidden, cfg.head_dim, cfg.intermediate
    sd = {}

    def t(name, shape, kind="normal", std=0.02, dtype=torch.bfloat16):
        sd[name] = seeded_tensor("eagle3." + name, shape, seed, device, kind, std, dtype)

    t("fc.weight", (H, 3 * H))
    m = "midlayer."
    for n in ("input_layernorm", "hidden_norm", "post_attention_layernorm"):
        t(m + n + ".weight", (H,), "zeros", dtype=torch.float32)
    t(m + "self_attn.q_proj.weight", (cfg.q_heads * 2 * D, 2 * H))
    t(m + "self_attn.k_proj.weight", (cfg.kv_heads * D, 2 * H))
    t(m + "self_attn.v_proj.weight", (cfg.kv_heads * D, 2 * H))
    t(m + "self_attn.o_proj.weight", (H, cfg.q_heads * D))
    t(m + "self_attn.q_norm.weight", (D,), "zeros", dtype=torch.float32)
    t(m + "self_attn.k_norm.weight", (D,), "zeros", dtype=torch.float32)
    t(m + "mlp.gate_proj.weight", (I, H))
    t(m + "mlp.up_proj.weight", (I, H))
    t(m + "mlp.down_proj.weight", (H, I))
    t("norm.weight", (H,), "zeros", dtype=torch.float32)
    t("lm_head.weight", (cfg.draft_vocab, H))
    sd["d2t"] = torch.zeros(cfg.draft_vocab, dtype=torch.int64, device=device)
    return sd


class Eagle3Draft:
    def __init__(self, cfg: Eagle3Config, device="cpu", dtype=torch.bfloat16):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.w: dict[str, torch.Tensor] = {}
        self.cos, self.sin = R.rope_table(1, cfg.rope_dim, cfg.rope_theta, device=self.device)

    def load(self, sd: dict[str, torch.Tensor]) -> "Eagle3Draft":
        dt, dev = self.dtype, self.device
        m = "midlayer."
        a = m + "self_attn."
        w = {
            "fc": sd["fc.weight"].to(dt),
            "in_norm": sd[m + "input_layernorm.weight"].float(),
            "hid_norm": sd[m + "hidden_norm.weight"].float(),
            "post_norm": sd[m + "post_attention_layernorm.weight"].float(),
            "qkv": torch.cat([sd[a + "q_proj.weight"], sd[a + "k_proj.weight"], sd[a + "v_proj.weight"]], 0).to(dt),
            "o_proj": sd[a + "o_proj.weight"].to(dt),
            "q_norm": sd[a + "q_norm.weight"].float(),
            "k_norm": sd[a + "k_norm.weight"].float(),
            "gate_up": O.interleave_gate_up(sd[m + "mlp.gate_proj.weight"], sd[m + "mlp.up_proj.weight"]).to(dt),
            "down": sd[m + "mlp.down_proj.weight"].to(dt),
            "norm": sd["norm.weight"].float(),
            "lm_head": sd["lm_head.weight"].to(dt),
            "d2t": sd["d2t"].long(),
        }
        self.w = {k: v.to(dev).contiguous() for k, v in w.items()}
        return self

    def init_random(self, seed: int = 0) -> "Eagle3Draft":
        return self.load(synthetic_eagle3(self.cfg, seed, "cpu"))

    def new_state(self, batch: int, max_seq: int) -> DraftState:
        if self.cos.shape[0] < max_seq:
            self.cos, self.sin = R.rope_table(max_seq, self.cfg.rope_dim, self.cfg.rope_theta, device=self.device)
        return DraftState(self.cfg, batch, max_seq, self.device, self.dtype)

    # ------------------------------------------------------------------ layer
    def fuse(self, feats: list[torch.Tensor]) -> torch.Tensor:
        """Target features ``3 x [R, H]`` -> fused hidden ``[R, H]``."""
        return O.linear(torch.cat(feats, dim=-1), self.w["fc"])

    def _layer(self, hid: torch.Tensor, tokens: torch.Tensor, attend):
        """One draft layer over rows; returns ``(pre-norm hidden [R, H], ids [R])``."""
        cfg, w = self.cfg, self.w
        e = O.embedding(tokens.reshape(-1).int(), self._embed, 0)
        xin = torch.cat([O.rms_norm(e, w["in_norm"], cfg.rms_eps), O.rms_norm(hid, w["hid_norm"], cfg.rms_eps)], -1)
        R_ = xin.shape[0]
        D, QH, KVH = cfg.head_dim, cfg.q_heads, cfg.kv_heads
        proj = O.linear(xin, w["qkv"])
        qg = proj[:, :QH * 2 * D].view(R_, QH, 2 * D)
        k = proj[:, QH * 2 * D:QH * 2 * D + KVH * D].view(R_, KVH, D)
        v = proj[:, QH * 2 * D + KVH * D:].view(R_, KVH, D)
        o = attend(qg, k, v)
        r = hid.clone()
        h2 = O.add_rms_norm(O.linear(o, w["o_proj"]), r, w["post_norm"], cfg.rms_eps)
        hn = O.add_rms_norm(O.linear(O.linear_swiglu(h2, w["gate_up"]), w["down"]), r, w["norm"], cfg.rms_eps)
        logits = O.linear(hn, w["lm_head"])
        ids = O.unpack_argmax(O.argmax_packed(logits, 0))
        return r, (ids.long() + w["d2t"][ids.long()]).int()

    def bind_embedding(self, table: torch.Tensor) -> None:
        """EAGLE3 drafts share the target's token embedding."""
        self._embed = table

    def prefill(self, hid: torch.Tensor, tokens_next: torch.Tensor, st: DraftState):
        """Rows of a prompt from position 0: ``hid [B*S, H]`` fused target
        features, ``tokens_next [B, S]`` the token after each position."""
        B, S = tokens_next.shape
        cfg = self.cfg

        def attend(qg, k, v):
            return O.gqa_prefill(qg.view(B, S, cfg.q_heads, -1), k.view(B, S, cfg.kv_heads, -1),
                                 v.view(B, S, cfg.kv_heads, -1), self.w["q_norm"], self.w["k_norm"], self.cos,
                                 self.sin, st.k_cache, st.v_cache, 0, cfg.rms_eps).reshape(B * S, -1)

        return self._layer(hid, tokens_next, attend)

    def rows(self, hid: torch.Tensor, tokens: torch.Tensor, positions: torch.Tensor, st: DraftState, n_tok: int = 1):
        """``n_tok`` consecutive rows per sequence at ``positions`` (one per row)."""
        cfg = self.cfg

        def attend(qg, k, v):
            return O.gqa_decode(qg, k, v, self.w["q_norm"], self.w["k_norm"], self.cos, self.sin, st.k_cache,
                                st.v_cache, positions, cfg.rms_eps, 0, n_tok)

        return self._layer(hid, tokens, attend)

    def weight_bytes(self) -> int:
        return sum(v.numel() * v.element_size() for v in self.w.values())
