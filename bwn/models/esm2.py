"""ESM-2 protein language model (HF ``EsmForMaskedLM`` layout and numerics).

The reference fine-tunes the HF model directly (``contrib/esm2/train_esm.py``,
``run_esm.py``): pre-LN transformer, rotary q/k, erf-GELU FFN, token-dropout
embedding scaling, LM head ``dense -> gelu -> LayerNorm -> decoder(tied) + bias``.
This module re-implements that forward with parameter names matching the HF
state dict, so HF checkpoints load as-is, and routes every Linear through the
tcgen05 GEMMs with their backward (``dX = dY W`` on the MN-major-B kernel,
``dW = dY^T X`` on the MN-major-A/B kernel, fp32 weight gradients) for bf16
training with fp32 master weights.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops as O
from ..config import ESM2Config


def _gemm_ok(*dims: int) -> bool:
    return all(d % 8 == 0 for d in dims)


class _BwnLinearFn(torch.autograd.Function):
    """y = x W^T (+ b) with bf16 tcgen05 GEMMs in both directions."""

    @staticmethod
    def forward(ctx, x2d, w, b, wb=None):
        xb = x2d.to(torch.bfloat16).contiguous()
        if wb is None:
            wb = w.to(torch.bfloat16).contiguous()
        y = O.linear(xb, wb) if b is None else O.linear_bias(xb, wb, b)
        ctx.save_for_backward(xb, wb)
        ctx.has_b = b is not None
        ctx.w_dtype = w.dtype
        return y

    @staticmethod
    def backward(ctx, gy):
        xb, wb = ctx.saved_tensors
        gyb = gy.to(torch.bfloat16).contiguous()
        gx = gw = gb = None
        if ctx.needs_input_grad[0]:
            gx = O.linear_kn(gyb, wb)
        if ctx.needs_input_grad[1]:
            rows = gyb.shape[0]
            if rows % 8:  # dW contracts over tokens: zero rows keep the TMA 16-byte rule and the sum
                pad = 8 - rows % 8
                gyb = torch.nn.functional.pad(gyb, (0, 0, 0, pad))
                xb = torch.nn.functional.pad(xb, (0, 0, 0, pad))
            gw = O.matmul_tn(gyb, xb, f32_out=True).to(ctx.w_dtype)
        if ctx.has_b and ctx.needs_input_grad[2]:
            gb = gy.float().sum(0).to(ctx.w_dtype)
        return gx, gw, gb, None


class BwnLinear(nn.Linear):
    """``nn.Linear`` whose CUDA forward/backward run on the bwn GEMM kernels."""

    def _bf16_weight(self) -> torch.Tensor:
        """bf16 copy of the (fp32 master) weight, re-made only when the weight
        changed (optimizer step, load), so a step's forward and recompute share it."""
        w = self.weight
        if w.dtype == torch.bfloat16:
            return w
        key = (w.data_ptr(), w._version, w.shape)
        c = self.__dict__.get("_wb")
        if c is None or c[0] != key:
            c = (key, w.detach().to(torch.bfloat16).contiguous())
            self.__dict__["_wb"] = c
        return c[1]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.is_cuda and _gemm_ok(self.in_features, self.out_features) and x.numel() > 0:
            shp = x.shape
            y = _BwnLinearFn.apply(x.reshape(-1, shp[-1]), self.weight, self.bias, self._bf16_weight())
            return y.reshape(*shp[:-1], self.out_features)  # bf16: consumers read it as is (no widening copy)
        return F.linear(x.to(self.weight.dtype), self.weight, self.bias)


def esm_gelu(x: torch.Tensor) -> torch.Tensor:
    """erf GELU as in the original ESM code (HF ``esm.modeling_esm.gelu``:
    ``x * 0.5 * (1 + erf(x / sqrt(2)))``), as one fused elementwise op forward
    and backward instead of five."""
    return F.gelu(x, approximate="none")


def _rotate_half(x):
    a, b = x.chunk(2, dim=-1)
    return torch.cat((-b, a), dim=-1)


class _RopeHeadsFn(torch.autograd.Function):
    """``x [B*S, H*D]`` (a projection's output) -> rotary-embedded, scaled
    ``[B, H, S, D]`` in one kernel; its backward is the transposed rotation back
    into the projection layout (``csrc/kernels/esm.cu``)."""

    @staticmethod
    def forward(ctx, x2d, cos, sin, B, S, H, scale):
        ctx.save_for_backward(cos, sin)
        ctx.dims = (B, S, H, scale)
        return O.rope_half(x2d, cos, sin, B, S, H, True, 1.0, scale)

    @staticmethod
    def backward(ctx, g):
        cos, sin = ctx.saved_tensors
        B, S, H, scale = ctx.dims
        gx = O.rope_half(g.contiguous(), cos, sin, B, S, H, False, -1.0, scale)
        return gx, None, None, None, None, None, None


class EsmSelfAttention(nn.Module):
    def __init__(self, cfg: ESM2Config):
        super().__init__()
        H = cfg.hidden
        self.heads = cfg.heads
        self.hd = cfg.head_dim
        self.query = BwnLinear(H, H)
        self.key = BwnLinear(H, H)
        self.value = BwnLinear(H, H)
        inv = 1.0 / (10000 ** (torch.arange(0, self.hd, 2).float() / self.hd))
        self.register_buffer("inv_freq", inv, persistent=False)

    def _tables(self, S: int, device) -> tuple[torch.Tensor, torch.Tensor]:
        """fp32 ``cos``/``sin`` ``[S, D/2]`` of the rotary angles (cached per length)."""
        key = (S, str(device))
        cache = self.__dict__.setdefault("_rope_cache", {})
        if key not in cache:
            f = torch.outer(torch.arange(S, device=device, dtype=torch.float32), self.inv_freq.float().to(device))
            cache.clear()
            cache[key] = (f.cos().contiguous(), f.sin().contiguous())
        return cache[key]

    def forward(self, x, attn_bias):
        B, S, _ = x.shape
        if x.is_cuda and self.hd % 4 == 0:
            # projections stay bf16; RoPE + q scaling + head-major layout in one kernel each
            ql, kl, vl = self.query(x), self.key(x), self.value(x)
            H = ql.shape[-1] // self.hd
            cos, sin = self._tables(S, x.device)
            q = _RopeHeadsFn.apply(ql.reshape(B * S, -1).to(torch.bfloat16), cos, sin, B, S, H, self.hd ** -0.5)
            k = _RopeHeadsFn.apply(kl.reshape(B * S, -1).to(torch.bfloat16), cos, sin, B, S, H, 1.0)
            v = vl.to(torch.bfloat16).view(B, S, H, self.hd).transpose(1, 2)
            o = F.scaled_dot_product_attention(q, k, v, attn_mask=attn_bias.to(torch.bfloat16), scale=1.0)
            return o.transpose(1, 2).reshape(B, S, -1)
        q = self.query(x).view(B, S, -1, self.hd).transpose(1, 2)
        k = self.key(x).view(B, S, -1, self.hd).transpose(1, 2)
        v = self.value(x).view(B, S, -1, self.hd).transpose(1, 2)
        q = q * self.hd ** -0.5
        t = torch.arange(S, device=x.device, dtype=self.inv_freq.dtype)
        f = torch.outer(t, self.inv_freq)
        emb = torch.cat([f, f], -1)
        cos, sin = emb.cos().to(q.dtype), emb.sin().to(q.dtype)
        q = q * cos + _rotate_half(q) * sin
        k = k * cos + _rotate_half(k) * sin
        out_dtype = v.dtype
        if x.is_cuda:  # bf16 attention (flash path) on the GPU, like the bf16 GEMMs
            q, k, v = q.bfloat16(), k.bfloat16(), v.bfloat16()
        else:
            q, k = q.to(v.dtype), k.to(v.dtype)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=attn_bias.to(v.dtype), scale=1.0)
        return o.transpose(1, 2).reshape(B, S, -1).to(out_dtype)


class EsmLayer(nn.Module):
    def __init__(self, cfg: ESM2Config):
        super().__init__()
        H = cfg.hidden
        self.attention = nn.Module()
        self.attention.self = EsmSelfAttention(cfg)
        self.attention.output = nn.Module()
        self.attention.output.dense = BwnLinear(H, H)
        self.attention.LayerNorm = nn.LayerNorm(H, eps=cfg.layer_norm_eps)
        self.intermediate = nn.Module()
        self.intermediate.dense = BwnLinear(H, cfg.ffn)
        self.output = nn.Module()
        self.output.dense = BwnLinear(cfg.ffn, H)
        self.LayerNorm = nn.LayerNorm(H, eps=cfg.layer_norm_eps)

    def forward(self, x, attn_bias):
        a = self.attention
        hn = a.LayerNorm(x)
        h = a.self(hn.to(torch.bfloat16) if hn.is_cuda else hn, attn_bias)  # one cast for q, k and v
        x = x + a.output.dense(h)
        h = esm_gelu(self.intermediate.dense(self.LayerNorm(x)))
        return x + self.output.dense(h)


class EsmForMaskedLM(nn.Module):
    """HF-compatible parameter names: ``esm.embeddings.word_embeddings.weight``,
    ``esm.encoder.layer.{i}...``, ``esm.encoder.emb_layer_norm_after``,
    ``lm_head.{dense,layer_norm,decoder,bias}`` (decoder tied to embeddings)."""

    def __init__(self, cfg: ESM2Config):
        super().__init__()
        self.cfg = cfg
        H, V = cfg.hidden, cfg.vocab
        self.esm = nn.Module()
        self.esm.embeddings = nn.Module()
        self.esm.embeddings.word_embeddings = nn.Embedding(V, H, padding_idx=cfg.pad_token_id)
        self.esm.encoder = nn.Module()
        self.esm.encoder.layer = nn.ModuleList([EsmLayer(cfg) for _ in range(cfg.num_layers)])
        self.esm.encoder.emb_layer_norm_after = nn.LayerNorm(H, eps=cfg.layer_norm_eps)
        self.lm_head = nn.Module()
        self.lm_head.dense = BwnLinear(H, H)
        self.lm_head.layer_norm = nn.LayerNorm(H, eps=cfg.layer_norm_eps)
        self.lm_head.bias = nn.Parameter(torch.zeros(V))
        self.vocab_pad = ((V + 63) // 64) * 64  # decoder GEMM rows padded for the 16-byte TMA rule

    def init_weights(self, seed: int = 0) -> "EsmForMaskedLM":
        g = torch.Generator().manual_seed(seed)
        for n, p in self.named_parameters():
            with torch.no_grad():
                if p.dim() >= 2:
                    p.copy_(torch.randn(p.shape, generator=g) * 0.02)
                elif "LayerNorm" in n or "layer_norm" in n:
                    p.fill_(1.0 if n.endswith("weight") else 0.0)
                else:
                    p.zero_()
        return self

    def embed(self, input_ids, attention_mask):
        cfg = self.cfg
        x = self.esm.embeddings.word_embeddings(input_ids)
        if cfg.token_dropout:
            is_mask = (input_ids == cfg.mask_token_id)
            x = x.masked_fill(is_mask.unsqueeze(-1), 0.0)
            mask_ratio_train = 0.15 * 0.8
            src_len = attention_mask.sum(-1)
            observed = is_mask.sum(-1).float() / src_len
            x = (x * (1 - mask_ratio_train) / (1 - observed)[:, None, None]).to(x.dtype)
        return (x * attention_mask.unsqueeze(-1)).to(x.dtype)

    def forward(self, input_ids: torch.Tensor, attention_mask: torch.Tensor | None = None,
                compute_dtype=torch.float32) -> torch.Tensor:
        if attention_mask is None:
            attention_mask = torch.ones_like(input_ids)
        x = self.embed(input_ids, attention_mask).to(compute_dtype)
        bias = torch.zeros(attention_mask.shape, dtype=compute_dtype, device=x.device)
        bias = bias.masked_fill(attention_mask == 0, torch.finfo(compute_dtype).min)[:, None, None, :]
        ckpt = getattr(self, "activation_checkpointing", False) and torch.is_grad_enabled()
        for layer in self.esm.encoder.layer:
            if ckpt:  # keep only each layer's input; recompute its activations in backward
                from torch.utils.checkpoint import checkpoint
                x = checkpoint(layer, x, bias, use_reentrant=False)
            else:
                x = layer(x, bias)
        x = self.esm.encoder.emb_layer_norm_after(x)
        h = self.lm_head.layer_norm(esm_gelu(self.lm_head.dense(x)).to(x.dtype))
        w = self.esm.embeddings.word_embeddings.weight
        if h.is_cuda:
            wp = F.pad(w, (0, 0, 0, self.vocab_pad - w.shape[0]))
            logits = BwnLinear.forward_with(h, wp)[..., : w.shape[0]]
        else:
            logits = F.linear(h.to(w.dtype), w)
        return logits + self.lm_head.bias.to(logits.dtype)

    def load_hf_state_dict(self, sd: dict) -> None:
        own = {k: v for k, v in sd.items() if not k.startswith("esm.contact_head") and "position_ids" not in k
               and "rotary_embeddings" not in k and k != "lm_head.decoder.weight"}
        missing, unexpected = self.load_state_dict(own, strict=False)
        bad = [m for m in missing if "inv_freq" not in m]
        if bad or unexpected:
            raise KeyError(f"ESM state dict mismatch: missing={bad} unexpected={unexpected}")


def _forward_with(h: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    shp = h.shape
    y = _BwnLinearFn.apply(h.reshape(-1, shp[-1]), w, None)
    return y.reshape(*shp[:-1], w.shape[0])


BwnLinear.forward_with = staticmethod(_forward_with)


def mlm_loss(logits: torch.Tensor, labels: torch.Tensor, loss_mask: torch.Tensor,
             divisor: str = "tokens") -> torch.Tensor:
    """Masked-LM cross entropy.  ``divisor="tokens"`` divides by every position
    (the reference's static divisor, ``contrib/esm2/train_esm.py:231-245``);
    ``"masked"`` divides by the number of masked positions."""
    lp = F.log_softmax(logits.float().reshape(-1, logits.shape[-1]), dim=-1)
    nll = -lp.gather(1, labels.reshape(-1, 1).long()).squeeze(1)
    m = loss_mask.reshape(-1).float()
    denom = m.numel() if divisor == "tokens" else m.sum().clamp(min=1)
    return (nll * m).sum() / denom
