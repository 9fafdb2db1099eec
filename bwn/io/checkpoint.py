"""Checkpoint directories: HF safetensors layouts for every bwn model.

:class:`Checkpoint` maps a directory (single file, sharded with an index, or a
bare set of shards) and serves tensors by their model-relative name:

* the language-model prefix is detected from where
  ``layers.0.input_layernorm.weight`` sits (``model.``,
  ``model.language_model.``, nested tiny-random prefixes), as the reference
  does (``contrib/qwen3.6-35b-a3b/static_decode_35b.py:2722-2740``);
* official FP8 weights (``F8_E4M3`` + ``<name>_scale_inv``, 128x128 blocks)
  come back as :class:`bwn.io.fp8.FP8Weight` on request, or dequantized;
* MoE experts are served stacked (``experts.gate_up_proj [E, 2I, H]``,
  ``experts.down_proj [E, H, I]``) whether the file stores them packed or
  per expert (``experts.{e}.{gate,up,down}_proj.weight``,
  ``static_decode_35b.py:2746, 2824-2843``).
"""
from __future__ import annotations

import json
import os

import torch

from .fp8 import FP8Weight, dequantize_block
from .safetensors import SafeReader, weight_map

_ANCHOR = "layers.0.input_layernorm.weight"


class Checkpoint:
    def __init__(self, path: str, prefix: str | None = None):
        self.dir = path if os.path.isdir(path) else os.path.dirname(os.path.abspath(path))
        if os.path.isfile(path):
            r = SafeReader(path)
            self.wm = {k: os.path.basename(path) for k in r.keys()}
            r.close()
        else:
            self.wm = weight_map(path)
        self._readers: dict[str, SafeReader] = {}
        if prefix is None:
            anchors = [k for k in self.wm if k.endswith(_ANCHOR)]
            prefix = anchors[0][: -len(_ANCHOR)] if anchors else ""
        self.prefix = prefix

    # ----------------------------------------------------------------- raw
    def _reader(self, key: str) -> SafeReader:
        fn = self.wm[key]
        r = self._readers.get(fn)
        if r is None:
            r = self._readers[fn] = SafeReader(os.path.join(self.dir, fn))
        return r

    def raw(self, key: str) -> torch.Tensor:
        return self._reader(key).get(key)

    def tag(self, key: str) -> str:
        return self._reader(key).dtype_tag(key)

    def config(self) -> dict:
        with open(os.path.join(self.dir, "config.json")) as f:
            return json.load(f)

    def close(self):
        for r in self._readers.values():
            r.close()
        self._readers.clear()

    # -------------------------------------------------------------- by name
    def resolve(self, name: str) -> str:
        """Full key of a model-relative name (``lm_head.weight`` is looked up
        at the top level too, where HF multimodal checkpoints keep it)."""
        for k in (self.prefix + name, name, "model." + name, "language_model." + name,
                  "model.language_model." + name):
            if k in self.wm:
                return k
        if name == "lm_head.weight":
            for k in self.wm:
                if k.endswith("lm_head.weight"):
                    return k
        raise KeyError(name)

    def has(self, name: str) -> bool:
        try:
            self.resolve(name)
            return True
        except KeyError:
            return False

    def get(self, name: str, fp8: str = "dequant"):
        """Tensor ``name``. An official FP8 weight (``F8_E4M3`` with a
        ``_scale_inv`` sibling) is returned per ``fp8``: ``"dequant"`` -> bf16,
        ``"keep"`` -> :class:`FP8Weight` (bytes + fp32 block scales)."""
        key = self.resolve(name)
        t = self.raw(key)
        if self.tag(key) == "F8_E4M3":
            sk = key + "_scale_inv"
            if sk not in self.wm:
                raise KeyError(f"{key} is FP8 but has no {sk}")
            scales = self.raw(sk).float()
            if fp8 == "keep":
                return FP8Weight(t.clone(), scales)
            return dequantize_block(t, scales).to(torch.bfloat16)
        return t

    def experts(self, layer_prefix: str, n_experts: int, e0: int = 0, e1: int | None = None):
        """``(gate_up [E, 2I, H], down [E, H, I])`` of experts ``[e0, e1)`` under
        ``layer_prefix + "mlp."`` from the packed or per-expert layout (FP8 per-expert
        weights are dequantized)."""
        e1 = n_experts if e1 is None else e1
        m = layer_prefix + "mlp.experts."
        if self.has(m + "gate_up_proj"):
            return self.get(m + "gate_up_proj")[e0:e1], self.get(m + "down_proj")[e0:e1]
        gus, dns = [], []
        for e in range(e0, e1):
            p = f"{m}{e}."
            gus.append(torch.cat([self.get(p + "gate_proj.weight"), self.get(p + "up_proj.weight")], 0))
            dns.append(self.get(p + "down_proj.weight"))
        return torch.stack(gus), torch.stack(dns)

    def fp8_experts(self, layer_prefix: str, e0: int, e1: int, c0: int = 0, width: int | None = None):
        """Official FP8 per-expert weights of experts ``[e0, e1)`` kept in fp8:
        ``(gate_up, down)`` as :class:`~bwn.io.fp8.FP8Experts` (gate/up rows
        interleaved in 16s with their own 128x128 block scales), no dequantize /
        requantize round trip.  ``c0`` / ``width`` select a slice of every
        expert's intermediate width (tensor parallelism within experts); a
        slice must not straddle two 128-column scale blocks of ``down``."""
        from .fp8 import FP8Experts, _scales16
        m = layer_prefix + "mlp.experts."
        g8s, u8s, g16, u16, d8s, d16 = [], [], [], [], [], []
        for e in range(e0, e1):
            p = f"{m}{e}."
            parts = []
            for name in ("gate_proj", "up_proj", "down_proj"):
                key = self.resolve(p + name + ".weight")
                if self.tag(key) != "F8_E4M3":
                    raise ValueError(f"{key} is not an FP8 weight")
                parts.append((self.raw(key), self.raw(key + "_scale_inv").float()))
            (g, gs), (u, us), (d, ds) = parts
            I = g.shape[0]
            w = I if width is None else width
            if c0 % 16 or w % 16 or c0 + w > I:
                raise ValueError(f"intermediate slice [{c0}, {c0 + w}) of {I} must follow 16-row groups")
            if width is not None and c0 % 128 and (c0 % 128) + w > 128:
                raise ValueError("the slice straddles two 128-column scale blocks of down_proj")
            g8s.append(g[c0:c0 + w])
            u8s.append(u[c0:c0 + w])
            g16.append(_scales16(gs, I)[c0 // 16:(c0 + w) // 16])
            u16.append(_scales16(us, I)[c0 // 16:(c0 + w) // 16])
            d8s.append(d[:, c0:c0 + w])
            k0 = c0 // 128
            d16.append(_scales16(ds, d.shape[0])[:, k0:k0 + -(-w // 128)])
        E, H = len(g8s), g8s[0].shape[1]
        w = g8s[0].shape[0]
        w8 = torch.stack([torch.stack(g8s).reshape(E, w // 16, 16, H), torch.stack(u8s).reshape(E, w // 16, 16, H)],
                         dim=2).reshape(E, 2 * w, H)
        s16 = torch.stack([torch.stack(g16), torch.stack(u16)], dim=2).reshape(E, 2 * w // 16, -1)
        return FP8Experts(w8.contiguous(), s16), FP8Experts(torch.stack(d8s).contiguous(), torch.stack(d16))

    def getter(self):
        """``get(name)`` callable for the model loaders (stacked expert names are
        synthesised from per-expert layouts on demand)."""
        cache: dict[str, torch.Tensor] = {}

        def get(name: str) -> torch.Tensor:
            if self.has(name):
                return self.get(name)
            for suffix, idx in ((".mlp.experts.gate_up_proj", 0), (".mlp.experts.down_proj", 1)):
                if name.endswith(suffix):
                    lp = name[: -len(suffix)] + "."
                    if name not in cache:
                        n = 0
                        while self.has(f"{lp}mlp.experts.{n}.down_proj.weight"):
                            n += 1
                        if n == 0:
                            raise KeyError(name)
                        gu, dn = self.experts(lp, n)
                        cache.clear()
                        cache[lp + "mlp.experts.gate_up_proj"] = gu
                        cache[lp + "mlp.experts.down_proj"] = dn
                    return cache[name]
            raise KeyError(name)

        return get
