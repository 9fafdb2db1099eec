"""DeepSeek V4 Flash checkpoint preprocessing: FP4 / FP8 -> bwn formats, TP/EP shards.

The released checkpoint mixes FP4 experts (E2M1 nibbles packed two per byte,
one E8M0 power-of-two scale per 32 inputs) with FP8 dense weights (E4M3FN,
one E8M0 scale per 128x128 block, key ``<name>.scale``).  The reference
dequantizes everything to bf16 and writes per-rank files
(``contrib/deepseek-v4-flash/preprocess_weights.py:24-121``).  Here:

* :func:`decode_fp4_e2m1` / :func:`decode_e8m0` decode from the bit layouts
  (E2M1: sign, 2 exponent bits with bias 1, 1 mantissa bit; E8M0: ``2^(b-127)``);
* FP8 dense weights stay FP8 for the W8A16 kernels (the E8M0 block scales become
  the fp32 ``weight_scale_inv`` those kernels read) or are dequantized to bf16;
* FP4 experts are dequantized and, in ``fp8`` mode, re-quantized onto the
  128x128 E4M3 grid;
* :func:`shard_for_rank` applies the reference's TP/EP split: experts by index
  (EP), ``wq_b`` by output rows, ``wo_b`` by input columns, the rest replicated.
"""
from __future__ import annotations

import os

import torch

from .fp8 import decode_e4m3fn, expand_block_scales, quantize_block
from .safetensors import SafeReader, save_file, weight_map

FP4_BLOCK = 32
FP8_BLOCK = 128


def decode_fp4_e2m1(codes: torch.Tensor) -> torch.Tensor:
    """4-bit E2M1 codes (0..15) -> float32."""
    c = codes.to(torch.int32)
    e = (c >> 1) & 3
    m = (c & 1).float()
    mag = torch.where(e == 0, m * 0.5, (1.0 + m * 0.5) * torch.exp2((e - 1).float()))
    return torch.where((c & 8) != 0, -mag, mag)


def decode_e8m0(raw: torch.Tensor) -> torch.Tensor:
    b = raw.contiguous().view(torch.uint8).to(torch.int32)
    v = torch.exp2((b - 127).float())
    return torch.where(b == 255, torch.full_like(v, float("nan")), v)


def _scales(t: torch.Tensor, tag: str) -> torch.Tensor:
    return decode_e8m0(t) if tag in ("F8_E8M0", "U8") else t.float()


def dequant_fp4(packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """``packed [out, in/2]`` (low nibble first) x ``scales [out, in/32]`` -> fp32 ``[out, in]``."""
    b = packed.contiguous().view(torch.uint8)
    out_f, half = b.shape
    v = torch.stack([decode_fp4_e2m1(b & 0xF), decode_fp4_e2m1(b >> 4)], -1).reshape(out_f, 2 * half)
    s = scales.float().repeat_interleave(FP4_BLOCK, 1)[:, : 2 * half]
    return v * s


def dequant_fp8(w8: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    v = decode_e4m3fn(w8, reject_nan=False)
    return v * expand_block_scales(scales.float(), v.shape, FP8_BLOCK)


def convert_tensor(reader: SafeReader, key: str, mode: str) -> dict[str, torch.Tensor]:
    """One checkpoint weight in bwn form: ``mode`` ``"bf16"`` -> ``{key: bf16}``;
    ``"fp8"`` -> ``{key: e4m3 bytes, key_scale_inv: fp32 [N/128, K/128]}`` for
    quantized weights (dense bf16 weights pass through)."""
    tag = reader.dtype_tag(key)
    sk = key[: -len(".weight")] + ".scale" if key.endswith(".weight") else None
    has_scale = sk is not None and sk in reader
    w = reader.get(key)
    if not has_scale or tag in ("BF16", "F16", "F32"):
        return {key: w if not w.is_floating_point() else w.to(torch.bfloat16 if w.dim() >= 2 else w.dtype)}
    s = _scales(reader.get(sk), reader.dtype_tag(sk))
    if tag == "F8_E4M3":
        if mode == "fp8":
            return {key: w.clone(), key + "_scale_inv": s.contiguous()}
        return {key: dequant_fp8(w, s).to(torch.bfloat16)}
    # FP4 packed in int8/uint8
    dense = dequant_fp4(w, s)
    if mode == "fp8":
        w8, s8 = quantize_block(dense)
        return {key: w8, key + "_scale_inv": s8}
    return {key: dense.to(torch.bfloat16)}


def shard_for_rank(key: str, t: torch.Tensor, rank: int, tp: int, cfg: dict):
    """``(new_key, tensor)`` of this rank, or ``None`` when another rank owns it."""
    n_exp = cfg["n_routed_experts"]
    if ".experts." in key and ".shared_experts." not in key:
        parts = key.split(".")
        i = parts.index("experts")
        if i + 1 < len(parts) and parts[i + 1].isdigit():
            per = n_exp // tp
            e = int(parts[i + 1])
            if e // per != rank:
                return None
            parts[i + 1] = str(e % per)
            return ".".join(parts), t
        return key, t
    if key.endswith(".wq_b.weight") or key.endswith(".wq_b.weight_scale_inv"):
        c = t.shape[0] // tp
        return key, t[rank * c:(rank + 1) * c].contiguous()
    if key.endswith(".wo_b.weight") or key.endswith(".wo_b.weight_scale_inv"):
        c = t.shape[1] // tp
        return key, t[:, rank * c:(rank + 1) * c].contiguous()
    return key, t


def preprocess(in_dir: str, out_dir: str, tp: int, mode: str = "fp8", cfg: dict | None = None):
    """Convert a DeepSeek V4 checkpoint and write ``rank{r}.safetensors`` per TP rank."""
    import json
    if cfg is None:
        with open(os.path.join(in_dir, "config.json")) as f:
            cfg = json.load(f)
    wm = weight_map(in_dir)
    readers = {fn: SafeReader(os.path.join(in_dir, fn)) for fn in sorted(set(wm.values()))}
    per_rank: list[dict[str, torch.Tensor]] = [{} for _ in range(tp)]
    tags: list[dict[str, str]] = [{} for _ in range(tp)]
    for key, fn in sorted(wm.items()):
        if key.endswith(".scale") and key[: -len(".scale")] + ".weight" in wm:
            continue
        for k, t in convert_tensor(readers[fn], key, mode).items():
            for r in range(tp):
                got = shard_for_rank(k, t, r, tp, cfg)
                if got is not None:
                    per_rank[r][got[0]] = got[1]
                    if t.dtype == torch.uint8 and k.endswith(".weight") and mode == "fp8":
                        tags[r][got[0]] = "F8_E4M3"
    os.makedirs(out_dir, exist_ok=True)
    for r in range(tp):
        save_file(per_rank[r], os.path.join(out_dir, f"rank{r}.safetensors"),
                  metadata={"tp": tp, "rank": r, "mode": mode}, dtype_tags=tags[r])
    for rd in readers.values():
        rd.close()
    return per_rank


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--input-path", required=True)
    ap.add_argument("--output-path", required=True)
    ap.add_argument("--tp", type=int, default=8)
    ap.add_argument("--mode", choices=("fp8", "bf16"), default="fp8")
    a = ap.parse_args()
    preprocess(a.input_path, a.output_path, a.tp, a.mode)
