"""FP8 (E4M3) weight formats and conversions.

* OCP E4M3FN (the ``F8_E4M3`` of official FP8 safetensors): decoded from the bit
  layout (exponent bias 7, finite through 448, only ``S.1111.111`` is NaN) --
  the reference's ``decode_e4m3fn`` (``contrib/qwen3.6-35b-a3b/moe_w8.py:26``).
* Legacy E4M3 (finite-only variant whose exponent 15 is reserved, max 240) with
  round-to-nearest-even encoding, as the reference stores Trn2 weights
  (``encode_legacy_e4m3`` / ``decode_legacy_e4m3``, ``moe_w8.py:73-118``).
* 128x128 block-scaled weights (``weight`` E4M3FN + ``weight_scale_inv``; value
  = fp8 * scale), the layout the bwn W8A16 kernels consume directly:
  :func:`quantize_block`, :func:`dequantize_block`, :func:`expand_block_scales`.
"""
from __future__ import annotations

import math

import torch

BLOCK = 128
E4M3FN_MAX = 448.0
LEGACY_E4M3_MAX = 240.0


def _bytes(raw: torch.Tensor) -> torch.Tensor:
    if raw.element_size() != 1:
        raise TypeError(f"FP8 storage must have one-byte elements, got {raw.dtype}")
    return raw.contiguous().view(torch.uint8)


def _value_of(exponent: torch.Tensor, mantissa: torch.Tensor) -> torch.Tensor:
    e = exponent.to(torch.float32)
    m = mantissa.to(torch.float32)
    return torch.where(exponent == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * torch.exp2(e - 7.0))


_E4M3FN_LUT: dict = {}


def _e4m3fn_lut(device) -> torch.Tensor:
    """The 256 E4M3FN values (NaN at 0x7F / 0xFF), built once per device from the bit layout."""
    key = str(device)
    if key not in _E4M3FN_LUT:
        _E4M3FN_LUT[key] = _decode_bits(torch.arange(256, dtype=torch.uint8), False).to(device)
    return _E4M3FN_LUT[key]


def decode_e4m3fn(raw: torch.Tensor, reject_nan: bool = True) -> torch.Tensor:
    """OCP E4M3FN bytes -> float32 (a 256-entry table built from the bit layout;
    no float8 dtype needed)."""
    b = _bytes(raw)
    if reject_nan and bool(((b & 0x7F) == 0x7F).any()):
        raise ValueError(f"E4M3FN tensor holds {int(((b & 0x7F) == 0x7F).sum())} NaN encodings")
    return _e4m3fn_lut(b.device)[b.long()]


def _decode_bits(raw: torch.Tensor, reject_nan: bool = True) -> torch.Tensor:
    b = _bytes(raw)
    sign = (b >> 7).bool()
    exp = ((b >> 3) & 0xF).to(torch.int32)
    man = (b & 0x7).to(torch.int32)
    nan = (exp == 0xF) & (man == 0x7)
    if reject_nan and bool(nan.any()):
        raise ValueError(f"E4M3FN tensor holds {int(nan.sum())} NaN encodings")
    v = _value_of(exp, man)
    v = torch.where(sign, -v, v)
    if not reject_nan:
        v = torch.where(nan, torch.full_like(v, float("nan")), v)
    return v


def _positive_table(max_code: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    codes = torch.arange(max_code + 1, dtype=torch.int32, device=device)
    return codes, _value_of(codes >> 3, codes & 7)


def _encode(values: torch.Tensor, max_code: int, vmax: float) -> torch.Tensor:
    """Round-to-nearest-even onto the positive code table, sign applied after."""
    v = values.float()
    if not bool(torch.isfinite(v).all()):
        raise ValueError("cannot encode non-finite values as E4M3")
    mag = v.abs().clamp_max(vmax).reshape(-1)
    codes, pos = _positive_table(max_code, v.device)
    mids = (pos[:-1] + pos[1:]) * 0.5
    sel = torch.bucketize(mag, mids, right=False)
    # a tie at a midpoint goes to the even code
    lower = sel.clamp_max(mids.numel() - 1)
    tie = (sel < pos.numel() - 1) & (mag == mids.index_select(0, lower))
    sel = sel + (tie & ((sel & 1) != 0)).to(sel.dtype)
    enc = codes.index_select(0, sel).to(torch.uint8).reshape(v.shape)
    neg = torch.signbit(v) & (v.abs() != 0)
    return enc | (neg.to(torch.uint8) << 7)


def encode_e4m3fn(values: torch.Tensor) -> torch.Tensor:
    """float -> E4M3FN bytes (uint8), saturating at 448, ties to even."""
    return _encode(values, 0x7E, E4M3FN_MAX)


def encode_legacy_e4m3(values: torch.Tensor) -> torch.Tensor:
    """float -> legacy finite E4M3 bytes (int8 view), saturating at 240."""
    return _encode(values, 0x77, LEGACY_E4M3_MAX).view(torch.int8)


def decode_legacy_e4m3(raw: torch.Tensor) -> torch.Tensor:
    b = _bytes(raw)
    if bool((((b >> 3) & 0xF) == 0xF).any()):
        raise ValueError("legacy E4M3 bytes use the reserved exponent 15")
    v = _value_of(((b >> 3) & 0xF).to(torch.int32), (b & 0x7).to(torch.int32))
    return torch.where((b >> 7).bool(), -v, v)


def scale_grid(shape, block: int = BLOCK) -> tuple[int, int]:
    return math.ceil(shape[-2] / block), math.ceil(shape[-1] / block)


def expand_block_scales(scales: torch.Tensor, shape, block: int = BLOCK) -> torch.Tensor:
    want = (*shape[:-2], *scale_grid(shape, block))
    if tuple(scales.shape) != want:
        raise ValueError(f"scales {tuple(scales.shape)} do not match {want}")
    e = scales.repeat_interleave(block, -2).repeat_interleave(block, -1)
    return e[..., : shape[-2], : shape[-1]]


def quantize_block(w: torch.Tensor, block: int = BLOCK):
    """``w [.., N, K]`` -> ``(w8 uint8 E4M3FN, scales fp32 [.., N/128, K/128])``
    with ``scale = amax(block) / 448`` (value = fp8 * scale)."""
    wf = w.float()
    *lead, N, K = wf.shape
    nb, kb = scale_grid(wf.shape, block)
    pad = torch.zeros(*lead, nb * block, kb * block, dtype=torch.float32, device=wf.device)
    pad[..., :N, :K] = wf
    blocks = pad.reshape(*lead, nb, block, kb, block)
    amax = blocks.abs().amax(dim=(-3, -1))
    scales = (amax / E4M3FN_MAX).clamp_min(1e-12)
    q = blocks / scales[..., :, None, :, None]
    w8 = q.reshape(*lead, nb * block, kb * block)[..., :N, :K].to(torch.float8_e4m3fn).view(torch.uint8)
    return w8.contiguous(), scales.contiguous()


def dequantize_block(w8: torch.Tensor, scales: torch.Tensor, block: int = BLOCK) -> torch.Tensor:
    v = decode_e4m3fn(w8, reject_nan=False)
    return v * expand_block_scales(scales.float(), v.shape, block)


class FP8Weight:
    """A 128x128 block-scaled E4M3FN weight ``[N, K]`` (W8A16 operand)."""

    __slots__ = ("w8", "scales")

    def __init__(self, w8: torch.Tensor, scales: torch.Tensor):
        self.w8 = w8
        self.scales = scales.float().contiguous()

    @staticmethod
    def from_dense(w: torch.Tensor) -> "FP8Weight":
        w8, s = quantize_block(w)
        return FP8Weight(w8.to(w.device), s.to(w.device))

    @property
    def shape(self):
        return self.w8.shape

    def dequant(self) -> torch.Tensor:
        return dequantize_block(self.w8, self.scales)

    def to(self, device) -> "FP8Weight":
        return FP8Weight(self.w8.to(device), self.scales.to(device))

    def nbytes(self) -> int:
        return self.w8.numel() + self.scales.numel() * 4


ROW_GROUP = 16  # rows per expert-weight scale (the gate/up interleave block)


def _scales16(scales: torch.Tensor, rows: int, block: int = BLOCK) -> torch.Tensor:
    """128-row block scales ``[.., ceil(rows/128), KB]`` repeated over their
    16-row groups: ``[.., rows/16, KB]``."""
    rep = scales.repeat_interleave(block // ROW_GROUP, dim=-2)
    return rep[..., : rows // ROW_GROUP, :].contiguous()


class FP8Experts:
    """Stacked expert weights ``[E, N, K]`` in E4M3FN with one fp32 scale per
    16 rows x 128 columns (``scales16 [E, N/16, ceil(K/128)]``, value = fp8 *
    scale): the operand of the fp8 grouped expert GEMM.  Built from 128x128
    block quantization of each original matrix (the official checkpoints'
    blocks); the 16-row granularity lets the block-16 gate/up interleave keep
    each row's own scale."""

    __slots__ = ("w8", "scales16")

    def __init__(self, w8: torch.Tensor, scales16: torch.Tensor):
        if w8.dim() != 3 or w8.shape[1] % ROW_GROUP:
            raise ValueError(f"expert weights [E, N, K] with N a multiple of {ROW_GROUP}, got {tuple(w8.shape)}")
        want = (w8.shape[0], w8.shape[1] // ROW_GROUP, math.ceil(w8.shape[2] / BLOCK))
        if tuple(scales16.shape) != want:
            raise ValueError(f"scales16 {tuple(scales16.shape)} != {want}")
        self.w8 = w8.contiguous()
        self.scales16 = scales16.float().contiguous()

    @staticmethod
    def quantize(w: torch.Tensor) -> "FP8Experts":
        """``w [E, N, K]`` with 128x128 blocks per expert (a down projection)."""
        w8, s = quantize_block(w)
        return FP8Experts(w8, _scales16(s, w.shape[1]))

    @staticmethod
    def quantize_gate_up(gate: torch.Tensor, up: torch.Tensor, block: int = ROW_GROUP) -> "FP8Experts":
        """``gate, up [E, I, K]``, each quantized in its own 128x128 blocks, rows
        interleaved in 16s (the layout of the fused SwiGLU epilogue)."""
        E, I, K = gate.shape
        g8, gs = quantize_block(gate)
        u8, us = quantize_block(up)
        w8 = torch.stack([g8.reshape(E, I // block, block, K), u8.reshape(E, I // block, block, K)], dim=2)
        s16 = torch.stack([_scales16(gs, I), _scales16(us, I)], dim=2)
        return FP8Experts(w8.reshape(E, 2 * I, K), s16.reshape(E, 2 * I // ROW_GROUP, -1))

    @staticmethod
    def from_interleaved(w_il: torch.Tensor, block: int = ROW_GROUP) -> "FP8Experts":
        """Quantize already-interleaved bf16 gate/up weights ``[E, 2I, K]``."""
        E, n2, K = w_il.shape
        x = w_il.reshape(E, n2 // (2 * block), 2, block, K)
        return FP8Experts.quantize_gate_up(x[:, :, 0].reshape(E, n2 // 2, K), x[:, :, 1].reshape(E, n2 // 2, K))

    @property
    def shape(self):
        return self.w8.shape

    def dequant(self) -> torch.Tensor:
        """fp32 ``[E, N, K]``."""
        v = decode_e4m3fn(self.w8, reject_nan=False)
        s = self.scales16.repeat_interleave(ROW_GROUP, dim=1).repeat_interleave(BLOCK, dim=2)
        return v * s[..., : v.shape[2]]

    def to(self, device) -> "FP8Experts":
        return FP8Experts(self.w8.to(device), self.scales16.to(device))

    def select(self, e0: int, e1: int) -> "FP8Experts":
        """Experts ``[e0, e1)`` (an expert-parallel rank's slice)."""
        return FP8Experts(self.w8[e0:e1], self.scales16[e0:e1])

    def nbytes(self) -> int:
        return self.w8.numel() + self.scales16.numel() * 4
