"""FP8 formats: exhaustive E4M3FN decode against torch's float8 dtype, legacy
E4M3 round trip, block quantisation error bounds, and the FP8 model path."""
import pytest
import torch

from bwn.io import fp8 as F


def test_decode_e4m3fn_exhaustive():
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8)
    ours = F.decode_e4m3fn(codes, reject_nan=False)
    theirs = codes.view(torch.float8_e4m3fn).float()
    nan = torch.isnan(theirs)
    assert torch.equal(torch.isnan(ours), nan)
    assert torch.equal(ours[~nan], theirs[~nan])
    with pytest.raises(ValueError):
        F.decode_e4m3fn(torch.tensor([0x7F], dtype=torch.uint8))


def test_encode_matches_torch_cast():
    x = torch.randn(5000) * 50
    x = torch.cat([x, torch.tensor([0.0, -0.0, 448.0, -448.0, 1000.0, 2 ** -9, 3 * 2 ** -10])])
    ours = F.encode_e4m3fn(x)
    ref = x.clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    assert torch.equal(F.decode_e4m3fn(ours), F.decode_e4m3fn(ref))


def test_legacy_roundtrip():
    x = torch.linspace(-300, 300, 4001)
    enc = F.encode_legacy_e4m3(x)
    dec = F.decode_legacy_e4m3(enc)
    assert dec.abs().max() <= F.LEGACY_E4M3_MAX
    inside = x.abs() <= 240
    rel = ((dec - x).abs() / x.abs().clamp_min(1e-3))[inside & (x.abs() > 0.05)]
    assert rel.max() < 0.07


def test_block_quantization():
    w = torch.randn(300, 260) * 0.05
    w8, s = F.quantize_block(w)
    assert w8.dtype == torch.uint8 and s.shape == (3, 3)
    back = F.dequantize_block(w8, s)
    err = (back - w).abs() / (w.abs().amax() + 1e-12)
    assert err.max() < 0.04
    assert ((back - w).norm() / w.norm()) < 0.04


def test_fp8_model_runs_cpu():
    from bwn.config import tiny_qwen36
    from bwn.models.qwen36 import build_qwen36

    cfg = tiny_qwen36()
    m = build_qwen36(cfg, seed=0, dtype=torch.float32)
    st = m.new_state(1, 32)
    toks = torch.randint(0, cfg.vocab, (1, 8))
    a = m.logits(m.prefill_hidden(toks, st))
    m.quantize_fp8()
    st2 = m.new_state(1, 32)
    b = m.logits(m.prefill_hidden(toks, st2))
    assert ((a - b).norm() / a.norm()) < 0.1


def test_fp8_experts_scale_layout_follows_the_interleave():
    """Gate and up quantized in their own 128x128 blocks, rows interleaved in
    16s: every 16-row group of the interleaved matrix carries the scale of
    the original block it came from, so dequantization equals interleaving
    the per-matrix dequantizations."""
    from bwn import ops as O
    from bwn.io.fp8 import FP8Experts, dequantize_block, quantize_block
    torch.manual_seed(0)
    E, I, K = 3, 192, 200  # partial 128-blocks in both dims
    gate = torch.randn(E, I, K) * torch.linspace(0.01, 2.0, I)[None, :, None]
    up = torch.randn(E, I, K) * 0.3
    fx = FP8Experts.quantize_gate_up(gate, up)
    assert fx.w8.shape == (E, 2 * I, K) and fx.scales16.shape == (E, 2 * I // 16, 2)
    g8, gs = quantize_block(gate)
    u8, us = quantize_block(up)
    want = torch.stack([O.interleave_gate_up(dequantize_block(g8[e], gs[e]), dequantize_block(u8[e], us[e]))
                        for e in range(E)])
    assert torch.equal(fx.dequant(), want)
    # from the interleaved bf16 layout the model holds
    il = torch.stack([O.interleave_gate_up(gate[e], up[e]) for e in range(E)])
    assert torch.equal(FP8Experts.from_interleaved(il).dequant(), want)
    assert (fx.dequant() - il).abs().max() <= 0.07 * il.abs().max()
    down = torch.randn(E, K - 8, I)  # N = 192 rows: 16-row groups of a partial 128-block
    fd = FP8Experts.quantize(down[:, :192])
    d8, ds = quantize_block(down[:, :192])
    assert torch.equal(fd.dequant(), torch.stack([dequantize_block(d8[e], ds[e]) for e in range(E)]))
    assert fd.nbytes() == fd.w8.numel() + fd.scales16.numel() * 4


def test_fp8_experts_through_the_moe_block():
    """The model's MoE block with fp8 experts equals the bf16 block run on the
    dequantized (bf16-rounded) weights."""
    from bwn.config import tiny_qwen36
    from bwn.models.moe import qwen_moe_forward
    from bwn.models.qwen36 import build_qwen36
    cfg = tiny_qwen36(moe=True)
    m = build_qwen36(cfg, seed=3, dtype=torch.float32)
    x = torch.randn(6, cfg.hidden)
    L = dict(m.layers[0])
    m.quantize_fp8(include_head=False, experts=True, dense=False)
    Lq = m.layers[0]
    assert hasattr(Lq["experts_gate_up"], "scales16") and hasattr(Lq["experts_down"], "scales16")
    assert torch.is_tensor(Lq["shared_gate_up"])  # dense=False: the other projections stay bf16
    got = qwen_moe_forward(m, Lq, x)
    L["experts_gate_up"] = Lq["experts_gate_up"].dequant().to(torch.bfloat16).float()
    L["experts_down"] = Lq["experts_down"].dequant().to(torch.bfloat16).float()
    ref = qwen_moe_forward(m, L, x)
    assert torch.allclose(got, ref, atol=1e-6)
