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
