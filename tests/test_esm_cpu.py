"""ESM-2: parity with HF EsmForMaskedLM, masking statistics, MLM training and
checkpoint/resume (config 1: ESM-2 8M on CPU fp32, b8 x s256)."""
import os

import torch

from bwn.config import ESM2Config
from bwn.models.esm2 import EsmForMaskedLM
from bwn.train.esm_mlm import MLMConfig, MLMTrainer, mask_tokens, synthetic_batch


def _tiny():
    return ESM2Config(name="esm-tiny", num_layers=2, hidden=64, heads=4, ffn=128)


def test_matches_hf_esm():
    from transformers import EsmConfig
    from transformers import EsmForMaskedLM as HF

    cfg = _tiny()
    hc = EsmConfig(vocab_size=cfg.vocab, hidden_size=cfg.hidden, num_hidden_layers=cfg.num_layers,
                   num_attention_heads=cfg.heads, intermediate_size=cfg.ffn, position_embedding_type="rotary",
                   token_dropout=True, mask_token_id=cfg.mask_token_id, pad_token_id=cfg.pad_token_id,
                   layer_norm_eps=cfg.layer_norm_eps, emb_layer_norm_before=False, max_position_embeddings=1026)
    torch.manual_seed(0)
    hf = HF(hc).eval()
    m = EsmForMaskedLM(cfg)
    m.load_hf_state_dict(hf.state_dict())
    ids, am = synthetic_batch(cfg, 2, 30, torch.Generator().manual_seed(0))
    ids[0, 5] = cfg.mask_token_id
    with torch.no_grad():
        ref = hf(input_ids=ids, attention_mask=am).logits
        got = m(ids, am)
    assert torch.allclose(got, ref, atol=2e-4, rtol=1e-4), (got - ref).abs().max()


def test_mask_tokens_ratios():
    cfg = ESM2Config()
    ids, _ = synthetic_batch(cfg, 64, 256, torch.Generator().manual_seed(0))
    new, labels, lm = mask_tokens(ids, cfg, torch.Generator().manual_seed(1))
    frac = lm[:, 1:-1].mean().item()
    assert 0.13 < frac < 0.17
    chosen = lm.bool()
    assert not chosen[:, 0].any() and not chosen[:, -1].any()
    as_mask = (new == cfg.mask_token_id) & chosen
    assert 0.75 < as_mask.sum().item() / chosen.sum().item() < 0.85
    assert torch.equal(labels, ids)


def test_train_step_and_resume(tmp_path):
    cfg = ESM2Config()  # ESM-2 8M, fp32 on CPU (config 1)
    torch.manual_seed(0)
    model = EsmForMaskedLM(cfg).init_weights(0)
    tr = MLMTrainer(model, MLMConfig(batch=8, seq_len=256, lr=1e-4, warmup=1, total_steps=10, bf16=False))
    losses = [float(tr.step()) for _ in range(2)]
    assert all(l == l and l > 0 for l in losses)
    path = os.path.join(tmp_path, "ckpt.pt")
    tr.save(path)
    nxt = float(tr.step())
    model2 = EsmForMaskedLM(cfg)
    tr2 = MLMTrainer(model2, MLMConfig(batch=8, seq_len=256, lr=1e-4, warmup=1, total_steps=10, bf16=False))
    tr2.load(path)
    assert tr2.step_idx == 2
    nxt2 = float(tr2.step())
    assert abs(nxt - nxt2) < 1e-5, (nxt, nxt2)


def test_training_reduces_loss():
    cfg = _tiny()
    model = EsmForMaskedLM(cfg).init_weights(0)
    tr = MLMTrainer(model, MLMConfig(batch=16, seq_len=32, lr=3e-3, warmup=1, total_steps=60, bf16=False,
                                     loss_divisor="masked"))
    first = float(tr.step())
    for _ in range(40):
        last = float(tr.step())
    assert last < first - 0.3, (first, last)


def test_tokenize_and_predict_masked_middle():
    from bwn.train.esm_infer import predict_masked_middle, tokenize
    from bwn.train.esm_mlm import build_esm
    m = build_esm("8M", seed=0)
    ids, am = tokenize(["AC<mask>D", "LL"], m.cfg, 8)
    assert ids.shape == (2, 8) and int(am[0].sum()) == 6 and int(am[1].sum()) == 4
    assert int(ids[0, 3]) == m.cfg.mask_token_id and int(ids[0, 0]) == m.cfg.cls_token_id
    res = predict_masked_middle(m, ["MKTVRQERLK", "KALTAR"])
    assert [r["position"] for r in res] == [5, 3] and all(0 < r["prob"] <= 1 for r in res)


def test_infer_command_with_reference_flags(capsys):
    """``python -m bwn.train.esm_infer`` with the reference's flag names
    (``--model-size``, ``--max-seq-len``, ``--sequences``)."""
    import json

    from bwn.train.esm_infer import main
    main(["--model-size", "8M", "--max-seq-len", "32", "--sequences", "MKTVRQERLK", "KALTAR"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert [r["position"] for r in res] == [5, 3] and [r["true"] for r in res] == ["Q", "T"]


def test_rope_half_layouts_match_rotate_half():
    """``O.rope_half`` (the CPU twin of the fused kernel) equals HF's
    ``x*cos + rotate_half(x)*sin`` with the head-major transpose, and its
    ``sign=-1`` backward layout is the transposed rotation."""
    import torch
    from bwn import ops as O
    from bwn.models.esm2 import _rotate_half
    B, S, H, D = 2, 7, 3, 8
    x = torch.randn(B * S, H * D)
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2).float() / D))
    f = torch.outer(torch.arange(S).float(), inv)
    cos, sin = f.cos(), f.sin()
    y = O.rope_half(x, cos, sin, B, S, H, True, 1.0, 0.5)
    xs = x.view(B, S, H, D).transpose(1, 2)
    emb = torch.cat([f, f], -1)
    ref = (xs * emb.cos() + _rotate_half(xs) * emb.sin()) * 0.5
    assert torch.allclose(y, ref, atol=1e-6)
    g = torch.randn(B, H, S, D)
    xr = xs.clone().requires_grad_(True)
    ((xr * emb.cos() + _rotate_half(xr) * emb.sin()) * 0.5).backward(g)
    gx = O.rope_half(g, cos, sin, B, S, H, False, -1.0, 0.5)
    assert torch.allclose(gx, xr.grad.transpose(1, 2).reshape(B * S, H * D), atol=1e-6)
