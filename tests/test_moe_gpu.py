"""MoE kernels (router top-k, stable route packing, grouped tcgen05 GEMMs,
combine) vs the fp32 PyTorch references, including expert-parallel slices."""
import pytest
import torch

import bwn.ops as O
from bwn.ops import reference as R

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("T,E,k", [(1, 256, 8), (37, 256, 8), (5, 16, 4), (300, 128, 6)])
def test_topk_softmax(T, E, k):
    logits = torch.randn(T, E, device=dev) * 3
    w, ids = O.moe_topk_softmax(logits, k)
    wr, ir = R.moe_route_softmax(logits.cpu(), k)
    assert torch.equal(ids.cpu().sort(-1).values, ir.sort(-1).values)
    assert torch.allclose(w.cpu().sort(-1).values, wr.sort(-1).values, atol=1e-5)


@pytest.mark.parametrize("func", ["sqrtsoftplus", "sigmoid"])
def test_topk_deepseek(func):
    logits = torch.randn(50, 256, device=dev)
    bias = torch.randn(256, device=dev) * 0.1
    w, ids = O.moe_topk_deepseek(logits, bias, 6, func, 1.5)
    wr, ir = R.moe_route_deepseek(logits.cpu(), bias.cpu(), 6, func, 1.5)
    assert torch.equal(ids.cpu().sort(-1).values, ir.sort(-1).values)
    assert torch.allclose(w.cpu().sort(-1).values, wr.sort(-1).values, atol=1e-5)


@pytest.mark.parametrize("T,E_total,E_local,e0,k,H,I", [(32, 64, 64, 0, 8, 256, 128), (7, 64, 16, 16, 4, 512, 256),
                                                         (200, 32, 8, 24, 8, 256, 64), (1, 256, 32, 0, 8, 2048, 512)])
def test_moe_experts(T, E_total, E_local, e0, k, H, I):
    x = torch.randn(T, H, device=dev).bfloat16()
    logits = torch.randn(T, E_total, device=dev)
    w, ids = O.moe_topk_softmax(logits, k)
    g = (torch.randn(E_local, I, H, device=dev) / H ** 0.5).bfloat16()
    u = (torch.randn(E_local, I, H, device=dev) / H ** 0.5).bfloat16()
    dn = (torch.randn(E_local, H, I, device=dev) / I ** 0.5).bfloat16()
    gu_il = torch.stack([O.interleave_gate_up(g[e], u[e]) for e in range(E_local)])
    sy = torch.randn(T, H, device=dev).bfloat16()
    sg = torch.randn(T, 1, device=dev)
    out = O.moe_experts(x, w, ids, gu_il, dn, e0, shared=(sy, sg))
    torch.cuda.synchronize()
    O.check_status("moe_experts")
    ref = R.moe_experts(x.cpu(), w.cpu(), ids.cpu(), torch.cat([g, u], 1).cpu(), dn.cpu(), e0)
    ref = ref + torch.sigmoid(sg.cpu()) * sy.cpu().float()
    assert _rel(out.cpu(), ref) < 2e-2
    out2 = O.moe_experts(x, w, ids, gu_il, dn, e0, shared=(sy, sg))
    assert torch.equal(out, out2)  # deterministic packing


def test_moe_model_decode_matches_cpu():
    from bwn.config import tiny_qwen36
    from bwn.io import qwen36_weights as W
    from bwn.models.qwen36 import build_qwen36

    cfg = tiny_qwen36(moe=True)
    hf = dict(W.synthetic_hf_globals(cfg, 9, "cpu"))
    for i in range(cfg.num_layers):
        hf.update(W.synthetic_hf_layer(cfg, i, 9, "cpu"))
    g = build_qwen36(cfg, device="cuda", hf_state=hf)
    c = build_qwen36(cfg, device="cpu", hf_state=hf, dtype=torch.float32)
    toks = torch.randint(0, cfg.vocab, (2, 40))
    sg, sc = g.new_state(2, 128), c.new_state(2, 128)
    hg = g.prefill_hidden(toks.cuda(), sg)
    hc = c.prefill_hidden(toks, sc)
    assert _rel(hg.cpu(), hc) < 5e-2
    t = c.logits(hc).argmax(-1).int()
    for _ in range(3):
        hg = g.decode_hidden(t.cuda(), sg)
        hc = c.decode_hidden(t, sc)
        torch.cuda.synchronize()
        assert _rel(hg.cpu(), hc) < 5e-2
        t = c.logits(hc).argmax(-1).int()
