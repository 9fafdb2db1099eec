"""DeepSeek V4 on the GPU (bwn kernels) against the CPU fp32 path of the same
weights, plus the HC / MQA / RoPE kernels against their references."""
import pytest
import torch

import bwn.ops as O
from bwn.config import tiny_deepseek_v4
from bwn.models.deepseek_v4 import DeepSeekV4Model, synthetic_checkpoint
from bwn.ops import reference as R

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.mark.parametrize("T", [5, 96])  # the mixes come from one bf16 tensor-core GEMM
def test_hc_kernels(T):
    hc, dim = 4, 256
    _check_hc(T, hc, dim)


def test_hc_pre_fused_gemv_fp32():
    """The in-kernel fp32 GEMV variant (BWN_HC_GEMM=0), run in a fresh interpreter."""
    import os
    import subprocess
    import sys
    code = ("import torch, tests.test_deepseek_gpu as t; t._check_hc(5, 4, 256, tol=1e-4)")
    r = subprocess.run([sys.executable, "-c", code], env={**os.environ, "BWN_HC_GEMM": "0"},
                       cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))), capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def _check_hc(T, hc, dim, tol=1e-2):  # 1e-2: the GEMM reads a bf16 copy of fn
    x = torch.randn(T, hc, dim, device="cuda").bfloat16()
    fn = torch.randn(24, hc * dim, device="cuda") * 0.02
    sc = torch.ones(3, device="cuda")
    bs = torch.randn(24, device="cuda") * 0.1
    y, post, comb = O.hc_pre(x, fn, sc, bs)
    yr, pr, cr = R.hc_pre(x.cpu(), fn.cpu(), sc.cpu(), bs.cpu())
    assert _rel(y.cpu(), yr) < 1e-2 and _rel(post.cpu(), pr) < tol and _rel(comb.cpu(), cr) < tol
    a = torch.randn(T, dim, device="cuda").bfloat16()
    out = O.hc_post(a, x, post, comb)
    assert _rel(out.cpu(), R.hc_post(a.cpu(), x.cpu(), pr, cr)) < 1e-2
    fnh = torch.randn(4, hc * dim, device="cuda") * 0.02
    yh, _, _ = O.hc_pre(x, fnh, sc[:1], bs[:4])
    assert _rel(yh.cpu(), R.hc_pre(x.cpu(), fnh.cpu(), sc[:1].cpu(), bs[:4].cpu())[0]) < 1e-2


@pytest.mark.parametrize("H,D", [(8, 512), (64, 512), (4, 64)])
def test_mqa_attn(H, D):
    B, S, per = 2, 300, 3
    q = torch.randn(B * per, H, D, device="cuda").bfloat16()
    kv = torch.randn(B, S, D, device="cuda").bfloat16()
    vis = torch.tensor([1, 150, 300, 7, 299, 64], dtype=torch.int32, device="cuda")
    out = O.mqa_attn(q, kv, vis, per, D ** -0.5)
    ref = R.mqa_attn(q.cpu(), kv.cpu(), vis.cpu(), per, D ** -0.5)
    assert _rel(out.cpu(), ref) < 2e-2


@pytest.mark.parametrize("H,per,S,start", [(8, 256, 320, 0), (8, 256, 320, 37), (64, 32, 64, 0)])
def test_mqa_prefill_tensor_core(H, per, S, start):
    """Prefill-sized MQA (the tcgen05 kernel: rows = token x head, causal per
    token, a chunk starting at ``start``) against the fp32 reference."""
    B, D = 2, 512
    q = torch.randn(B * per, H, D, device="cuda").bfloat16()
    kv = torch.randn(B, S, D, device="cuda").bfloat16()
    vis = (start + 1 + torch.arange(per, dtype=torch.int32)).repeat(B).cuda()
    out = O.mqa_attn(q, kv, vis, per, D ** -0.5)
    torch.cuda.synchronize()
    O.check_status("mqa prefill")
    ref = R.mqa_attn(q.cpu(), kv.cpu(), vis.cpu(), per, D ** -0.5)
    assert _rel(out.cpu(), ref) < 2e-2


def test_deepseek_gpu_matches_cpu():
    cfg = tiny_deepseek_v4()
    sd = synthetic_checkpoint(cfg, 4, "cpu")
    g = DeepSeekV4Model(cfg, device="cuda").load(sd)
    c = DeepSeekV4Model(cfg, dtype=torch.float32).load(sd)
    toks = torch.randint(0, cfg.vocab, (2, 20))
    sg, sc = g.new_state(2, 64), c.new_state(2, 64)
    ig, ic = g.prefill(toks.cuda(), sg), c.prefill(toks, sc)
    torch.cuda.synchronize()
    O.check_status("deepseek prefill")
    agree = (ig.cpu() == ic).float().mean().item()
    assert agree >= 0.5
    B = 2
    bidx = torch.arange(B, dtype=torch.int32)
    hg = g.forward_tokens(ic.cuda(), sg.positions, bidx.cuda(), sg, 1)
    hc = c.forward_tokens(ic, sc.positions, bidx, sc, 1)
    assert _rel(hg.cpu(), hc) < 6e-2


def test_deepseek_fp8_weights_match_bf16():
    """Block-scaled E4M3 dense projections, LM head and routed experts (the
    benchmark's fp8 configuration) against the bf16 model on the same weights."""
    cfg = tiny_deepseek_v4()
    sd = synthetic_checkpoint(cfg, 5, "cpu")
    g = DeepSeekV4Model(cfg, device="cuda").load(sd)
    q = DeepSeekV4Model(cfg, device="cuda").load(sd).quantize_fp8(include_head=True, experts=True)
    toks = torch.randint(0, cfg.vocab, (2, 24), generator=torch.Generator().manual_seed(1)).cuda()
    sg, sq = g.new_state(2, 64), q.new_state(2, 64)
    g.prefill(toks, sg)
    q.prefill(toks, sq)
    bidx = torch.arange(2, dtype=torch.int32, device="cuda")
    nxt = toks[:, -1].int()
    hg = g.forward_tokens(nxt, sg.positions, bidx, sg, 1)
    hq = q.forward_tokens(nxt, sq.positions, bidx, sq, 1)
    torch.cuda.synchronize()
    O.check_status("deepseek fp8")
    assert torch.isfinite(hq).all()
    assert _rel(hq.cpu(), hg.cpu()) < 0.15
