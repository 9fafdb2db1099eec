"""Prefill kernels (chunked DeltaNet, tcgen05 flash attention) vs the fp32
PyTorch references, including a non-zero start offset (prefix already in the
cache / conv ring), pad rows beyond valid_len, and a ragged last chunk."""
import pytest
import torch

import bwn.ops as O
from bwn.ops import reference as R

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _dn_case(B, S, KH, VH, start, near_one=False, seed=0):
    torch.manual_seed(seed)
    C = 2 * KH * 128 + VH * 128
    W = C + VH * 128 + 2 * VH
    proj = (torch.randn(B, S, W, device=dev) * 0.5).bfloat16()
    ring = (torch.randn(B, 4, C, device=dev) * 0.5).bfloat16() if start else torch.zeros(B, 4, C, device=dev).bfloat16()
    state = torch.randn(B, VH, 128, 128, device=dev) * 0.05 if start else torch.zeros(B, VH, 128, 128, device=dev)
    vl = torch.tensor([S - 3 * i for i in range(B)], dtype=torch.int32, device=dev)
    conv_w = torch.randn(C, 4, device=dev) * 0.5
    # near_one: decay exp(g) within 1e-3 of 1 (A_log very negative): the state
    # keeps almost everything over the whole prompt
    A_log = (torch.full((VH,), -8.0, device=dev) if near_one else torch.rand(VH, device=dev) * 2)
    return proj, ring, state, vl, conv_w, A_log


@pytest.mark.parametrize("B,S,KH,VH,start", [(2, 100, 2, 4, 0), (1, 64, 2, 6, 7), (3, 130, 2, 4, 2)])
def test_deltanet_prefill(B, S, KH, VH, start):
    _check_deltanet_prefill(B, S, KH, VH, start)


@pytest.mark.parametrize("near_one", [False, True], ids=["decaying", "near_one_decay"])
def test_deltanet_prefill_production_shape(near_one):
    """Qwen3.6-27B's shape at one GPU (16 K-heads, 48 V-heads) over a 2048-token prompt."""
    _check_deltanet_prefill(2, 2048, 16, 48, 0, near_one=near_one)


def _check_deltanet_prefill(B, S, KH, VH, start, near_one=False):
    C = 2 * KH * 128 + VH * 128
    proj, ring, state, vl, conv_w, A_log = _dn_case(B, S, KH, VH, start, near_one)
    qkv, z = proj[..., :C], proj[..., C:C + VH * 128]
    b_, a_ = proj[..., C + VH * 128:C + VH * 128 + VH], proj[..., C + VH * 128 + VH:]
    dt = torch.randn(VH, device=dev) * 0.1
    nw = torch.randn(128, device=dev) * 0.1 + 1
    ring_r, state_r = ring.cpu().clone(), state.cpu().clone()
    out = O.deltanet_prefill(qkv, z, a_, b_, ring, state, start, vl, conv_w, A_log, dt, nw, KH)
    torch.cuda.synchronize()
    ref = R.deltanet_prefill(qkv.cpu(), a_.cpu(), b_.cpu(), z.cpu(), ring_r, state_r, start, vl.cpu(), conv_w.cpu(),
                             A_log.cpu(), dt.cpu(), nw.cpu(), KH, 128, 128)
    for bi in range(B):
        n = int(vl[bi])
        assert _rel(out[bi, :n].cpu(), ref[bi, :n]) < 3e-2, bi
    assert _rel(state.cpu(), state_r) < 3e-2
    assert torch.equal(ring.cpu(), ring_r)


@pytest.mark.parametrize("B,S,QH,KVH,start", [(2, 200, 4, 2, 0), (1, 128, 6, 1, 37), (2, 300, 8, 1, 130),
                                               (1, 5, 3, 1, 0)])
def test_gqa_prefill(B, S, QH, KVH, start):
    D, SM = 256, 512
    proj = torch.randn(B, S, QH * 2 * D + 2 * KVH * D, device=dev).bfloat16()
    qg = proj[..., :QH * 2 * D].reshape(B, S, QH, 2 * D)
    k = proj[..., QH * 2 * D:QH * 2 * D + KVH * D].reshape(B, S, KVH, D)
    v = proj[..., QH * 2 * D + KVH * D:].reshape(B, S, KVH, D)
    qn = torch.randn(D, device=dev) * 0.1
    kn = torch.randn(D, device=dev) * 0.1
    cos, sin = R.rope_table(SM, 64, 1e7, device=dev)
    kc = torch.randn(B, KVH, SM, D, device=dev).bfloat16()
    vc = torch.randn(B, KVH, SM, D, device=dev).bfloat16()
    kc_r, vc_r = kc.cpu().clone(), vc.cpu().clone()
    out = O.gqa_prefill(qg, k, v, qn, kn, cos, sin, kc, vc, start)
    torch.cuda.synchronize()
    O.check_status("gqa_prefill")
    ref = O.gqa_prefill(qg.cpu(), k.cpu(), v.cpu(), qn.cpu(), kn.cpu(), cos.cpu(), sin.cpu(), kc_r, vc_r, start)
    assert _rel(out.cpu(), ref) < 3e-2
    assert _rel(kc.cpu(), kc_r) < 1e-2 and torch.equal(vc.cpu(), vc_r)


def test_model_prefill_matches_cpu():
    from bwn.config import tiny_qwen36
    from bwn.io import qwen36_weights as W
    from bwn.models.qwen36 import build_qwen36

    cfg = tiny_qwen36()
    hf = dict(W.synthetic_hf_globals(cfg, 5, "cpu"))
    for i in range(cfg.num_layers):
        hf.update(W.synthetic_hf_layer(cfg, i, 5, "cpu"))
    g = build_qwen36(cfg, device="cuda", hf_state=hf)
    c = build_qwen36(cfg, device="cpu", hf_state=hf, dtype=torch.float32)
    toks = torch.randint(0, cfg.vocab, (2, 150))
    vl = torch.tensor([150, 111], dtype=torch.int32)
    sg, sc = g.new_state(2, 256), c.new_state(2, 256)
    hg = g.prefill_hidden(toks.cuda(), sg, vl)
    hc = c.prefill_hidden(toks, sc, vl)
    torch.cuda.synchronize()
    assert _rel(hg.cpu(), hc) < 5e-2
    assert sg.positions.tolist() == [150, 111]
    # bucketed prefill on the GPU equals the one-shot GPU prefill
    sb = g.new_state(2, 256)
    ids_b = g.prefill(toks.cuda(), sb, vl, bucket=64)
    ids_1 = g.greedy(hg)
    assert torch.equal(ids_b, ids_1)
    assert _rel(sb.ssm, sg.ssm) < 2e-2


def test_graph_captured_bucketed_prefill():
    """One captured prefill chunk replayed at every offset (the start position is
    a device scalar) equals the eager bucketed prefill, with the short row first
    and a ragged last chunk padded to the bucket."""
    from bwn.config import tiny_qwen36
    from bwn.models.qwen36 import build_qwen36
    from bwn.runtime.static_decode import StaticDecoder

    cfg = tiny_qwen36()
    g = build_qwen36(cfg, device="cuda", seed=7)
    toks = torch.randint(0, cfg.vocab, (2, 150))
    vl = torch.tensor([111, 150], dtype=torch.int32)
    eager = g.new_state(2, 256)
    ids_e = g.prefill(toks.cuda(), eager, vl.cuda(), bucket=64)
    dec = StaticDecoder(g, 2, 256)
    dec.capture_prefill(64)
    ids_g = dec.prefill(toks, vl, bucket=64)
    torch.cuda.synchronize()
    from bwn.ops import check_status
    check_status("graphed prefill")
    assert torch.equal(ids_g, ids_e)
    assert dec.st.positions.tolist() == [111, 150]
    assert _rel(dec.st.ssm, eager.ssm) < 1e-3
    assert _rel(dec.st.k_cache[:, :, :, :111], eager.k_cache[:, :, :, :111]) < 1e-3
    # a second prompt through the same graph after a reset
    dec.reset()
    ids_g2 = dec.prefill(toks, vl, bucket=64)
    assert torch.equal(ids_g2, ids_e)
