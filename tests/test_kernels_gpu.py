"""CUDA kernels vs the fp32 PyTorch references (GPU tier).

Each test runs the tcgen05/TMA kernel through ``torch.ops.bwn`` and compares
against :mod:`bwn.ops.reference` evaluated in fp32 on the same inputs.
"""
import math

import pytest
import torch

import bwn.ops as O
from bwn.ops import reference as R

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize(
    "M,N,K",
    [
        (1, 256, 512),
        (7, 384, 1024),
        (32, 5120, 768),     # decode o_proj/out_proj at TP=8 (swap-AB + split-K)
        (32, 2176 * 2, 5120),
        (128, 1000, 256),    # ragged N
        (300, 640, 4096),    # normal orientation, ragged M
        (2048, 2048, 2048),  # prefill-sized, many tiles
    ],
)
def test_linear(M, N, K):
    x = torch.randn(M, K, device=dev).bfloat16()
    w = (torch.randn(N, K, device=dev) / math.sqrt(K)).bfloat16()
    y = O.linear(x, w)
    torch.cuda.synchronize()
    O.check_status("linear")
    ref = x.float() @ w.float().t()
    assert y.shape == (M, N)
    assert _rel(y, ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(256, 512, 1024), (104, 320, 192), (4096, 2560, 2560), (8, 64, 128)])
def test_mn_major_gemms(M, N, K):
    """MN-major B (dX = dY @ W) and MN-major A+B (dW = dY^T @ X) descriptors."""
    x = torch.randn(M, K, device=dev).bfloat16()
    w_kn = (torch.randn(K, N, device=dev) / math.sqrt(K)).bfloat16()
    y = O.linear_kn(x, w_kn)
    assert _rel(y, x.float() @ w_kn.float()) < 1e-2
    a = torch.randn(K, M, device=dev).bfloat16()
    b = torch.randn(K, N, device=dev).bfloat16()
    for f32 in (False, True):
        z = O.matmul_tn(a, b, f32)
        assert z.dtype == (torch.float32 if f32 else torch.bfloat16)
        assert _rel(z, a.float().t() @ b.float()) < 1e-2
    O.check_status("mn-major gemm")


@pytest.mark.parametrize("M,N,K", [(1, 320, 320), (24, 1280, 320), (2048, 1280, 320), (4096, 2560, 10240)])
def test_linear_bias_epilogue(M, N, K):
    """``x @ w.T + b`` with the bias read through a row stride of 0 by the
    residual epilogue: token-swapped, split-K and full-tile paths."""
    x = torch.randn(M, K, device=dev).bfloat16()
    w = (torch.randn(N, K, device=dev) / math.sqrt(K)).bfloat16()
    b = torch.randn(N, device=dev)  # fp32 master bias, rounded to bf16 inside
    y = O.linear_bias(x, w, b)
    torch.cuda.synchronize()
    O.check_status("linear_bias")
    assert y.shape == (M, N) and y.dtype == torch.bfloat16
    assert _rel(y, x.float() @ w.float().t() + b.bfloat16().float()) < 1e-2


@pytest.mark.parametrize("T", [1, 16, 300])
def test_linear_into_strided_views(T):
    """Grouped low-rank projection (DeepSeek's wo_a): each group's GEMM reads a
    column slice of the attention output and writes a column slice of the
    result, through the row strides; the columns around it stay untouched."""
    G, Kg, R = 4, 512, 256
    og = torch.randn(T, G * Kg, device=dev).bfloat16().view(T, G, Kg)
    w = (torch.randn(G, R, Kg, device=dev) / math.sqrt(Kg)).bfloat16()
    out = torch.full((T, G * R), 7.0, device=dev).bfloat16()
    for g in range(0, G, 2):  # every other group: the skipped slices must keep their fill
        O.linear_into(og[:, g], w[g], out[:, g * R:(g + 1) * R])
    torch.cuda.synchronize()
    O.check_status("linear_into")
    for g in range(G):
        got = out[:, g * R:(g + 1) * R]
        if g % 2:
            assert bool((got == 7.0).all())
        else:
            assert _rel(got, og[:, g].float() @ w[g].float().t()) < 1e-2


@pytest.mark.parametrize("M", [1, 32, 200])
def test_linear_swiglu_and_resid(M):
    K, I = 1024, 512
    x = torch.randn(M, K, device=dev).bfloat16()
    g = (torch.randn(I, K, device=dev) / math.sqrt(K)).bfloat16()
    u = (torch.randn(I, K, device=dev) / math.sqrt(K)).bfloat16()
    w = O.interleave_gate_up(g, u)
    y = O.linear_swiglu(x, w)
    ref = torch.nn.functional.silu(x.float() @ g.float().t()) * (x.float() @ u.float().t())
    assert _rel(y, ref) < 1e-2
    r = torch.randn(M, I, device=dev).bfloat16()
    y2 = O.linear_residual(x, g, r)
    assert _rel(y2, x.float() @ g.float().t() + r.float()) < 1e-2
    y3 = O.linear_f32(x, g)
    assert y3.dtype == torch.float32 and _rel(y3, x.float() @ g.float().t()) < 1e-2


def test_linear_repeat_graph():
    """split-K tickets re-arm: repeated launches (and a CUDA graph replay) stay exact."""
    x = torch.randn(16, 2048, device=dev).bfloat16()
    w = (torch.randn(1024, 2048, device=dev) / 45).bfloat16()
    ref = O.linear(x, w).clone()
    for _ in range(5):
        assert torch.equal(O.linear(x, w), ref)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        O.linear(x, w)
        with torch.cuda.graph(g, stream=s):
            out = O.linear(x, w)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("rows,cols", [(1, 5120), (33, 2048), (4, 256)])
def test_rms_norms(rows, cols):
    x = torch.randn(rows, cols, device=dev).bfloat16()
    w = torch.randn(cols, device=dev) * 0.1
    assert _rel(O.rms_norm(x, w), R.rms_norm(x.float(), w)) < 1e-2
    res = torch.randn(rows, cols, device=dev).bfloat16()
    res_ref = res.clone()
    out = O.add_rms_norm(x, res, w)
    r2, n2 = R.add_rms_norm(x, res_ref, w)
    assert _rel(res, r2) < 1e-2 and _rel(out, n2) < 1e-2


def test_embedding_and_argmax():
    table = torch.randn(1000, 256, device=dev).bfloat16()
    ids = torch.tensor([0, 5, 999, 1200, -3], device=dev, dtype=torch.int32)
    e = O.embedding(ids, table, offset=0)
    assert torch.equal(e[:3], table[[0, 5, 999]]) and (e[3:] == 0).all()
    e2 = O.embedding(ids, table[500:], offset=500)
    assert torch.equal(e2[2], table[999]) and (e2[0] == 0).all()
    logits = torch.randn(3, 777, device=dev)
    logits[1, 10] = 50.0
    logits[1, 20] = 50.0  # tie -> lowest id
    k = O.argmax_packed(logits, id_offset=100)
    ids = O.unpack_argmax(k)
    assert ids.tolist()[1] == 110
    assert ids.tolist()[0] == int(logits[0].argmax()) + 100
    kc = O.argmax_packed(logits.cpu(), id_offset=100)
    assert torch.equal(kc, k.cpu())


@pytest.mark.parametrize("B,KH,VH", [(1, 2, 6), (4, 16, 48), (3, 2, 4)])
@pytest.mark.parametrize("state_dtype", [torch.float32, torch.bfloat16])
def test_deltanet_decode(B, KH, VH, state_dtype):
    C = 2 * KH * 128 + VH * 128
    fused = torch.randn(B, C + VH * 128 + 2 * VH, device=dev).bfloat16()  # [qkv | z | b | a]
    qkv, z = fused[:, :C], fused[:, C:C + VH * 128]
    b_, a_ = fused[:, C + VH * 128:C + VH * 128 + VH], fused[:, C + VH * 128 + VH:]
    ring = torch.randn(B, 4, C, device=dev).bfloat16()
    state = (torch.randn(B, VH, 128, 128, device=dev) * 0.1).to(state_dtype)
    pos = torch.tensor([5 + 3 * i for i in range(B)], device=dev, dtype=torch.int32)
    conv_w = torch.randn(C, 4, device=dev) * 0.5
    A_log = torch.rand(VH, device=dev) * 2
    dt_bias = torch.randn(VH, device=dev) * 0.1
    norm_w = torch.randn(128, device=dev) * 0.1 + 1
    ring_r, state_r = ring.clone().cpu(), state.clone().float().cpu()
    for step in range(3):
        out = O.deltanet_decode(qkv, z, a_, b_, ring, state, pos, conv_w, A_log, dt_bias, norm_w, KH)
        ref = R.deltanet_decode(qkv.cpu(), a_.cpu(), b_.cpu(), z.cpu(), ring_r, state_r, pos.cpu(), conv_w.cpu(),
                                A_log.cpu(), dt_bias.cpu(), norm_w.cpu(), KH, 128, 128)
        torch.cuda.synchronize()
        tol = 2e-2 if state_dtype == torch.float32 else 5e-2
        assert _rel(out.cpu(), ref) < tol, step
        assert _rel(state.float().cpu(), state_r) < tol
        assert torch.equal(ring.cpu(), ring_r)
        pos += 1
        qkv.copy_(torch.randn_like(qkv.float()).bfloat16())


@pytest.mark.parametrize("B,QH,KVH,S,plen", [(1, 3, 1, 512, 77), (4, 24, 4, 1024, 300), (2, 16, 2, 4096, 2049),
                                            (3, 2, 1, 256, 0)])
def test_gqa_decode(B, QH, KVH, S, plen):
    D = 256
    qg = torch.randn(B, QH, 2 * D, device=dev).bfloat16()
    kv = torch.randn(B, 2, KVH, D, device=dev).bfloat16()
    k_new, v_new = kv[:, 0], kv[:, 1]
    qn = torch.randn(D, device=dev) * 0.1
    kn = torch.randn(D, device=dev) * 0.1
    cos, sin = R.rope_table(S, 64, 1e7, device=dev)
    kc = torch.randn(B, KVH, S, D, device=dev).bfloat16()
    vc = torch.randn(B, KVH, S, D, device=dev).bfloat16()
    pos = torch.tensor([max(0, plen - i) for i in range(B)], device=dev, dtype=torch.int32)
    kc_r, vc_r = kc.clone().cpu(), vc.clone().cpu()
    out = O.gqa_decode(qg, k_new, v_new, qn, kn, cos, sin, kc, vc, pos)
    torch.cuda.synchronize()
    O.check_status("gqa_decode")
    ref = R.gqa_decode(qg.cpu(), k_new.cpu(), v_new.cpu(), qn.cpu(), kn.cpu(), cos.cpu(), sin.cpu(), kc_r, vc_r,
                       pos.cpu())
    assert _rel(out.cpu(), ref) < 2e-2
    assert _rel(kc.cpu(), kc_r) < 1e-2 and torch.equal(vc.cpu(), vc_r)
    # a second call (tickets re-armed) gives the same answer
    out2 = O.gqa_decode(qg, k_new, v_new, qn, kn, cos, sin, kc, vc, pos)
    assert _rel(out2, out) < 1e-3


@pytest.mark.parametrize("T,N,K", [(1, 512, 1024), (32, 5120, 6144), (32, 2176 * 2, 5120), (7, 384, 256),
                                   (100, 1024, 2048)])
def test_linear_w8(T, N, K):
    """FP8 W8A16 with 128x128 block scales vs the fp32 product with dequantised weights."""
    from bwn.io.fp8 import FP8Weight
    x = torch.randn(T, K, device=dev).bfloat16()
    w = torch.randn(N, K, device=dev) * 0.05
    w[: N // 2] *= 4.0  # blocks with different scales
    fw = FP8Weight.from_dense(w)
    wd = fw.dequant().cuda()
    ref = x.float() @ wd.t()
    assert _rel(O.linear(x, fw), ref) < 1e-2
    assert _rel(O.linear_f32(x, fw), ref) < 1e-2
    r = torch.randn(T, N, device=dev).bfloat16()
    assert _rel(O.linear_residual(x, fw, r), ref + r.float()) < 1e-2
    if N % 32 == 0:
        g, u = w[: N // 2], w[N // 2:]
        fil = FP8Weight.from_dense(O.interleave_gate_up(g, u))
        gd, ud = O.deinterleave_gate_up(fil.dequant().cuda())
        want = torch.nn.functional.silu(x.float() @ gd.t()) * (x.float() @ ud.t())
        assert _rel(O.linear_swiglu(x, fil), want) < 2e-2
    O.check_status("linear_w8")
