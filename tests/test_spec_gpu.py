"""Speculative-verify kernels vs their fp32 oracles: the DeltaNet deferred-commit
verify over several steps with random acceptance, and the multi-token GQA
decode (n_tok query rows per cache sequence)."""
import pytest
import torch

from bwn import ops as O
from bwn.ops import reference as R
from _spec_util import dn_params, dn_rows

pytestmark = pytest.mark.gpu
dev = torch.device("cuda", 0)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-6)).item()


@pytest.mark.parametrize("B,KH,VH,N,state_dtype", [(2, 1, 2, 4, torch.float32), (3, 2, 6, 5, torch.float32),
                                                  (1, 16, 48, 5, torch.float32), (2, 2, 4, 3, torch.bfloat16)])
def test_deltanet_verify_vs_oracle(B, KH, VH, N, state_dtype):
    P = dn_params(KH, VH, dev, 7)
    Pc = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in P.items()}
    C = P["C"]
    gen = torch.Generator().manual_seed(3)
    ring = torch.zeros(B, 8, C, device=dev).bfloat16()
    state = torch.zeros(B, VH, 128, 128, device=dev, dtype=state_dtype)
    sq = torch.zeros(2, B, N, C, device=dev).bfloat16()
    sab = torch.zeros(2, B, N, 2 * VH, device=dev).bfloat16()
    vstep = torch.zeros(1, dtype=torch.int32, device=dev)
    pos = torch.arange(B, dtype=torch.int32, device=dev) * 3
    pend = torch.zeros(B, dtype=torch.int32, device=dev)
    ring_r, state_r, sq_r, sab_r = ring.cpu(), state.float().cpu(), sq.cpu(), sab.cpu()
    for step in range(5):
        qkv, z, a, b = dn_rows(B * N, KH, VH, dev, gen)
        out = O.deltanet_verify(qkv, z, a, b, sq, sab, vstep, ring, state, pos, pend, P["conv_w"], P["A_log"],
                                P["dt_bias"], P["norm_w"], KH, N)
        ref = R.deltanet_verify(qkv.cpu(), z.cpu(), a.cpu(), b.cpu(), sq_r, sab_r, vstep.cpu(), ring_r, state_r,
                                pos.cpu(), pend.cpu(), Pc["conv_w"], Pc["A_log"], Pc["dt_bias"], Pc["norm_w"], KH, N)
        torch.cuda.synchronize()
        tol = 2e-2 if state_dtype == torch.float32 else 6e-2
        assert _rel(out.cpu(), ref) < tol, step
        assert _rel(state.float().cpu(), state_r) < tol, step
        acc = torch.randint(1, N + 1, (B,), generator=gen).int()
        pos += acc.to(dev)
        pend.copy_(acc.to(dev))
        vstep += 1
    O.check_status("verify")


@pytest.mark.parametrize("B,QH,KVH,N,S", [(1, 24, 4, 5, 1024), (2, 6, 1, 4, 512), (3, 16, 2, 2, 2048)])
def test_gqa_decode_multi_token(B, QH, KVH, N, S):
    D = 256
    g = torch.Generator().manual_seed(5)
    qg = torch.randn(B * N, QH, 2 * D, generator=g).bfloat16().to(dev)
    kv = torch.randn(B * N, 2, KVH, D, generator=g).bfloat16().to(dev)
    k_new, v_new = kv[:, 0], kv[:, 1]
    kc = torch.randn(B, KVH, S, D, generator=g).bfloat16().to(dev)
    vc = torch.randn(B, KVH, S, D, generator=g).bfloat16().to(dev)
    qn = (torch.randn(D, generator=g) * 0.1).to(dev)
    kn = (torch.randn(D, generator=g) * 0.1).to(dev)
    cos, sin = R.rope_table(S, 64, 1e7, device=dev)
    start = torch.tensor([100 + 37 * i for i in range(B)], dtype=torch.int32)
    pos = (start[:, None] + torch.arange(N)[None]).reshape(-1).int().to(dev)
    kc_r, vc_r = kc.cpu(), vc.cpu()
    out = O.gqa_decode(qg, k_new, v_new, qn, kn, cos, sin, kc, vc, pos, n_tok=N)
    ref = R.gqa_decode(qg.cpu(), k_new.cpu(), v_new.cpu(), qn.cpu(), kn.cpu(), cos.cpu(), sin.cpu(), kc_r, vc_r,
                       pos.cpu(), 1e-6, N)
    torch.cuda.synchronize()
    assert _rel(out.cpu(), ref) < 2e-2
    assert _rel(kc.cpu(), kc_r) < 1e-2 and torch.equal(vc.cpu(), vc_r)
    O.check_status("gqa multi-token")
