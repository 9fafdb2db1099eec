"""The fp8 grouped expert GEMM (``moe_experts_w8``: block-scaled E4M3FN expert
weights, 16-row scale groups across the gate/up interleave) against the fp32
PyTorch reference on the dequantized, bf16-rounded weights.  Shapes cover
every token-tile width (BN 16..128), DeepSeek's clamped SwiGLU, a K of 64
(experts sliced across ranks) and an expert-parallel slice.

Each case runs in its own interpreter, so an error in this kernel is reported
as this test's failure without touching the CUDA context of the other tests."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, sys, torch
sys.path.insert(0, {root!r})
import bwn.ops as O
from bwn.io.fp8 import FP8Experts
from bwn.ops import reference as R
T, E_total, E_local, e0, k, H, I, limit = {case}
dev = "cuda"
torch.manual_seed(0)
x = torch.randn(T, H, device=dev).bfloat16()
w, ids = O.moe_topk_softmax(torch.randn(T, E_total, device=dev), k)
g = torch.randn(E_local, I, H, device=dev) / H ** 0.5
u = torch.randn(E_local, I, H, device=dev) / H ** 0.5
dn = torch.randn(E_local, H, I, device=dev) / I ** 0.5
gu8 = FP8Experts.quantize_gate_up(g, u)
dn8 = FP8Experts.quantize(dn)
sy = torch.randn(T, H, device=dev).bfloat16()
sg = torch.randn(T, 1, device=dev)
out = O.moe_experts(x, w, ids, gu8, dn8, e0, shared=(sy, sg), swiglu_limit=limit)
torch.cuda.synchronize()
O.check_status("moe_experts_w8")
gq = gu8.dequant().to(torch.bfloat16).float().cpu()
gate_up = torch.cat([gq.reshape(E_local, I // 16, 2, 16, H)[:, :, 0].reshape(E_local, I, H),
                     gq.reshape(E_local, I // 16, 2, 16, H)[:, :, 1].reshape(E_local, I, H)], 1)
ref = R.moe_experts(x.cpu(), w.cpu(), ids.cpu(), gate_up, dn8.dequant().to(torch.bfloat16).float().cpu(), e0, limit)
ref = ref + torch.sigmoid(sg.cpu()) * sy.cpu().float()
rel = ((out.cpu().float() - ref).norm() / (ref.norm() + 1e-12)).item()
again = O.moe_experts(x, w, ids, gu8, dn8, e0, shared=(sy, sg), swiglu_limit=limit)
print(json.dumps({{"rel": rel, "deterministic": bool(torch.equal(out, again))}}))
"""


@pytest.mark.parametrize("case", [
    (5, 16, 16, 0, 4, 256, 128, 0.0),       # BN 16
    (24, 32, 32, 0, 4, 512, 128, 0.0),      # BN 32
    (40, 16, 16, 0, 8, 256, 256, 0.0),      # BN 64
    (300, 8, 8, 0, 4, 256, 128, 0.0),       # BN 128, several row tiles per expert
    (7, 64, 16, 16, 4, 512, 256, 7.0),      # expert-parallel slice, clamped SwiGLU
    (9, 32, 32, 0, 8, 2048, 64, 0.0),       # K = 64 down projection (experts sliced 8 ways)
])
def test_moe_experts_w8(case):
    code = CHILD.format(root=ROOT, case=case)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["rel"] < 2e-2, res
    assert res["deterministic"]
