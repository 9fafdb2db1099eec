"""The NVLS fused all-reduce kernels on a one-GPU multicast object
(``FusedComm.on_local_multicast``): a world of one still runs the
``multimem.ld_reduce`` code path, so the epilogues can be checked in one
process against the fp32 PyTorch reference.

* ``gemm_allreduce_add_norm`` / ``allreduce_add_norm``: residual += partial,
  RMSNorm(1+w);
* ``gemm_allreduce_hc_post`` / ``allreduce_hc_post``: DeepSeek V4's
  hyper-connection post-mix of the reduced partial.

Every call is made twice, so both slots of the alternating selector are read.
Each case runs in its own interpreter.  The one-GPU multicast object and the
fused post-mix have not had their first GPU run yet; until they have, these
cases run only when ``LOCAL_MC_GPU_TEST=1`` is set."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(os.environ.get("LOCAL_MC_GPU_TEST") != "1",
                                 reason="one-GPU multicast path awaiting its first GPU run (LOCAL_MC_GPU_TEST=1)")]
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, sys, torch
sys.path.insert(0, {root!r})
import bwn.ops as O
from bwn.ops import reference as R
from bwn.parallel.fused import FusedComm
kind, T, H, K = {case}
dev = torch.device("cuda", 0)
g = torch.Generator(device=dev).manual_seed(1)
fc = FusedComm.on_local_multicast(H, max_rows=max(T, 32), device=dev, timeout_s=2.0)
errs = []
for it in range(2):
    a = torch.randn(T, K, device=dev, generator=g).bfloat16()
    w = (torch.randn(H, K, device=dev, generator=g) * K ** -0.5).bfloat16()
    part = (a.float() @ w.float().t()).bfloat16()
    if kind == "norm":
        nw = torch.randn(H, device=dev, generator=g) * 0.1
        resid = torch.randn(T, H, device=dev, generator=g).bfloat16()
        r0 = resid.float().clone()
        y = fc.gemm_allreduce_add_norm(a, w, resid, nw, 1e-6) if it == 0 else fc.allreduce_add_norm(part, resid, nw, 1e-6)
        s = r0 + part.float()
        ref = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-6) * (1 + nw)
        errs.append(float((resid.float() - s).abs().max() / s.abs().max()))
        errs.append(float((y.float() - ref).abs().max() / ref.abs().max()))
    else:
        resid = torch.randn(T, 4, H, device=dev, generator=g).bfloat16()
        post = torch.rand(T, 4, device=dev, generator=g) * 2
        comb = torch.rand(T, 4, 4, device=dev, generator=g)
        y = fc.gemm_allreduce_hc_post(a, w, resid, post, comb) if it == 0 else fc.allreduce_hc_post(part, resid, post, comb)
        ref = R.hc_post(part.cpu().float(), resid.cpu().float(), post.cpu(), comb.cpu())
        errs.append(float((y.cpu().float() - ref).abs().max() / ref.abs().max()))
torch.cuda.synchronize()
O.check_status("local multicast")
fc.mcbuf.close()
print(json.dumps({{"errs": errs}}))
"""

CASES = [("norm", 8, 1024, 512), ("norm", 64, 4096, 256), ("hc", 8, 1024, 512), ("hc", 48, 4096, 1024)]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c)))
def test_fused_allreduce_on_local_multicast(case):
    r = subprocess.run([sys.executable, "-c", CHILD.format(root=ROOT, case=case)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    errs = json.loads(r.stdout.strip().splitlines()[-1])["errs"]
    assert max(errs) < 2e-2, errs
