"""Model-level GPU tests: the full decode step through the bwn kernels (and its
CUDA-graph replay) against the CPU reference path of the same weights."""
import pytest
import torch

from bwn.config import tiny_qwen36
from bwn.io import qwen36_weights as W
from bwn.models.qwen36 import build_qwen36
from bwn.ops import check_status
from bwn.runtime.static_decode import StaticDecoder

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-9)).item()


@pytest.mark.parametrize("moe", [False])
def test_decode_matches_cpu(moe):
    cfg = tiny_qwen36(moe=moe)
    hf = dict(W.synthetic_hf_globals(cfg, 7, "cpu"))
    for i in range(cfg.num_layers):
        hf.update(W.synthetic_hf_layer(cfg, i, 7, "cpu"))
    g = build_qwen36(cfg, device="cuda", hf_state=hf)
    c = build_qwen36(cfg, device="cpu", hf_state=hf, dtype=torch.float32)
    B = 3
    sg, sc = g.new_state(B, 64), c.new_state(B, 64)
    # start from an identical non-trivial state
    torch.manual_seed(0)
    for name in ("conv", "ssm"):
        t = torch.randn_like(getattr(sc, name)) * 0.1
        getattr(sc, name).copy_(t)
        getattr(sg, name).copy_(t.to(getattr(sg, name).dtype).cuda())
    kv = torch.randn_like(sc.k_cache)
    sc.k_cache.copy_(kv); sg.k_cache.copy_(kv.bfloat16().cuda())
    sc.v_cache.copy_(kv * 0.5); sg.v_cache.copy_((kv * 0.5).bfloat16().cuda())
    sc.positions.fill_(9); sg.positions.fill_(9)
    tok = torch.tensor([3, 100, 511], dtype=torch.int32)
    for _ in range(3):
        hg = g.decode_hidden(tok.cuda(), sg)
        hc = c.decode_hidden(tok, sc)
        torch.cuda.synchronize()
        check_status("decode")
        assert _rel(hg.cpu(), hc) < 5e-2
        lg, lc = g.logits(hg), c.logits(hc)
        assert _rel(lg.cpu(), lc) < 5e-2
        tok = lc.argmax(-1).int()
    assert sg.positions.tolist() == [12, 12, 12]


def test_graph_replay_equals_eager():
    cfg = tiny_qwen36()
    m = build_qwen36(cfg, device="cuda", seed=1)
    d1 = StaticDecoder(m, 2, 64, use_graph=True)
    d2 = StaticDecoder(m, 2, 64, use_graph=False)
    d1.capture()
    for d in (d1, d2):
        d.st.positions.fill_(4)
        d.tokens.copy_(torch.tensor([5, 6], dtype=torch.int32, device="cuda"))
    outs1, outs2 = [], []
    for _ in range(4):
        d1.step_device(); outs1.append(d1.next_ids.clone())
        d2.step_device(); outs2.append(d2.next_ids.clone())
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(outs1, outs2))
    assert torch.allclose(d1.st.ssm, d2.st.ssm, atol=1e-3)
    # host API: H2D of the tokens, D2H of the ids
    out = d1.step(torch.tensor([7, 8], dtype=torch.int32))
    assert out.shape == (2,) and out.dtype == torch.int32


def test_every_layer_state_changes_every_step_on_gpu():
    """The kernels' decode step writes every per-layer state slice each step
    (DeltaNet recurrent state and conv-ring slot, K/V row at the position)."""
    from bwn.utils import fingerprint as F
    cfg = tiny_qwen36()
    m = build_qwen36(cfg, device="cuda", seed=5)
    st = m.new_state(4, 32)
    tok = torch.tensor([1, 5, 9, 11], dtype=torch.int32, device="cuda")
    for _ in range(3):
        snap = F.snapshot_state(st)
        tok = m.decode_step(tok, st).int()
        torch.cuda.synchronize()
        check_status("decode")
        F.assert_state_advanced(snap, st)
