"""Chunked gated delta rule numerics (the reference's inverse-stability and
pad-token tests, ``contrib/qwen3.6-35b-a3b/kernels/tests/test_dn_block_inverse_stability.py``,
``contrib/qwen3.6-27b/kernels/tests/test_pad_token_state.py``): the chunked
form (forward-substitution inverse per chunk) equals the token-by-token
recurrence across chunk sizes, including near-1 decay and beta near 1; pad rows
(g = beta = 0) leave the state untouched; prefill of a padded batch equals
prefill of each sequence alone."""
import pytest
import torch
import torch.nn.functional as F

from bwn.config import tiny_qwen36
from bwn.models.qwen36 import build_qwen36
from bwn.ops import reference as R


def _inputs(B, H, S, D, g_scale, beta_lo, seed=0):
    gen = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(B, H, S, D, generator=gen, dtype=torch.float64), dim=-1) * D ** -0.5
    k = F.normalize(torch.randn(B, H, S, D, generator=gen, dtype=torch.float64), dim=-1)
    v = torch.randn(B, H, S, D, generator=gen, dtype=torch.float64)
    g = -torch.rand(B, H, S, generator=gen, dtype=torch.float64) * g_scale   # log-decay <= 0
    beta = beta_lo + (1 - beta_lo) * torch.rand(B, H, S, generator=gen, dtype=torch.float64)
    return q.float(), k.float(), v.float(), g.float(), beta.float()


@pytest.mark.parametrize("chunk", [16, 32, 64])
@pytest.mark.parametrize("g_scale,beta_lo", [(1.0, 0.0), (1e-3, 0.9), (1e-6, 0.99), (5.0, 0.5)])
def test_chunked_equals_recurrent(chunk, g_scale, beta_lo):
    q, k, v, g, beta = _inputs(1, 2, 150, 32, g_scale, beta_lo)
    st0 = torch.randn(1, 2, 32, 32, generator=torch.Generator().manual_seed(9)) * 0.1
    o1, s1 = R.chunk_gated_delta_rule(q, k, v, g, beta, st0, chunk)
    o2, s2 = R.recurrent_gated_delta_rule(q, k, v, g, beta, st0)
    assert torch.isfinite(o1).all() and torch.isfinite(s1).all()
    scale = o2.abs().max().clamp_min(1.0)
    assert (o1 - o2).abs().max() / scale < 2e-3, (chunk, g_scale, beta_lo)
    assert (s1 - s2).abs().max() / s2.abs().max().clamp_min(1.0) < 2e-3


def test_pad_rows_leave_state_untouched():
    q, k, v, g, beta = _inputs(1, 2, 64, 32, 1.0, 0.0)
    n = 40
    g[..., n:] = 0.0
    beta[..., n:] = 0.0
    _, s_pad = R.chunk_gated_delta_rule(q, k, v, g, beta, None, 64)
    _, s_ref = R.recurrent_gated_delta_rule(q[..., :n, :], k[..., :n, :], v[..., :n, :], g[..., :n], beta[..., :n])
    assert (s_pad - s_ref).abs().max() < 1e-4


def test_padded_batch_prefill_equals_single_sequences():
    cfg = tiny_qwen36(layers=4)
    m = build_qwen36(cfg, device="cpu", dtype=torch.float32)
    gen = torch.Generator().manual_seed(2)
    lens = [9, 16, 5]
    S = max(lens)
    ids = torch.randint(0, cfg.vocab, (len(lens), S), generator=gen)
    st = m.new_state(len(lens), 32)
    h = m.prefill_hidden(ids, st, torch.tensor(lens, dtype=torch.int32))
    for i, n in enumerate(lens):
        st1 = m.new_state(1, 32)
        h1 = m.prefill_hidden(ids[i:i + 1, :n], st1)
        assert torch.allclose(h[i], h1[0], atol=1e-4), i
        assert torch.allclose(st.ssm[:, i], st1.ssm[:, 0], atol=1e-4), i
        assert int(st.positions[i]) == n
