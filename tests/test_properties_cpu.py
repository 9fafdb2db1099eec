"""Property tests (hypothesis) of the numeric invariants the kernels' CPU twins
rely on:

* packed greedy keys: for any logits (signs, ties, infinities) and any split
  into vocab shards, the int64 max over the shards' keys decodes to the
  largest logit with the lowest global id;
* fp8 block codec: dequantize(quantize(w)) stays within E4M3's relative step
  of each 128x128 block's scale, zeros stay zero, and FP8Experts keeps every
  row's own block scale through the gate/up interleave.
"""
import math

import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from bwn import ops as O
from bwn.io.fp8 import FP8Experts, dequantize_block, quantize_block

finite = st.floats(min_value=-2.0 ** 100, max_value=2.0 ** 100, allow_nan=False, allow_infinity=False, width=32)


@settings(max_examples=60, deadline=None)
@given(vals=st.lists(st.one_of(finite, st.sampled_from([0.0, -0.0, 1.5, -1.5, float("inf"), -float("inf")])),
                     min_size=2, max_size=64),
       shards=st.integers(min_value=1, max_value=8))
def test_packed_greedy_any_split(vals, shards):
    v = torch.tensor(vals, dtype=torch.float32)[None]
    V = v.shape[1]
    bounds = sorted({0, V, *[(V * i) // shards for i in range(1, shards)]})
    keys = [O.argmax_packed(v[:, a:b], a) for a, b in zip(bounds, bounds[1:]) if b > a]
    got = int(O.unpack_argmax(torch.stack(keys).max(0).values)[0])
    best = v[0].max()
    want = int(torch.nonzero(v[0] == best)[0, 0])
    assert got == want, (vals, shards, got, want)


@settings(max_examples=40, deadline=None)
@given(rows=st.integers(1, 300), cols=st.integers(1, 300), scale=st.floats(1e-4, 1e3), seed=st.integers(0, 10_000))
def test_fp8_block_roundtrip_bound(rows, cols, scale, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(rows, cols, generator=g) * scale
    w[0, 0] = 0.0
    w8, s = quantize_block(w)
    d = dequantize_block(w8, s)
    assert d[0, 0] == 0.0
    # E4M3: 3 mantissa bits -> |error| <= 2^-4 * |value| for normals, plus the
    # subnormal spacing 2^-9 of the block scale
    se = s.repeat_interleave(128, 0).repeat_interleave(128, 1)[:rows, :cols]
    assert bool(((d - w).abs() <= w.abs() * 2 ** -4 + se * 2 ** -9 + 1e-30).all())


@settings(max_examples=25, deadline=None)
@given(E=st.integers(1, 3), I16=st.integers(1, 12), K=st.integers(1, 260), seed=st.integers(0, 10_000))
def test_fp8_experts_interleave_keeps_row_scales(E, I16, K, seed):
    g = torch.Generator().manual_seed(seed)
    I = 16 * I16
    gate = torch.randn(E, I, K, generator=g) * torch.rand(E, I, 1, generator=g) * 10
    up = torch.randn(E, I, K, generator=g)
    fx = FP8Experts.quantize_gate_up(gate, up)
    d = fx.dequant()
    x = d.reshape(E, I // 16, 2, 16, K)
    dg, du = x[:, :, 0].reshape(E, I, K), x[:, :, 1].reshape(E, I, K)
    for e in range(E):
        g8, gs = quantize_block(gate[e])
        u8, us = quantize_block(up[e])
        assert torch.equal(dg[e], dequantize_block(g8, gs))
        assert torch.equal(du[e], dequantize_block(u8, us))
    assert fx.scales16.shape == (E, 2 * I // 16, math.ceil(K / 128))


def test_signed_zero_maxima_tie_across_shards():
    """-0.0 and +0.0 are equal logits: the lowest id wins, whichever shard holds it."""
    ka = O.argmax_packed(torch.tensor([[-0.0, -1.0]]), 0)
    kb = O.argmax_packed(torch.tensor([[0.0, -2.0]]), 5)
    assert int(O.unpack_argmax(torch.stack([ka, kb]).max(0).values)[0]) == 0
    assert int(O.unpack_argmax(O.argmax_packed(torch.tensor([[-1.0, -0.0, 0.0]]), 0))[0]) == 1


@settings(max_examples=20, deadline=None)
@given(S=st.integers(1, 40), chunk=st.sampled_from([4, 8, 16]), g_scale=st.sampled_from([1e-4, 0.3, 3.0]),
       seed=st.integers(0, 10_000))
def test_chunked_delta_rule_equals_recurrent(S, chunk, g_scale, seed):
    import torch.nn.functional as F

    from bwn.ops import reference as R
    gen = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(1, 2, S, 16, generator=gen, dtype=torch.float64), dim=-1).float() * 0.25
    k = F.normalize(torch.randn(1, 2, S, 16, generator=gen, dtype=torch.float64), dim=-1).float()
    v = torch.randn(1, 2, S, 8, generator=gen)
    g = -torch.rand(1, 2, S, generator=gen) * g_scale
    beta = torch.rand(1, 2, S, generator=gen)
    s0 = torch.randn(1, 2, 16, 8, generator=gen) * 0.1
    o1, s1 = R.chunk_gated_delta_rule(q, k, v, g, beta, s0, chunk)
    o2, s2 = R.recurrent_gated_delta_rule(q, k, v, g, beta, s0)
    assert torch.allclose(o1, o2, atol=2e-4, rtol=1e-3) and torch.allclose(s1, s2, atol=2e-4, rtol=1e-3)


@settings(max_examples=20, deadline=None)
@given(T=st.integers(1, 12), E=st.integers(2, 12), k=st.integers(1, 4), seed=st.integers(0, 10_000))
def test_sparse_moe_equals_masked_dense(T, E, k, seed):
    import torch.nn.functional as F

    from bwn.ops import reference as R
    k = min(k, E)
    gen = torch.Generator().manual_seed(seed)
    H, I = 16, 8
    x = torch.randn(T, H, generator=gen)
    w, ids = R.moe_route_softmax(torch.randn(T, E, generator=gen), k)
    gu = torch.randn(E, 2 * I, H, generator=gen) * 0.2
    dn = torch.randn(E, H, I, generator=gen) * 0.2
    dense = torch.zeros(T, E).scatter_add_(1, ids.long(), w)
    gg, uu = torch.einsum("th,eih->eti", x, gu).chunk(2, dim=-1)
    ref = torch.einsum("te,eth->th", dense, torch.einsum("eti,ehi->eth", F.silu(gg) * uu, dn))
    assert torch.allclose(R.moe_experts(x, w, ids, gu, dn), ref, atol=1e-5)


@settings(max_examples=50, deadline=None)
@given(B=st.integers(1, 4), N=st.integers(2, 6), vocab=st.integers(2, 5), seed=st.integers(0, 10_000))
def test_accept_greedy_matches_a_plain_loop(B, N, vocab, seed):
    """Accepted drafts = the longest prefix of drafts equal to the target's
    greedy ids; emitted = those drafts then the target's next id."""
    from bwn.runtime.spec_decode import accept_greedy
    gen = torch.Generator().manual_seed(seed)
    tok = torch.randint(0, vocab, (B, N), generator=gen)
    tgt = torch.randint(0, vocab, (B, N), generator=gen)
    m, bonus, out = accept_greedy(tok, tgt)
    for b in range(B):
        mm = 0
        while mm < N - 1 and int(tok[b, mm + 1]) == int(tgt[b, mm]):
            mm += 1
        emitted = [int(t) for t in tok[b, 1:mm + 1]] + [int(tgt[b, mm])]
        assert int(m[b]) == mm and int(bonus[b]) == int(tgt[b, mm])
        assert out[b, :mm + 1].tolist() == emitted and (out[b, mm + 1:] == -1).all()
