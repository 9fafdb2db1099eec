"""Speculative verify bookkeeping (CPU oracle): after any sequence of
(verify N tokens, accept a of them) steps, the outputs of the accepted rows and
the committed recurrent state equal a plain token-by-token decode over exactly
the accepted stream -- the invariant of the reference's rollback test
(contrib/qwen3.6-27b/kernels/tests/test_deltanet_spec_verify_rollback.py)."""
import pytest
import torch

from bwn.ops import reference as R
from _spec_util import dn_params, dn_rows


@pytest.mark.parametrize("N,seed", [(4, 0), (5, 1), (2, 2)])
def test_deltanet_verify_deferred_commit_matches_sequential(N, seed):
    KH, VH, B = 1, 2, 2
    P = dn_params(KH, VH, "cpu", seed)
    C = P["C"]
    gen = torch.Generator().manual_seed(100 + seed)
    ring = torch.zeros(B, 8, C).bfloat16()
    state = torch.zeros(B, VH, 128, 128)
    stash_qkv = torch.zeros(2, B, N, C).bfloat16()
    stash_ab = torch.zeros(2, B, N, 2 * VH).bfloat16()
    vstep = torch.zeros(1, dtype=torch.int32)
    pos = torch.zeros(B, dtype=torch.int32)
    pending = torch.zeros(B, dtype=torch.int32)
    # plain decoder over the accepted stream
    ring_s, state_s = ring.clone(), state.clone()
    pos_s = torch.zeros(B, dtype=torch.int32)
    for step in range(6):
        qkv, z, a, b = dn_rows(B * N, KH, VH, "cpu", gen)
        out = R.deltanet_verify(qkv, z, a, b, stash_qkv, stash_ab, vstep, ring, state, pos, pending, P["conv_w"],
                                P["A_log"], P["dt_bias"], P["norm_w"], KH, N)
        acc = torch.randint(1, N + 1, (B,), generator=gen)
        for bi in range(B):
            for i in range(int(acc[bi])):
                r = bi * N + i
                ref = R.deltanet_decode(qkv[r][None], a[r][None], b[r][None], z[r][None], ring_s[bi:bi + 1],
                                        state_s[bi:bi + 1], pos_s[bi:bi + 1], P["conv_w"], P["A_log"],
                                        P["dt_bias"], P["norm_w"], KH, 128, 128)
                assert torch.allclose(out[r].float(), ref[0].float(), atol=1e-2, rtol=1e-2), (step, bi, i)
                pos_s[bi] += 1
        pos += acc.int()
        pending.copy_(acc)
        vstep += 1
    # final commit only
    empty = torch.zeros(0, C).bfloat16()
    R.deltanet_verify(empty, torch.zeros(0, VH * 128).bfloat16(), torch.zeros(0, VH).bfloat16(),
                      torch.zeros(0, VH).bfloat16(), stash_qkv, stash_ab, vstep, ring, state, pos, pending,
                      P["conv_w"], P["A_log"], P["dt_bias"], P["norm_w"], KH, 0)
    assert torch.allclose(state, state_s, atol=1e-5)
    assert torch.equal(pos, pos_s)
