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


# ---------------------------------------------------------------------------
# model level: greedy speculative decoding == plain greedy decoding
# ---------------------------------------------------------------------------
from bwn.config import tiny_qwen36  # noqa: E402
from bwn.models.eagle3 import Eagle3Draft, eagle3_config  # noqa: E402
from bwn.models.qwen36 import build_qwen36  # noqa: E402
from bwn.runtime.spec_decode import SpecDecoder, accept_greedy  # noqa: E402


def test_accept_greedy():
    tok = torch.tensor([[5, 7, 9, 11], [5, 7, 9, 11], [5, 1, 9, 11]])
    tgt = torch.tensor([[7, 9, 11, 13], [7, 8, 11, 13], [7, 9, 11, 13]])
    m, bonus, out = accept_greedy(tok, tgt)
    assert m.tolist() == [3, 1, 0]
    assert bonus.tolist() == [13, 8, 7]
    assert out.tolist() == [[7, 9, 11, 13], [7, 8, -1, -1], [7, -1, -1, -1]]


def _plain_greedy(model, prompt, n):
    st = model.new_state(prompt.shape[0], prompt.shape[1] + n + 16)
    tok = model.prefill(prompt, st)
    out = [tok]
    for _ in range(n - 1):
        tok = model.decode_step(tok, st)
        out.append(tok)
    return torch.stack(out, 1)


class _OracleDraft(SpecDecoder):
    """Drafts the known greedy continuation, corrupted at random positions."""

    def __init__(self, *a, truth=None, corrupt=0.0, seed=0, **k):
        super().__init__(*a, **k)
        self.truth, self.corrupt = truth, corrupt
        self.g = torch.Generator().manual_seed(seed)

    def _draft_from(self, r, d1, pos0):
        S = self.S
        for b in range(self.B):
            for j in range(self.K):
                i = int(pos0[b]) - S + 1 + j  # index into the generated continuation
                v = int(self.truth[b, i]) if 0 <= i < self.truth.shape[1] else 0
                if torch.rand(1, generator=self.g).item() < self.corrupt:
                    v = (v + 1) % 512
                self.tok[b, j + 1] = v


@pytest.mark.parametrize("moe", [False, True])
def test_spec_decode_matches_plain_greedy_random_draft(moe):
    cfg = tiny_qwen36(moe=moe, layers=4)
    target = build_qwen36(cfg, device="cpu", dtype=torch.float32)
    draft = Eagle3Draft(eagle3_config(cfg, draft_vocab=256), "cpu", torch.float32).init_random(1)
    prompt = torch.randint(0, cfg.vocab, (2, 12), generator=torch.Generator().manual_seed(4))
    want = _plain_greedy(target, prompt, 10)
    sd = SpecDecoder(target, draft, 2, 64, num_draft=4, use_graph=False)
    got = sd.generate(prompt, 10)
    assert got == want.tolist()


@pytest.mark.parametrize("corrupt", [0.0, 0.35])
def test_spec_decode_with_accepting_drafts(corrupt):
    cfg = tiny_qwen36(layers=4)
    target = build_qwen36(cfg, device="cpu", dtype=torch.float32)
    draft = Eagle3Draft(eagle3_config(cfg, draft_vocab=256), "cpu", torch.float32).init_random(1)
    prompt = torch.randint(0, cfg.vocab, (2, 9), generator=torch.Generator().manual_seed(8))
    want = _plain_greedy(target, prompt, 24)
    sd = _OracleDraft(target, draft, 2, 80, num_draft=4, use_graph=False, truth=want, corrupt=corrupt)
    sd.S = prompt.shape[1]
    got = sd.generate(prompt, 18)
    assert got == want[:, :18].tolist()
    if corrupt == 0.0:
        assert sd.mean_accepted() > 3.0  # every draft accepted (4 per step) until the end
    # after committing, plain decode continues the same sequence
    sd.finish()
    assert int(sd.sp.pending.sum()) == 0
