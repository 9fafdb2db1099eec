"""Temperature sampling by the Gumbel-max trick on the vocab-sharded head:
the empirical token distribution matches softmax(logits / T), rows at T = 0
are exactly greedy, and a vocab-sharded draw with the same noise equals the
unsharded one (each rank perturbs its own shard, one int64 max picks)."""
import torch

from bwn import ops as O
from bwn.config import tiny_qwen36
from bwn.models.qwen36 import build_qwen36
from bwn.ops import reference as R
from bwn.runtime.static_decode import StaticDecoder


def _gumbel_pick(logits, t, u):
    noisy = torch.where(t[:, None] > 0, logits / t[:, None].clamp_min(1e-6) - torch.log(-torch.log(u)), logits)
    return O.unpack_argmax(O.argmax_packed(noisy, 0)).long()


def test_gumbel_max_matches_softmax():
    g = torch.Generator().manual_seed(0)
    logits = torch.tensor([[2.0, 1.0, 0.5, -1.0, 0.0, 1.5, -0.5, 0.25]])
    T = 0.7
    n = 40000
    u = torch.rand(n, 8, generator=g).clamp_(1e-20, 1.0)
    picks = _gumbel_pick(logits.expand(n, 8), torch.full((n,), T), u)
    freq = torch.bincount(picks, minlength=8).float() / n
    p = torch.softmax(logits[0] / T, -1)
    assert (freq - p).abs().max() < 0.01, (freq, p)


def test_sharded_draw_equals_unsharded():
    g = torch.Generator().manual_seed(1)
    B, V, W = 5, 96, 4
    logits = torch.randn(B, V, generator=g) * 3
    u = torch.rand(B, V, generator=g).clamp_(1e-20, 1.0)
    t = torch.tensor([0.0, 0.5, 1.0, 2.0, 0.0])
    full = _gumbel_pick(logits, t, u)
    per = V // W
    keys = []
    for r in range(W):
        sl = slice(r * per, (r + 1) * per)
        noisy = torch.where(t[:, None] > 0, logits[:, sl] / t[:, None].clamp_min(1e-6) - torch.log(-torch.log(u[:, sl])),
                            logits[:, sl])
        keys.append(O.argmax_packed(noisy, r * per))
    sharded = O.unpack_argmax(torch.stack(keys).max(0).values).long()
    assert torch.equal(sharded, full)
    assert torch.equal(full[[0, 4]], R.sharded_greedy([logits[[0, 4], r * per:(r + 1) * per] for r in range(W)]).long())


def test_decoder_sampling_rows():
    cfg = tiny_qwen36()
    m = build_qwen36(cfg, seed=6, dtype=torch.float32)
    prompt = torch.randint(0, cfg.vocab, (3, 7), generator=torch.Generator().manual_seed(2))
    greedy = StaticDecoder(m, 3, 32, use_graph=False).generate(prompt, 6)
    d = StaticDecoder(m, 3, 32, use_graph=False, sampling=True, seed=5)
    d.temperature.copy_(torch.tensor([0.0, 1.0, 0.0]))
    out = d.generate(prompt, 6)
    assert torch.equal(out[0], greedy[0]) and torch.equal(out[2], greedy[2])  # T = 0 rows are greedy
    assert not torch.equal(out[1], greedy[1])  # the sampled row departs (fixed seed)
    d2 = StaticDecoder(m, 3, 32, use_graph=False, sampling=True, seed=5)
    d2.temperature.copy_(torch.tensor([0.0, 1.0, 0.0]))
    assert torch.equal(d2.generate(prompt, 6), out)  # reproducible from the seed
