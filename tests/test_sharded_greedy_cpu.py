"""Sharded greedy top-1 over simulated vocab shards (world sizes 1/2/4/8), with
ties inside and across shards and negative logits: the max over shards of the
packed (value, ~id) keys equals the global argmax with the lowest-id tie break
(the reference's ``test_decode_sharded_lm_cpu.py:7-48`` semantics)."""
import pytest
import torch

from bwn import ops as O


def _sharded(logits, world):
    V = logits.shape[-1]
    per = V // world
    keys = torch.stack([O.argmax_packed(logits[:, r * per:(r + 1) * per], r * per) for r in range(world)])
    return O.unpack_argmax(keys.max(0).values)


def _lowest_argmax(logits):
    m = logits.max(-1, keepdim=True).values
    ids = torch.arange(logits.shape[-1]).expand_as(logits)
    return torch.where(logits == m, ids, torch.full_like(ids, 1 << 30)).min(-1).values.int()


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_sharded_greedy_ties(world):
    g = torch.Generator().manual_seed(world)
    V = 64
    logits = torch.randn(6, V, generator=g)
    logits[1] = -torch.rand(V, generator=g) - 1.0          # all negative
    logits[2, 5] = logits[2, 40] = logits[2].max() + 1.0    # tie across shards (when world > 1)
    logits[3, 17] = logits[3, 18] = logits[3].max() + 1.0   # tie inside one shard
    logits[4] = 0.0                                         # everything tied -> id 0
    logits[5, 63] = 100.0                                   # max in the last shard
    got = _sharded(logits, world)
    assert torch.equal(got, _lowest_argmax(logits)), (got, _lowest_argmax(logits))
