"""bwn's Qwen3.6-35B-A3B decode against the reference's own harness code.

The reference (installed under ``baseline/_ref``; skipped when absent) is run
unmodified through ``load_sharded_weights`` + ``StaticDecode35B.decode_step``
(``contrib/qwen3.6-35b-a3b/static_decode_35b.py:2682, 836, 1532``) on CPU in
fp32, with the same synthetic HF-layout weights bwn initialises from seed 0
(served to the reference's loader by ``bench/reference_arm.py``).  Two decode
steps from a zero state must give the same logits as bwn's CPU path.
"""
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "bench"))

import reference_arm as RA  # noqa: E402

pytestmark = pytest.mark.skipif(not os.path.isfile(os.path.join(RA.REF_DIR, "static_decode_35b.py")),
                                reason="reference not installed under baseline/_ref")


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def test_decode_matches_reference_harness():
    from bwn.config import tiny_qwen36
    from bwn.models.qwen36 import build_qwen36
    cfg = tiny_qwen36(moe=True, layers=4)
    mod, st = RA.build_reference(cfg, 0, 1, 2, 64, torch.device("cpu"), dtype=torch.float32)
    m = build_qwen36(cfg, seed=0, dtype=torch.float32)
    s = m.new_state(2, 64)
    ids = torch.tensor([5, 17])
    state = [st["dn"], st["conv"], st["k"], st["v"]]
    with torch.no_grad():
        for step in range(2):
            logits, nxt, *state = mod.decode_step(ids, torch.tensor(step), *state)
            ours = m.logits(m.decode_hidden(ids.int(), s))
            assert _rel(ours, logits) < 1e-4, step
            assert torch.equal(ours.argmax(-1), nxt)
            ids = nxt
