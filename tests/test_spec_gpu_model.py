"""EAGLE3 speculative decoding on the GPU (tiny Qwen3.6 target, CUDA graph):
the emitted tokens equal plain greedy decoding, with a random draft and with
an all-accepting oracle draft."""
import pytest
import torch

from bwn.config import tiny_qwen36
from bwn.models.eagle3 import Eagle3Draft, eagle3_config
from bwn.models.qwen36 import build_qwen36
from bwn.ops import check_status
from bwn.runtime.spec_decode import SpecDecoder

pytestmark = pytest.mark.gpu
dev = torch.device("cuda", 0)


def _plain(model, prompt, n):
    st = model.new_state(prompt.shape[0], prompt.shape[1] + n + 16)
    tok = model.prefill(prompt.to(dev), st)
    out = [tok]
    for _ in range(n - 1):
        tok = model.decode_step(tok, st)
        out.append(tok)
    return torch.stack(out, 1).cpu()


@pytest.mark.parametrize("oracle", [False, True])
def test_spec_decode_gpu_matches_plain(oracle):
    cfg = tiny_qwen36(layers=4)
    target = build_qwen36(cfg, device=dev)
    draft = Eagle3Draft(eagle3_config(cfg, draft_vocab=256), dev).init_random(1)
    prompt = torch.randint(0, cfg.vocab, (2, 16), generator=torch.Generator().manual_seed(4))
    want = _plain(target, prompt, 20)
    sd = SpecDecoder(target, draft, 2, 128, num_draft=4, use_graph=True)
    if oracle:
        sd.set_oracle(want, prompt.shape[1])
    g0 = sd.prefill(prompt)
    sd.capture()
    res = [[int(x)] for x in g0.cpu()]
    while min(len(r) for r in res) < 16:
        ids, cnt = sd.step()
        for b in range(2):
            res[b].extend(int(x) for x in ids[b, :int(cnt[b])])
    check_status("spec decode")
    got = torch.tensor([r[:16] for r in res])
    assert torch.equal(got, want[:, :16]), (got, want[:, :16])
    if oracle:
        assert sd.mean_accepted() > 3.5
    sd.release()
