"""ESM-2 MLM training on the GPU (bf16 tcgen05 GEMMs fwd+bwd, fp32 master)
against the fp32 CPU path of the same weights and batch."""
import pytest
import torch

from bwn.config import ESM2_SIZES
from bwn.models.esm2 import EsmForMaskedLM, mlm_loss
from bwn.train.esm_mlm import MLMConfig, MLMTrainer, mask_tokens, synthetic_batch

pytestmark = pytest.mark.gpu


def test_esm_loss_and_grads_match_cpu():
    cfg = ESM2_SIZES["8M"]
    cpu = EsmForMaskedLM(cfg).init_weights(0)
    gpu = EsmForMaskedLM(cfg).init_weights(0).cuda()
    gen = torch.Generator().manual_seed(0)
    ids, am = synthetic_batch(cfg, 8, 256, gen)
    ids, labels, lm = mask_tokens(ids, cfg, gen)
    lc = mlm_loss(cpu(ids, am), labels, lm)
    lg = mlm_loss(gpu(ids.cuda(), am.cuda()), labels.cuda(), lm.cuda())
    lc.backward()
    lg.backward()
    assert abs(lc.item() - lg.item()) < 2e-2 * abs(lc.item())
    for (n, pc), (_, pg) in zip(cpu.named_parameters(), gpu.named_parameters()):
        if pc.grad is None:
            continue
        rel = (pg.grad.cpu() - pc.grad).norm() / (pc.grad.norm() + 1e-8)
        assert rel < 0.1, (n, float(rel))


def test_esm_gpu_training_steps():
    cfg = ESM2_SIZES["8M"]
    model = EsmForMaskedLM(cfg).init_weights(0).cuda()
    tr = MLMTrainer(model, MLMConfig(batch=8, seq_len=256, lr=1e-3, warmup=1, total_steps=20, loss_divisor="masked"))
    losses = [float(tr.step()) for _ in range(12)]
    assert all(l == l for l in losses)
    assert min(losses[-4:]) < losses[0]


@pytest.mark.parametrize("D", [64, 128])
def test_rope_half_kernel_matches_fp32(D):
    """The fused rotary + scale + transpose kernel, both directions, against the
    fp32 PyTorch formula (HF ``x*cos + rotate_half(x)*sin``)."""
    from bwn import ops as O
    from bwn.models.esm2 import _rotate_half
    B, S, H = 2, 300, 5
    x = torch.randn(B * S, H * D, device="cuda").bfloat16()
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device="cuda").float() / D))
    f = torch.outer(torch.arange(S, device="cuda").float(), inv)
    cos, sin = f.cos().contiguous(), f.sin().contiguous()
    y = O.rope_half(x, cos, sin, B, S, H, True, 1.0, D ** -0.5)
    xs = x.float().view(B, S, H, D).transpose(1, 2)
    emb = torch.cat([f, f], -1)
    ref = (xs * emb.cos() + _rotate_half(xs) * emb.sin()) * D ** -0.5
    assert ((y.float() - ref).norm() / ref.norm()).item() < 1e-2
    g = torch.randn(B, H, S, D, device="cuda").bfloat16()
    xr = xs.clone().requires_grad_(True)
    ((xr * emb.cos() + _rotate_half(xr) * emb.sin()) * D ** -0.5).backward(g.float())
    gx = O.rope_half(g, cos, sin, B, S, H, False, -1.0, D ** -0.5)
    gref = xr.grad.transpose(1, 2).reshape(B * S, H * D)
    assert ((gx.float() - gref).norm() / gref.norm()).item() < 1e-2
