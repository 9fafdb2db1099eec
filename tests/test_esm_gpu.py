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
