"""The decode-sized MoE block in four launches (``csrc/kernels/moe_decode.cu``:
fused routing + gather, the shared expert folded into the grouped GEMMs, the
combine fused with the residual add + RMSNorm) against the twelve-launch path
it replaces and against the fp32 PyTorch path on the CPU (same weights)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _models(cfg):
    from bwn.models.qwen36 import Qwen36Model
    gpu = Qwen36Model(cfg, None, torch.device("cuda")).init_random(0, gen_device="cpu")
    cpu = Qwen36Model(cfg, None, "cpu", dtype=torch.float32).init_random(0)
    return gpu, cpu


def _inputs(cfg, T, seed=0):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(T, cfg.hidden, generator=g).bfloat16()
    x = torch.randn(T, cfg.hidden, generator=g).bfloat16()
    return h, x


@pytest.mark.parametrize("moe,layers,T", [(True, 4, 7), (True, 4, 32), ("35b", 1, 32)])
def test_fused_moe_decode_matches_unfused_and_cpu(moe, layers, T):
    from bwn.config import QWEN36_35B_A3B, tiny_qwen36
    cfg = QWEN36_35B_A3B.scaled(num_layers=layers) if moe == "35b" else tiny_qwen36(moe=True, layers=layers)
    gpu, cpu = _models(cfg)
    i = 0
    assert "experts_gate_up_x" in gpu.layers[i] and gpu._moe_decode_ok(i, torch.zeros(T, cfg.hidden, device="cuda"))
    h, x = _inputs(cfg, T)
    nxt_g = gpu.layers[min(i + 1, layers - 1)]["in_norm"]
    dev = torch.device("cuda")
    for rep in range(2):  # the second call re-uses the barrier words and the graph-free scratch
        x1, x2 = x.to(dev).clone(), x.to(dev).clone()
        fused = gpu._moe_decode(i, h.to(dev), x1, nxt_g)
        ref = gpu._reduce_add_norm(gpu._mlp(i, h.to(dev)), x2, nxt_g)
        torch.cuda.synchronize()
        from bwn.ops import check_status
        check_status("moe_decode")
        assert _rel(x1, x2) < 1e-2, rep
        assert _rel(fused, ref) < 2e-2, rep
    xc = x.float().clone()
    out_c = cpu._reduce_add_norm(cpu._mlp(i, h.float()), xc, cpu.layers[min(i + 1, layers - 1)]["in_norm"])
    assert _rel(fused.cpu(), out_c) < 3e-2
    assert _rel(x1.cpu(), xc) < 2e-2


def test_fused_moe_decode_fp8_experts():
    from bwn.config import tiny_qwen36
    cfg = tiny_qwen36(moe=True, layers=4)
    from bwn.models.qwen36 import Qwen36Model
    gpu = Qwen36Model(cfg, None, torch.device("cuda")).init_random(0)
    gpu.quantize_fp8(include_head=False, experts=True, dense=False)
    i, T = 0, 24
    assert hasattr(gpu.layers[i]["experts_gate_up_x"], "w8")  # shared expert folded into the fp8 stack
    h, x = _inputs(cfg, T, seed=3)
    dev = torch.device("cuda")
    x1, x2 = x.to(dev).clone(), x.to(dev).clone()
    nxt = gpu.layers[1]["in_norm"]
    fused = gpu._moe_decode(i, h.to(dev), x1, nxt)
    ref = gpu._reduce_add_norm(gpu._mlp(i, h.to(dev)), x2, nxt)
    torch.cuda.synchronize()
    assert _rel(fused, ref) < 2e-2 and _rel(x1, x2) < 1e-2


@pytest.mark.parametrize("moe", ["tiny", "35b"])
def test_fused_moe_decode_exact_ties_pick_lowest_id(moe):
    """Duplicated router rows give bit-equal logits: the fused top-k must pick
    the lower expert id, as the unfused router does, or the expert rows
    (different weights for the duplicate) change the output."""
    from bwn.config import QWEN36_35B_A3B, tiny_qwen36
    cfg = QWEN36_35B_A3B.scaled(num_layers=2) if moe == "35b" else tiny_qwen36(moe=True, layers=4)
    from bwn.models.qwen36 import Qwen36Model
    gpu = Qwen36Model(cfg, None, torch.device("cuda")).init_random(0)
    i, T = 0, 16
    L = gpu.layers[i]
    E = cfg.num_experts
    L["router"][E // 2:].copy_(L["router"][:E // 2])
    L["router_x"][E // 2:E].copy_(L["router_x"][:E // 2])  # the fused path's copy (+ the shared gate row)
    h, x = _inputs(cfg, T, seed=5)
    dev = torch.device("cuda")
    x1, x2 = x.to(dev).clone(), x.to(dev).clone()
    nxt = gpu.layers[1]["in_norm"]
    fused = gpu._moe_decode(i, h.to(dev), x1, nxt)
    ref = gpu._reduce_add_norm(gpu._mlp(i, h.to(dev)), x2, nxt)
    torch.cuda.synchronize()
    assert _rel(fused, ref) < 2e-2 and _rel(x1, x2) < 1e-2
