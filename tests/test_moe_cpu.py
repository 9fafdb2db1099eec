"""MoE formulation equivalence on CPU (the reference's ``test_moe_oracle_cpu.py``,
``test_moe_sparse_eq.py`` and ``test_moe_decode_tp_cpu.py`` tier): the
masked-dense formulation, the sparse per-expert gather, bwn's fused-layer MoE
block and HF ``Qwen3_5MoeSparseMoeBlock`` agree, and the expert-parallel
partials of world sizes 1/2/4/8 (simulated by looping over ranks) sum to the
full block; plus the router semantics of both model families."""
from dataclasses import replace

import pytest
import torch
import torch.nn.functional as F

from bwn import ops as O
from bwn.config import tiny_qwen36
from bwn.ops import reference as R


def _hf_block(cfg, seed=0):
    from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as M
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    hc = Qwen3_5MoeTextConfig(hidden_size=cfg.hidden, num_experts=cfg.num_experts, num_experts_per_tok=cfg.top_k,
                              moe_intermediate_size=cfg.moe_inter,
                              shared_expert_intermediate_size=cfg.shared_inter)
    torch.manual_seed(seed)
    blk = M.Qwen3_5MoeSparseMoeBlock(hc).eval()
    with torch.no_grad():
        for p in blk.parameters():
            p.normal_(0, 0.05)
    return blk


def _masked_dense(x, w, ids, gate_up, down):
    """Every expert on every token, weighted by the dense [T, E] routing matrix."""
    T, E = x.shape[0], gate_up.shape[0]
    dense = torch.zeros(T, E).scatter_add_(1, ids.long(), w.float())
    g, u = torch.einsum("th,eih->eti", x.float(), gate_up.float()).chunk(2, dim=-1)
    y = torch.einsum("eti,ehi->eth", F.silu(g) * u, down.float())
    return torch.einsum("te,eth->th", dense, y)


def _layer_state(blk, cfg):
    """HF-layout layer 0 (random attention weights) whose MoE block is ``blk``."""
    from bwn.io import qwen36_weights as W
    sd = W.synthetic_hf_layer(cfg, 0, 0, "cpu")
    sd.update({f"layers.0.mlp.{k}": v.detach().clone() for k, v in blk.state_dict().items()})
    return sd


def test_router_matches_hf():
    cfg = tiny_qwen36(moe=True)
    blk = _hf_block(cfg)
    x = torch.randn(20, cfg.hidden)
    _, w_hf, ids_hf = blk.gate(x)
    w, ids = R.moe_route_softmax(x @ blk.gate.weight.detach().t(), cfg.top_k, True)
    assert torch.equal(ids.long(), ids_hf)
    assert torch.allclose(w, w_hf, atol=1e-6)
    assert torch.allclose(w.sum(-1), torch.ones(20), atol=1e-6)


def test_formulations_agree_with_hf_block():
    cfg = tiny_qwen36(moe=True)
    blk = _hf_block(cfg)
    T = 24
    x = torch.randn(T, cfg.hidden)
    with torch.no_grad():
        ref = blk(x[None])[0]
        _, w, ids = blk.gate(x)
    gu, dn = blk.experts.gate_up_proj.detach(), blk.experts.down_proj.detach()
    routed_sparse = R.moe_experts(x, w, ids.int(), gu, dn)
    routed_dense = _masked_dense(x, w, ids, gu, dn)
    assert torch.allclose(routed_sparse, routed_dense, atol=1e-5)
    with torch.no_grad():
        shared = torch.sigmoid(blk.shared_expert_gate(x)) * blk.shared_expert(x)
    assert torch.allclose(routed_sparse + shared, ref, atol=1e-5)
    # the fused CPU path on the interleaved gate/up layout the kernels use
    gu_il = torch.stack([O.interleave_gate_up(gu[e, :cfg.moe_inter], gu[e, cfg.moe_inter:])
                         for e in range(cfg.num_experts)])
    fused = O.moe_experts(x, w, ids.int(), gu_il, dn)
    assert torch.allclose(fused.float(), routed_sparse, atol=1e-5)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_expert_parallel_partials_sum_to_block(world):
    """Each simulated rank builds its own layer shard (``E/world`` experts, a
    ``1/world`` slice of the shared expert) through the model's weight fusion
    and runs the model's MoE block; the partials sum to HF's block."""
    from bwn.models.moe import qwen_moe_forward
    from bwn.models.qwen36 import Qwen36Model
    from bwn.io import qwen36_weights as W
    from bwn.parallel.comm import Comm
    # head counts and the shared expert split over 8 ranks (16-row gate/up blocks)
    cfg = replace(tiny_qwen36(moe=True), dn_k_heads=8, dn_v_heads=16, q_heads=8, shared_inter=128)
    blk = _hf_block(cfg, seed=1)
    sd = _layer_state(blk, cfg)
    x = torch.randn(16, cfg.hidden)
    with torch.no_grad():
        ref = blk(x[None])[0]
    total = torch.zeros_like(ref)
    held = []
    for r in range(world):
        m = Qwen36Model(cfg, Comm(None, r, world), "cpu", torch.float32)
        L = W.fuse_layer(cfg, 0, W.hf_getter(sd), world, r, torch.float32)
        held.append((m.d.expert_offset, L["experts_gate_up"].shape[0]))
        total += qwen_moe_forward(m, L, x).float()
    assert torch.allclose(total, ref, atol=1e-5), (total - ref).abs().max()
    # the ranks' expert ranges tile [0, E) exactly once
    assert held == [(r * cfg.num_experts // world, cfg.num_experts // world) for r in range(world)]


def test_gate_up_interleave_roundtrip():
    g, u = torch.randn(64, 32), torch.randn(64, 32)
    il = O.interleave_gate_up(g, u)
    assert il.shape == (128, 32)
    # 16-row blocks alternate gate / up, so a 32-wide output tile holds matching pairs
    assert torch.equal(il[:16], g[:16]) and torch.equal(il[16:32], u[:16])
    g2, u2 = O.deinterleave_gate_up(il)
    assert torch.equal(g2, g) and torch.equal(u2, u)


def test_deepseek_router_bias_only_selects():
    torch.manual_seed(0)
    T, E, k = 12, 32, 6
    logits = torch.randn(T, E)
    bias = torch.zeros(E)
    bias[5] = 100.0  # expert 5 is always selected ...
    w, ids = R.moe_route_deepseek(logits, bias, k, "sqrtsoftplus", 1.5)
    assert (ids == 5).any(-1).all()
    # ... but weighted by its unbiased score
    s = F.softplus(logits).sqrt()
    sel = s.gather(1, ids.long())
    assert torch.allclose(w, sel / sel.sum(-1, keepdim=True) * 1.5, atol=1e-6)
    assert torch.allclose(w.sum(-1), torch.full((T,), 1.5), atol=1e-5)
    w2, ids2 = R.moe_route_deepseek(logits, None, k, "sigmoid", 1.0)
    assert torch.equal(ids2.long(), torch.topk(logits.sigmoid(), k, -1).indices)


def test_swiglu_limit_clamps_both_halves():
    gu = torch.tensor([[10.0, -10.0, 10.0, -10.0]])  # gate (10, -10), up (10, -10)
    out = R.swiglu(gu, limit=7.0)
    g = torch.tensor([7.0, -10.0])
    u = torch.tensor([7.0, -7.0])
    assert torch.allclose(out[0], F.silu(g) * u)
    assert torch.allclose(R.swiglu(gu), F.silu(gu[0, :2]) * gu[0, 2:])


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_experts_sum_to_block(world):
    """``moe_sharding="tp"``: every simulated rank holds all experts with a
    ``1/world`` slice of their intermediate width; the partials sum to HF's block."""
    from bwn.io import qwen36_weights as W
    from bwn.models.moe import qwen_moe_forward
    from bwn.models.qwen36 import Qwen36Model
    from bwn.parallel.comm import Comm
    cfg = replace(tiny_qwen36(moe=True), dn_k_heads=4, dn_v_heads=8, moe_inter=128, shared_inter=128)
    blk = _hf_block(cfg, seed=2)
    sd = _layer_state(blk, cfg)
    x = torch.randn(5, cfg.hidden)
    with torch.no_grad():
        ref = blk(x[None])[0]
    total = torch.zeros_like(ref)
    for r in range(world):
        m = Qwen36Model(cfg, Comm(None, r, world), "cpu", torch.float32, moe_sharding="tp")
        L = W.fuse_layer(cfg, 0, W.hf_getter(sd), world, r, torch.float32, "tp")
        assert m.d.expert_offset == 0 and L["experts_gate_up"].shape == (cfg.num_experts, 2 * 128 // world, cfg.hidden)
        assert L["experts_down"].shape == (cfg.num_experts, cfg.hidden, 128 // world)
        total += qwen_moe_forward(m, L, x).float()
    assert torch.allclose(total, ref, atol=1e-5), (total - ref).abs().max()


def test_tensor_parallel_experts_dims():
    """Per-rank dims of the tensor-parallel expert layout and its checks."""
    from bwn.config import tp_dims
    cfg = tiny_qwen36(moe=True)
    with pytest.raises(ValueError):
        tp_dims(cfg, 8, 0, "tp")  # 64 / 8 = 8 columns: below a 16-row gate/up block
    with pytest.raises(ValueError):
        tp_dims(cfg, 2, 0, "xx")
    d = tp_dims(cfg, 2, 1, "tp")
    assert (d.experts, d.expert_offset, d.moe_inter) == (cfg.num_experts, 0, cfg.moe_inter // 2)


def test_shared_only_probe(monkeypatch):
    from bwn.models.moe import qwen_moe_forward
    from bwn.models.qwen36 import build_qwen36
    cfg = tiny_qwen36(moe=True)
    monkeypatch.setenv("BWN_MOE_SHARED_ONLY", "1")
    m = build_qwen36(cfg, seed=1, dtype=torch.float32)
    x = torch.randn(3, cfg.hidden)
    L = m.layers[0]
    got = qwen_moe_forward(m, L, x)
    sy = O.linear(O.linear_swiglu(x, L["shared_gate_up"]), L["shared_down"])
    assert torch.allclose(got, torch.sigmoid(x @ L["shared_gate"].t()) * sy, atol=1e-6)
