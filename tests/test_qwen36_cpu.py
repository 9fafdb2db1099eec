"""Model-level CPU parity: bwn's Qwen3.6 (reference-op path, fp32) against the
HF ``Qwen3_5ForCausalLM`` / ``Qwen3_5MoeForCausalLM`` oracles on a tiny
random checkpoint (the reference's ``test_parity_vs_hf.py`` and
``test_prefill_decode_consistency.py`` tiers)."""
import pytest
import torch

from bwn.config import tiny_qwen36
from bwn.models.qwen36 import build_qwen36


def _hf_model(cfg):
    from transformers.models.qwen3_5 import modeling_qwen3_5 as M
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    hc = Qwen3_5TextConfig(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
        num_hidden_layers=cfg.num_layers, num_attention_heads=cfg.q_heads, num_key_value_heads=cfg.kv_heads,
        head_dim=cfg.head_dim, linear_num_key_heads=cfg.dn_k_heads, linear_num_value_heads=cfg.dn_v_heads,
        linear_key_head_dim=cfg.dn_k_dim, linear_value_head_dim=cfg.dn_v_dim, rms_norm_eps=cfg.rms_eps,
        rope_parameters={"rope_type": "default", "rope_theta": cfg.rope_theta,
                         "partial_rotary_factor": cfg.partial_rotary},
        tie_word_embeddings=False,
    )
    torch.manual_seed(1)
    m = M.Qwen3_5ForCausalLM(hc).eval()
    with torch.no_grad():  # make norms/gates non-trivial
        for n, p in m.named_parameters():
            if n.endswith("norm.weight") or n.endswith("layernorm.weight"):
                p.add_(torch.randn_like(p) * 0.1)
    return m


def _hf_moe_model(cfg):
    from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as M
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    hc = Qwen3_5MoeTextConfig(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, num_hidden_layers=cfg.num_layers,
        num_attention_heads=cfg.q_heads, num_key_value_heads=cfg.kv_heads, head_dim=cfg.head_dim,
        linear_num_key_heads=cfg.dn_k_heads, linear_num_value_heads=cfg.dn_v_heads,
        linear_key_head_dim=cfg.dn_k_dim, linear_value_head_dim=cfg.dn_v_dim, rms_norm_eps=cfg.rms_eps,
        num_experts=cfg.num_experts, num_experts_per_tok=cfg.top_k, moe_intermediate_size=cfg.moe_inter,
        shared_expert_intermediate_size=cfg.shared_inter,
        rope_parameters={"rope_type": "default", "rope_theta": cfg.rope_theta,
                         "partial_rotary_factor": cfg.partial_rotary},
        tie_word_embeddings=False,
    )
    torch.manual_seed(2)
    m = M.Qwen3_5MoeForCausalLM(hc).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if "experts" in n or n.endswith("gate.weight"):
                p.normal_(0, 0.05)
    return m


@pytest.mark.parametrize("moe", [False, True])
def test_prefill_and_decode_match_hf(moe):
    cfg = tiny_qwen36(moe=moe)
    hf = _hf_moe_model(cfg) if moe else _hf_model(cfg)
    sd = {k: v.detach().clone() for k, v in hf.state_dict().items()}
    m = build_qwen36(cfg, hf_state=sd, dtype=torch.float32)
    B, S = 2, 11
    toks = torch.randint(0, cfg.vocab, (B, S))
    st = m.new_state(B, 64)
    h = m.prefill_hidden(toks, st)
    with torch.no_grad():
        ref = hf(toks).logits[:, -1].float()
    got = m.logits(h)
    assert torch.allclose(got, ref, atol=2e-3, rtol=2e-3), (got - ref).abs().max()
    assert st.positions.tolist() == [S, S]
    seq = toks
    for _ in range(3):
        nxt = got.argmax(-1)
        seq = torch.cat([seq, nxt[:, None]], 1)
        h = m.decode_hidden(nxt.int(), st)
        got = m.logits(h)
        with torch.no_grad():
            ref = hf(seq).logits[:, -1].float()
        assert torch.allclose(got, ref, atol=2e-3, rtol=2e-3), (got - ref).abs().max()


@pytest.mark.parametrize("lens", [(37, 29), (29, 37)])
def test_bucketed_prefill_equals_whole(lens):
    """Chunked (bucketed) prefill with state carry == one-shot prefill, including
    pad rows (valid_len) that must leave the state untouched, whichever row is
    the short one (a chunk starts at the largest row position)."""
    cfg = tiny_qwen36()
    m = build_qwen36(cfg, seed=3, dtype=torch.float32)
    B, S = 2, 37
    toks = torch.randint(0, cfg.vocab, (B, S))
    vl = torch.tensor(lens, dtype=torch.int32)
    short = lens.index(29)
    st1 = m.new_state(B, 64)
    ids1 = m.prefill(toks, st1, valid_len=vl)
    st2 = m.new_state(B, 64)
    ids2 = m.prefill(toks, st2, valid_len=vl, bucket=16)
    assert torch.equal(ids1, ids2)
    assert st1.positions.tolist() == list(lens) and st2.positions.tolist() == list(lens)
    assert torch.allclose(st1.ssm, st2.ssm, atol=1e-4)
    # each row equals a standalone run of its real tokens
    for r in range(B):
        st3 = m.new_state(1, 64)
        ids3 = m.prefill(toks[r:r + 1, :lens[r]], st3)
        assert ids3.item() == ids2[r].item()
        assert torch.allclose(st3.ssm[:, 0], st2.ssm[:, r], atol=1e-4)
        assert torch.allclose(st3.conv[:, 0], st1.conv[:, r], atol=1e-5)  # (the bucketed ring keeps a stale 4th slot)
    assert short in (0, 1)


def test_greedy_decode_consistency():
    """prefill(prompt) + decode == prefill of the longer prompt (state handoff)."""
    cfg = tiny_qwen36()
    m = build_qwen36(cfg, seed=4, dtype=torch.float32)
    toks = torch.randint(0, cfg.vocab, (1, 9))
    st = m.new_state(1, 32)
    nxt = m.prefill(toks, st)
    h = m.decode_hidden(nxt, st)
    a = m.logits(h)
    st2 = m.new_state(1, 32)
    m.prefill_hidden(torch.cat([toks, nxt[:, None].long()], 1), st2)
    b = m.logits(m.prefill_hidden(torch.zeros(1, 0, dtype=torch.long), st2)) if False else None
    st3 = m.new_state(1, 32)
    h3 = m.prefill_hidden(torch.cat([toks, nxt[:, None].long()], 1), st3)
    assert torch.allclose(a, m.logits(h3), atol=1e-4)
    assert torch.allclose(st.ssm, st3.ssm, atol=1e-5)


def test_weight_bytes_counts_each_storage_once():
    """The decode path's expert stacks hold the routed experts as views: the
    weight count must not double them."""
    from bwn.config import tiny_qwen36
    from bwn.models.qwen36 import Qwen36Model
    m = Qwen36Model(tiny_qwen36(moe=True, layers=4), None, "cpu").init_random(0)
    L = m.layers[0]
    assert L["experts_gate_up"].untyped_storage().data_ptr() == L["experts_gate_up_x"].untyped_storage().data_ptr()
    seen = {}
    for Ld in list(m.layers) + [m.g]:
        for v in Ld.values():
            if torch.is_tensor(v):
                st = v.untyped_storage()
                seen[st.data_ptr()] = st.nbytes()
    assert m.weight_bytes() == sum(seen.values())
