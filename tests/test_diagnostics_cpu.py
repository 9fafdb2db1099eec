"""Decode diagnostics on CPU: the tapped decode step advances the state exactly
as the regular step does, its per-layer residual taps match HF's hidden
states, captures round-trip through files, and the comparison localizes a
perturbed layer and applies the near-tie greedy gate (the reference's
``decode_step_diagnostics`` and ``test_decode_fullgraph_device.py`` capture /
compare tier)."""
import copy

import pytest
import torch

from bwn.config import tiny_qwen36
from bwn.models.qwen36 import build_qwen36
from bwn.runtime import diagnostics as D


def test_near_tie_gate():
    ref = torch.tensor([[1.0, 0.0, 0.9375, -1.0], [2.0, 1.0, 0.0, 0.0]])
    ref_ids = torch.tensor([0, 0])
    cand = torch.tensor([[0.9375, 0.0, 1.0, -1.0], [1.0, 2.0, 0.0, 0.0]])
    cand_ids = torch.tensor([2, 1])
    rejected, details = D.near_tie_mismatches(ref, ref_ids, cand, cand_ids, 0.125)
    assert details[0] == (0, 0, 2, 0.0625, 0.0625, True)   # a mutual near tie: accepted
    assert rejected == [1] and details[1][-1] is False     # a 1.0 margin: rejected


@pytest.mark.parametrize("moe", [False, True])
def test_tapped_step_equals_regular_step(moe):
    cfg = tiny_qwen36(moe=moe)
    m = build_qwen36(cfg, seed=4, dtype=torch.float32)
    toks = torch.randint(0, cfg.vocab, (2, 7), generator=torch.Generator().manual_seed(0))
    st = m.new_state(2, 32)
    m.prefill_hidden(toks, st)
    st2 = copy.deepcopy(st)
    nxt = torch.tensor([5, 9], dtype=torch.int32)
    h = m.decode_hidden(nxt, st)
    cap = D.decode_diagnostics(m, nxt, st2, layers=[0, 3])
    assert sorted(cap["layers"]) == [0, 3]
    assert torch.allclose(cap["hidden"], h, atol=1e-5)
    assert torch.equal(st.positions, st2.positions)
    for a, b in [(st.ssm, st2.ssm), (st.conv, st2.conv), (st.k_cache, st2.k_cache), (st.v_cache, st2.v_cache)]:
        assert torch.allclose(a, b, atol=1e-5)
    taps = cap["layers"][3]
    expect = {"input", "mixer", "attn", "post_attn", "moe_in", "mlp", "output"}
    if moe:
        expect |= {"router_ids", "router_w", "routed_local", "routed", "shared"}
        assert torch.allclose(taps["routed"] + taps["shared"], taps["mlp"], atol=1e-5)
    assert set(taps) == expect
    assert torch.allclose(taps["post_attn"], taps["input"] + taps["attn"], atol=1e-5)
    assert torch.allclose(taps["output"], taps["post_attn"] + taps["mlp"], atol=1e-5)
    assert torch.equal(cap["next_id"], cap["logits"].argmax(-1).int())


def test_residual_taps_match_hf_hidden_states():
    from test_qwen36_cpu import _hf_model
    cfg = tiny_qwen36()
    hf = _hf_model(cfg)
    m = build_qwen36(cfg, hf_state={k: v.detach().clone() for k, v in hf.state_dict().items()},
                     dtype=torch.float32)
    toks = torch.randint(0, cfg.vocab, (1, 9), generator=torch.Generator().manual_seed(1))
    st = m.new_state(1, 32)
    m.prefill_hidden(toks[:, :-1], st)
    cap = D.decode_diagnostics(m, toks[0, -1:].int(), st)
    with torch.no_grad():
        hs = hf(toks, output_hidden_states=True).hidden_states
    for i in range(cfg.num_layers):
        assert torch.allclose(cap["layers"][i]["input"][0], hs[i][0, -1], atol=2e-3), i
    for i in range(cfg.num_layers - 1):  # the last entry of hidden_states is final-normed
        assert torch.allclose(cap["layers"][i]["output"][0], hs[i + 1][0, -1], atol=2e-3), i


def _capture(m, cfg, out_dir):
    toks = torch.randint(0, cfg.vocab, (3, 6), generator=torch.Generator().manual_seed(2))
    st = m.new_state(3, 32)
    ids = m.greedy(m.prefill_hidden(toks, st))
    cap = D.decode_diagnostics(m, ids.int(), st)
    D.save_capture(cap, str(out_dir), rank=0, meta={"cfg": cfg.name})
    return D.load_captures(str(out_dir))


def test_capture_compare_localizes_a_perturbed_layer(tmp_path):
    cfg = tiny_qwen36(moe=True)
    a = build_qwen36(cfg, seed=7, dtype=torch.float32)
    ref = _capture(a, cfg, tmp_path / "a")
    assert ref[0]["meta"] == {"cfg": cfg.name}
    same = D.compare_captures(ref, _capture(build_qwen36(cfg, seed=7, dtype=torch.float32), cfg, tmp_path / "b"))
    assert same["ok"] and same["first_diverging_tap"] is None and same["logits"]["cosine"] > 0.99999
    bad = build_qwen36(cfg, seed=7, dtype=torch.float32)
    bad.layers[2]["experts_down"].mul_(-1.0)  # corrupt layer 2's routed experts
    rep = D.compare_captures(ref, _capture(bad, cfg, tmp_path / "c"))
    assert rep["first_diverging_tap"] == "rank0/layer2/mlp"
    assert all(rep["taps"][f"rank0/layer{i}/output"]["cosine"] > 0.99999 for i in (0, 1))
    assert rep["taps"]["rank0/layer2/router_ids"]["match"] == 1.0  # routing itself unchanged
    assert D.main(["compare", str(tmp_path / "a"), str(tmp_path / "b")]) == 0


def test_global_logits_concatenates_vocab_shards():
    caps = [{"logits": torch.ones(2, 3)}, {"logits": torch.zeros(2, 3)}]
    assert D.global_logits(caps).shape == (2, 6)
    assert D.global_logits(caps, width=3).shape == (2, 3)


def test_prefill_trace(monkeypatch, capsys):
    cfg = tiny_qwen36()
    m = build_qwen36(cfg, seed=4, dtype=torch.float32)
    monkeypatch.setenv("BWN_PREFILL_TRACE", "1")
    st = m.new_state(1, 32)
    m.prefill_hidden(torch.randint(0, cfg.vocab, (1, 5)), st)
    lines = [ln for ln in capsys.readouterr().out.splitlines() if ln.startswith("[prefill-trace]")]
    assert len(lines) == cfg.num_layers and all("finite=True" in ln for ln in lines)
    assert f"layer=3 type={cfg.layer_type(3)}" in lines[3]
    monkeypatch.setenv("BWN_PREFILL_TRACE", "2")
    m.layers[1]["post_norm"][0] = float("nan")
    with pytest.raises(FloatingPointError, match="layer 1"):
        m.prefill_hidden(torch.randint(0, cfg.vocab, (1, 5)), m.new_state(1, 32))


def test_capture_command_tp2_against_single_rank(tmp_path):
    """Captures taken by the command under two gloo ranks (experts sliced
    across ranks) and by one process compare as equal (replicated taps)."""
    import os
    import socket
    import subprocess
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, PYTHONPATH=repo, OMP_NUM_THREADS="2")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    args = ["-m", "bwn.runtime.diagnostics", "capture", "--model", "tiny-moe", "--cpu", "--moe-sharding", "tp"]
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port)] + args + ["--out", str(tmp_path / "tp2")],
                       env=env, capture_output=True, text=True, timeout=300, cwd=repo)
    assert r.returncode == 0, r.stderr[-3000:]
    r = subprocess.run([sys.executable] + args + ["--out", str(tmp_path / "one")], env=env, capture_output=True,
                       text=True, timeout=300, cwd=repo)
    assert r.returncode == 0, r.stderr[-3000:]
    one, tp2 = D.load_captures(str(tmp_path / "one")), D.load_captures(str(tmp_path / "tp2"))
    assert len(one) == 1 and len(tp2) == 2 and tp2[1]["meta"]["world"] == 2
    rep = D.compare_captures(one, tp2)
    assert rep["ok"], rep["logits"]
    assert rep["first_diverging_tap"] is None
    assert all("mixer" not in k for k in rep["taps"])  # shard-local taps skipped across world sizes
