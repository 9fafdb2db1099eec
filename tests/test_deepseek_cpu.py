"""DeepSeek V4: bwn's model (CPU reference-op path) against the reference's own
torch model code (``contrib/deepseek-v4-flash/run_deepseek_v4_tp.py``), imported
with torch.compile made a no-op, on a tiny random config; plus a prefill/decode
consistency check of the static KV cache."""
import importlib.util
import os
import sys

import pytest
import torch

from bwn.config import tiny_deepseek_v4
from bwn.models.deepseek_v4 import DeepSeekV4Model

# the reference checkout: BWN_REFERENCE_ROOT, else a "reference" directory beside this repository
_REF_ROOT = os.environ.get("BWN_REFERENCE_ROOT") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference")
REF = os.path.join(_REF_ROOT, "contrib", "deepseek-v4-flash", "run_deepseek_v4_tp.py")


def _load_reference():
    if not os.path.exists(REF):
        pytest.skip("reference tree not mounted")
    import types

    real = torch.compile
    torch.compile = lambda fn=None, **kw: fn  # the reference compiles for its own device
    stub = sys.modules.setdefault("torch_neuronx", types.ModuleType("torch_neuronx"))  # its device bridge
    try:
        spec = importlib.util.spec_from_file_location("ref_dsv4", REF)
        mod = importlib.util.module_from_spec(spec)
        sys.modules["ref_dsv4"] = mod
        spec.loader.exec_module(mod)
    finally:
        torch.compile = real
        if sys.modules.get("torch_neuronx") is stub:
            del sys.modules["torch_neuronx"]
    return mod


def test_matches_reference_model():
    R = _load_reference()
    cfg = tiny_deepseek_v4()
    args = R.ModelArgs(vocab_size=cfg.vocab, dim=cfg.dim, n_layers=cfg.num_layers, n_heads=cfg.n_heads,
                       head_dim=cfg.head_dim, n_routed_experts=cfg.n_routed_experts, n_activated_experts=cfg.n_activated_experts,
                       moe_inter_dim=cfg.moe_inter, q_lora_rank=cfg.q_lora_rank, rope_head_dim=cfg.rope_head_dim,
                       o_groups=cfg.o_groups, o_lora_rank=cfg.o_lora_rank, n_hash_layers=cfg.n_hash_layers,
                       max_seq_len=cfg.max_seq_len)
    torch.manual_seed(0)
    ref = R.DeepSeekV4(args, rank=0, world_size=1).float()
    with torch.no_grad():
        for n, p in ref.named_parameters():
            if "norm" in n and n.endswith("weight"):
                p.fill_(1.0)
            elif n.endswith("scale"):
                p.fill_(1.0)
            elif n.endswith("base") or n.endswith("bias"):
                p.normal_(0, 0.05)
            else:
                p.normal_(0, 0.05 if p.dim() > 1 else 0.02)
    sd = {k: v.detach().clone() for k, v in ref.state_dict().items()}
    m = DeepSeekV4Model(cfg, dtype=torch.float32).load(sd)
    toks = torch.randint(0, cfg.vocab, (1, 12))
    with torch.no_grad():
        want = ref(toks).float()[0]
    st = m.new_state(1, 64)
    B, S = toks.shape
    pos = torch.arange(S, dtype=torch.int32)
    h = m.forward_tokens(toks.reshape(-1), pos, torch.zeros(S, dtype=torch.int32), st, S)
    got = m.logits(h)
    assert torch.allclose(got, want, atol=2e-3, rtol=2e-3), (got - want).abs().max()


def test_prefill_then_decode_matches_longer_prefill():
    cfg = tiny_deepseek_v4()
    m = DeepSeekV4Model(cfg, dtype=torch.float32).init_random(0)
    toks = torch.randint(0, cfg.vocab, (2, 9))
    st = m.new_state(2, 32)
    nxt = m.prefill(toks, st)
    d = m.decode_step(nxt, st)
    st2 = m.new_state(2, 32)
    full = torch.cat([toks, nxt[:, None].long()], 1)
    B, S = full.shape
    pos = torch.arange(S, dtype=torch.int32).repeat(B)
    bidx = torch.arange(B, dtype=torch.int32).repeat_interleave(S)
    h = m.forward_tokens(full.reshape(-1), pos, bidx, st2, S)
    want = m.logits(h.view(B, S, -1)[:, -1]).argmax(-1).int()
    assert torch.equal(d, want)


def test_fp8_dense_weights_close_to_bf16():
    from bwn.models.deepseek_v4 import synthetic_checkpoint
    cfg = tiny_deepseek_v4()
    sd = synthetic_checkpoint(cfg, 0)
    a = DeepSeekV4Model(cfg, None, "cpu", torch.float32).load(sd)
    b = DeepSeekV4Model(cfg, None, "cpu", torch.float32).load(sd).quantize_fp8()
    toks = torch.randint(0, cfg.vocab, (2, 8), generator=torch.Generator().manual_seed(1))
    hs = []
    for m in (a, b):
        st = m.new_state(2, 16)
        pos = torch.arange(8, dtype=torch.int32).repeat(2)
        bidx = torch.arange(2, dtype=torch.int32).repeat_interleave(8)
        hs.append(m.logits(m.forward_tokens(toks.reshape(-1), pos, bidx, st, 8)))
    rel = float((hs[0] - hs[1]).norm() / hs[0].norm())
    assert 0 < rel < 0.1


def test_fp8_experts_close_to_bf16():
    from bwn.models.deepseek_v4 import synthetic_checkpoint
    cfg = tiny_deepseek_v4()
    sd = synthetic_checkpoint(cfg, 0)
    a = DeepSeekV4Model(cfg, None, "cpu", torch.float32).load(sd)
    b = DeepSeekV4Model(cfg, None, "cpu", torch.float32).load(sd).quantize_fp8(include_head=False, experts=True)
    assert hasattr(b.L[-1]["experts_gate_up"], "scales16")
    toks = torch.randint(0, cfg.vocab, (2, 8), generator=torch.Generator().manual_seed(2))
    hs = []
    for m in (a, b):
        st = m.new_state(2, 16)
        pos = torch.arange(8, dtype=torch.int32).repeat(2)
        bidx = torch.arange(2, dtype=torch.int32).repeat_interleave(8)
        hs.append(m.logits(m.forward_tokens(toks.reshape(-1), pos, bidx, st, 8)))
    rel = float((hs[0] - hs[1]).norm() / hs[0].norm())
    assert 0 < rel < 0.1


def test_runner_command_single_tp2_and_hybrid():
    """The runner command generates the same ids on one process, two
    tensor-parallel gloo ranks and two ranks in the hybrid layout (TP 1 x EP 2)."""
    import json
    import socket
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, PYTHONPATH=root, OMP_NUM_THREADS="2")
    args = ["-m", "bwn.models.deepseek_v4", "--tiny", "--cpu", "--max-new", "5", "--prompt-len", "9"]

    def run(pre):
        r = subprocess.run([sys.executable] + pre + args + extra, env=env, cwd=root, capture_output=True,
                           text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-3000:]
        return json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])

    def torchrun():
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
        s.close()
        return ["-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
                "--master-port", str(port)]

    extra = []
    one = run([])
    assert one["finite"] and len(one["generated"]) == 5
    tp2 = run(torchrun())
    extra = ["--hybrid-tp", "1"]
    hyb = run(torchrun())
    assert (tp2["tp"], tp2["ep"], hyb["tp"], hyb["ep"]) == (2, 2, 1, 2)
    assert tp2["generated"] == one["generated"] == hyb["generated"]
