#!/usr/bin/env python
"""Run one bwn kernel on a fixed small case a few times (for ncu captures and
quick timing).  Each op here is one kernel launch per iteration, except the
MoE blocks (route, gather, two grouped GEMMs, combine: five launches).

    python bench/kernel_case.py --op linear --M 32 --N 5120 --K 6144
    python bench/kernel_case.py --op gqa --B 32 --QH 24 --KVH 4 --ctx 2048
    python bench/kernel_case.py --op deltanet --B 32 --KH 16 --VH 48
    python bench/kernel_case.py --op moe_w8 --T 32 --E 256 --k 8 --H 2048 --I 512
    # model-level cases (a few full-width layers): pick the kernel with ncu -k
    python bench/kernel_case.py --op prefill --model 35b --layers 4 --B 2 --ctx 2048   # flash / chunked DeltaNet
    python bench/kernel_case.py --op decode --model 35b --layers 4 --B 32             # fused MoE decode kernels
    python bench/kernel_case.py --op deepseek --layers 2 --B 1 --ctx 1024             # HC mixing, MQA attention
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bwn.ops as O  # noqa: E402
from bwn.ops import reference as R  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", required=True, choices=["linear", "linear_w8", "swiglu", "gqa", "deltanet", "moe", "moe_w8",
                                                    "prefill", "decode", "deepseek"])
    ap.add_argument("--model", default="35b", choices=["27b", "35b"])
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--fp8-experts", action="store_true")
    ap.add_argument("--M", type=int, default=32)
    ap.add_argument("--N", type=int, default=5120)
    ap.add_argument("--K", type=int, default=6144)
    ap.add_argument("--B", type=int, default=32)
    ap.add_argument("--QH", type=int, default=24)
    ap.add_argument("--KVH", type=int, default=4)
    ap.add_argument("--KH", type=int, default=16)
    ap.add_argument("--VH", type=int, default=48)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--T", type=int, default=32, help="MoE tokens")
    ap.add_argument("--E", type=int, default=256, help="MoE experts (all local)")
    ap.add_argument("--k", type=int, default=8, help="MoE experts per token")
    ap.add_argument("--H", type=int, default=2048)
    ap.add_argument("--I", type=int, default=512)
    ap.add_argument("--iters", type=int, default=5)
    a = ap.parse_args()
    dev = "cuda"
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    if a.op == "linear_w8":
        from bwn.io.fp8 import FP8Weight
        x = torch.randn(a.M, a.K, device=dev).bfloat16()
        fw = FP8Weight.from_dense(torch.randn(a.N, a.K, device=dev) * 0.02)
        fn = lambda: O.linear(x, fw)  # noqa: E731
        nbytes = a.N * a.K
    elif a.op in ("linear", "swiglu"):
        x = torch.randn(a.M, a.K, device=dev).bfloat16()
        w = (torch.randn(a.N, a.K, device=dev) * 0.02).bfloat16()
        fn = (lambda: O.linear(x, w)) if a.op == "linear" else (lambda: O.linear_swiglu(x, w))
        nbytes = a.N * a.K * 2
    elif a.op in ("moe", "moe_w8"):
        from bwn.io.fp8 import FP8Experts
        x = torch.randn(a.T, a.H, device=dev).bfloat16()
        w, ids = O.moe_topk_softmax(torch.randn(a.T, a.E, device=dev), a.k)
        g = torch.randn(a.E, a.I, a.H, device=dev) * 0.02
        u = torch.randn(a.E, a.I, a.H, device=dev) * 0.02
        dn = torch.randn(a.E, a.H, a.I, device=dev) * 0.02
        if a.op == "moe_w8":
            gu, dw = FP8Experts.quantize_gate_up(g, u), FP8Experts.quantize(dn)
        else:
            gu = torch.stack([O.interleave_gate_up(g[e], u[e]) for e in range(a.E)]).bfloat16()
            dw = dn.bfloat16()
        del g, u, dn
        fn = lambda: O.moe_experts(x, w, ids, gu, dw, 0)  # noqa: E731
        active = int(torch.unique(ids).numel())
        nbytes = active * 3 * a.I * a.H * (1 if a.op == "moe_w8" else 2)
    elif a.op == "gqa":
        D = 256
        qg = torch.randn(a.B, a.QH, 2 * D, device=dev).bfloat16()
        kv = torch.randn(a.B, 2, a.KVH, D, device=dev).bfloat16()
        qn = torch.zeros(D, device=dev)
        cos, sin = R.rope_table(a.ctx + 64, 64, 1e7, device=dev)
        kc = torch.randn(a.B, a.KVH, a.ctx + 64, D, device=dev).bfloat16()
        vc = torch.randn_like(kc)
        pos = torch.full((a.B,), a.ctx, dtype=torch.int32, device=dev)
        fn = lambda: O.gqa_decode(qg, kv[:, 0], kv[:, 1], qn, qn, cos, sin, kc, vc, pos)  # noqa: E731
        nbytes = a.B * a.KVH * (a.ctx + 1) * D * 2 * 2
    elif a.op in ("prefill", "decode"):
        from bwn.config import QWEN36_27B, QWEN36_35B_A3B
        from bwn.models.qwen36 import Qwen36Model
        cfg = (QWEN36_27B if a.model == "27b" else QWEN36_35B_A3B).scaled(num_layers=a.layers)
        m = Qwen36Model(cfg, None, torch.device(dev)).init_random(0)
        if a.fp8_experts:
            m.quantize_fp8(include_head=False, experts=True, dense=False)
        g = torch.Generator().manual_seed(0)
        if a.op == "prefill":
            prompt = torch.randint(0, cfg.vocab, (a.B, a.ctx), generator=g).to(dev)
            st = m.new_state(a.B, a.ctx + 64)

            def fn():
                st.reset()
                m.prefill(prompt, st)
            nbytes = m.weight_bytes()
        else:
            st = m.new_state(a.B, a.ctx + 64 + 64)
            st.k_cache.normal_()
            st.v_cache.normal_()
            st.ssm.normal_(0, 0.05)
            tok = torch.randint(0, cfg.vocab, (a.B,), generator=g).int().to(dev)

            def fn():
                st.positions.fill_(a.ctx)
                m.decode_step(tok, st)
            nbytes = m.weight_bytes()
    elif a.op == "deepseek":
        from bwn.config import DeepSeekV4Config
        from bwn.models.deepseek_v4 import DeepSeekV4Model
        cfg = DeepSeekV4Config().scaled(num_layers=a.layers, max_seq_len=a.ctx + 64)
        m = DeepSeekV4Model(cfg, None, torch.device(dev)).init_random_local(0)
        prompt = torch.randint(0, cfg.vocab, (a.B, a.ctx), generator=torch.Generator().manual_seed(0)).to(dev)

        def fn():
            st = m.new_state(a.B, a.ctx + 64)
            m.prefill(prompt, st)
        nbytes = 1
    else:
        C = 2 * a.KH * 128 + a.VH * 128
        fused = torch.randn(a.B, C + a.VH * 128 + 2 * a.VH, device=dev).bfloat16()
        qkv, z = fused[:, :C], fused[:, C:C + a.VH * 128]
        bb, aa = fused[:, C + a.VH * 128:C + a.VH * 129], fused[:, C + a.VH * 129:]
        ring = torch.randn(a.B, 4, C, device=dev).bfloat16()
        st = torch.randn(a.B, a.VH, 128, 128, device=dev) * 0.05
        pos = torch.full((a.B,), 100, dtype=torch.int32, device=dev)
        cw = torch.randn(C, 4, device=dev)
        hv = torch.zeros(a.VH, device=dev)
        nw = torch.ones(128, device=dev)
        fn = lambda: O.deltanet_decode(qkv, z, aa, bb, ring, st, pos, cw, hv, hv, nw, a.KH)  # noqa: E731
        nbytes = a.B * a.VH * 128 * 128 * 4 * 2
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(a.iters):
        ev[0].record()
        fn()
        ev[1].record()
        torch.cuda.synchronize()
        ts.append(ev[0].elapsed_time(ev[1]))
    t = sorted(ts)[len(ts) // 2]
    O.check_status(a.op)
    print(f"{a.op}: median {t * 1e3:.1f} us, {nbytes / t / 1e6:.1f} GB/s (algorithmic bytes {nbytes / 1e6:.1f} MB)")


if __name__ == "__main__":
    main()
