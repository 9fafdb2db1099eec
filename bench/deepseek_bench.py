#!/usr/bin/env python
"""DeepSeek V4 Flash (284B total / 13B active; dims of the public config) on
N GPUs: tensor-parallel attention + expert-parallel MoE, random-init bf16
weights (each rank initialises its own shards), uniform-random prompt ids.
Prefill TTFT of ``--prompt-len`` tokens at batch 1, then decode ms/step at
each ``--batch`` (CUDA events, max over ranks; the decode step is captured as
a CUDA graph when possible).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 bench/deepseek_bench.py --prompt-len 4096 --batch 1 32
"""
import argparse
import json
import os
import sys
import time

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from bwn.config import DeepSeekV4Config  # noqa: E402
from bwn.models.deepseek_v4 import DeepSeekV4Model  # noqa: E402
from bwn.ops import check_status  # noqa: E402
from bwn.parallel.comm import init_distributed  # noqa: E402


def ev_ms(fn, comm, n=1):
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    comm.barrier()
    a.record()
    for _ in range(n):
        fn()
    b.record()
    torch.cuda.synchronize()
    return comm.max_scalar(a.elapsed_time(b) / n)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--prompt-len", type=int, default=4096)
    ap.add_argument("--batch", type=int, nargs="+", default=[1, 32])
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--layers", type=int, default=0, help="debug only: fewer layers (marked in the output)")
    ap.add_argument("--fp8", action="store_true", help="dense projections and LM head as 128x128 block-scaled E4M3")
    ap.add_argument("--fp8-experts", action="store_true", help="routed experts as block-scaled E4M3 (fp8 grouped GEMM)")
    ap.add_argument("--skip-prefill", action="store_true")
    ap.add_argument("--fused-comm", default="off", choices=["on", "off"],
                    help="N>1: row-parallel wo_b GEMM and MoE partials reduced through the fused NVLS kernels")
    args = ap.parse_args()
    comm = init_distributed("nccl", timeout_s=600)
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = DeepSeekV4Config()
    if args.layers:
        cfg = cfg.scaled(num_layers=args.layers)
    S = args.prompt_len
    cfg = cfg.scaled(max_seq_len=S + 64)
    t_start = time.perf_counter()

    def note(msg):
        if comm.rank == 0:
            print(f"[deepseek_bench +{time.perf_counter() - t_start:.1f}s] {msg}", file=sys.stderr, flush=True)

    model = DeepSeekV4Model(cfg, comm, dev).init_random_local(0)
    if args.fp8 or args.fp8_experts:
        model.quantize_fp8(include_head=args.fp8, experts=args.fp8_experts)
    if args.fused_comm == "on" and comm.size > 1:
        from bwn.parallel.fused import enable_fused_comm
        enable_fused_comm(model)
    torch.cuda.synchronize()
    note("weights ready")
    res = {"model": cfg.name + (f"-{args.layers}L (debug)" if args.layers else ""), "n_gpus": comm.size,
           "parallelism": f"tp{comm.size}+ep{comm.size}", "comm": "fused NVLS" if model.fused_comm else "NCCL",
           "dtype": "bf16 activations" + (", fp8 dense weights" if args.fp8 else "") +
                    (", fp8 routed experts" if args.fp8_experts else ""),
           "data": "synthetic (uniform-random prompt ids, random-init weights)",
           "weights_gb_per_gpu": round(sum(v.numel() * v.element_size() if torch.is_tensor(v) else v.nbytes()
                                           for L in model.L for v in L.values()
                                           if torch.is_tensor(v) or hasattr(v, "nbytes")) / 1e9, 1)}
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab, (1, S), generator=g).to(dev)
    if not args.skip_prefill:
        st = model.new_state(1, S + 64)
        model.prefill(prompt[:, :128], st)  # warm-up
        st = model.new_state(1, S + 64)
        res["prefill_ttft_ms"] = round(ev_ms(lambda: model.prefill(prompt, st), comm), 1)
        res["prefill_tok_s"] = round(S / res["prefill_ttft_ms"] * 1e3, 1)
        check_status("prefill")
        note("prefill done")
    for B in args.batch:
        st = model.new_state(B, S + args.steps * 4 + 64)
        st.positions.fill_(S)
        st.kv.normal_()
        tok = torch.randint(0, cfg.vocab, (B,), generator=g).int().to(dev)
        nxt = torch.zeros_like(tok)

        def step():
            nxt.copy_(model.decode_step(tok, st))

        step()
        graph = None
        try:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                step()
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=s):
                    step()
            torch.cuda.current_stream().wait_stream(s)
        except Exception as e:  # noqa: BLE001
            graph = None
            if comm.rank == 0:
                print(f"[deepseek_bench] graph capture failed, timing eager steps: {e}", file=sys.stderr)
        run = graph.replay if graph is not None else step
        st.positions.fill_(S)
        for _ in range(3):
            run()
        ms = ev_ms(run, comm, args.steps)
        check_status("decode")
        res[f"decode_b{B}"] = {"ms_per_step": round(ms, 3), "tok_s": round(B / ms * 1e3, 1),
                               "graph": graph is not None}
        note(f"decode batch {B} done")
        # release the captured graph (it holds NCCL calls) before the process group goes
        run = None
        del graph
        torch.cuda.synchronize()
    if comm.rank == 0:
        print(json.dumps({"metric": "DeepSeek V4 Flash prefill TTFT + decode tok/s", **res}))
    if comm.size > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
