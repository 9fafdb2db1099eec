#!/usr/bin/env python
"""Serving throughput at fixed concurrency (the reference's vLLM-Neuron
assessment: output tok/s at concurrency 1/4/8 with 256-token prompts and 128
new tokens, TTFT and TPOT at concurrency 1;
``contrib/qwen3.6-35b-a3b/VLLM_NEURON_ASSESSMENT.md:135-137``).

The continuous engine keeps ``c`` requests in flight: whenever one finishes the
next is admitted, until ``--requests`` have completed.  Output tok/s = all
generated tokens / wall time; TTFT = a request's prefill (admission to first
token); TPOT = its time after the first token / (tokens - 1).  Synthetic uniform-random
prompts, random-init weights.  One JSON line per concurrency.

    python bench/serve_bench.py --model 35b --concurrency 1 4 8 --prompt-len 256 --max-tokens 128
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 bench/serve_bench.py --model 35b
"""
import argparse
import json
import os
import statistics
import sys
import time

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="27b", choices=["27b", "35b", "tiny", "tiny-moe"])
    ap.add_argument("--concurrency", type=int, nargs="+", default=[1, 4, 8])
    ap.add_argument("--requests", type=int, default=0, help="per concurrency (default 2 x concurrency, min 4)")
    ap.add_argument("--prompt-len", type=int, default=256)
    ap.add_argument("--max-tokens", type=int, default=128)
    ap.add_argument("--layers", type=int, default=0, help="debug only: fewer layers (marked in the output)")
    ap.add_argument("--fp8-experts", action="store_true")
    ap.add_argument("--cpu", action="store_true")
    a = ap.parse_args(argv)

    from bwn.config import QWEN36_27B, QWEN36_35B_A3B, tiny_qwen36
    from bwn.models.qwen36 import build_qwen36
    from bwn.parallel.comm import init_distributed
    from bwn.serve.continuous import ContinuousEngine
    from bwn.serve.engine import Request

    cpu = a.cpu or not torch.cuda.is_available()
    comm = init_distributed("gloo" if cpu else "nccl", timeout_s=600)
    dev = torch.device("cpu") if cpu else torch.device("cuda", torch.cuda.current_device())
    cfg = {"27b": QWEN36_27B, "35b": QWEN36_35B_A3B, "tiny": tiny_qwen36(), "tiny-moe": tiny_qwen36(moe=True)}[a.model]
    if a.layers:
        cfg = cfg.scaled(num_layers=a.layers)
    model = build_qwen36(cfg, comm, dev, seed=0, dtype=torch.float32 if cpu else torch.bfloat16)
    if a.fp8_experts and cfg.is_moe:
        model.quantize_fp8(include_head=False, experts=True, dense=False)
    if comm.size > 1 and not cpu:
        from bwn.parallel.fused import enable_fused_comm
        enable_fused_comm(model)
    g = torch.Generator().manual_seed(0)
    max_seq = a.prompt_len + a.max_tokens + 8
    for c in a.concurrency:
        eng = ContinuousEngine(model, c, max_seq, use_graph=not cpu)
        n = a.requests or max(4, 2 * c)
        reqs = [Request(torch.randint(0, cfg.vocab, (a.prompt_len,), generator=g).tolist(), a.max_tokens)
                for _ in range(n)]
        # warm-up: one request through admission and a few steps
        eng.run([Request(reqs[0].prompt, 4)])
        comm.barrier()
        t0 = time.perf_counter()
        results = eng.run(reqs)
        wall = comm.max_scalar(time.perf_counter() - t0, dev if not cpu else None)
        toks = sum(len(r.tokens) for r in results)
        ttft = statistics.median(r.prefill_ms for r in results)
        tpot = statistics.median(r.decode_ms / max(1, len(r.tokens) - 1) for r in results)
        if comm.rank == 0:
            print(json.dumps({
                "model": cfg.name + (f"-{a.layers}L (debug)" if a.layers else ""), "n_gpus": comm.size,
                "concurrency": c, "requests": n, "prompt_len": a.prompt_len, "max_tokens": a.max_tokens,
                "output_tok_s": round(toks / wall, 2), "ttft_ms_p50": round(ttft, 2), "tpot_ms_p50": round(tpot, 3),
                "wall_s": round(wall, 3), "engine_steps": eng.stats["steps"],
                "data": "synthetic prompts, random-init weights", "timing": "host wall clock, max over ranks"}),
                flush=True)
        eng.dec.release()
    if comm.size > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
