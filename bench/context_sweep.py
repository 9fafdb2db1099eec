#!/usr/bin/env python
"""Qwen3.6 prefill context sweep and decode batch sweep (the reference's
long-context prefill, ``contrib/qwen3.6-35b-a3b/PREFILL_RECIPE.md:155-160, 274-283``
and ``BENCHMARK.md:820-835``; its decode batch sweep, ``BENCHMARK.md:543-547``).

For each context S: a fresh state, a bucketed prefill of ``--prefill-batch``
uniform-random prompts of S tokens (TTFT and aggregate prompt tok/s, CUDA
events, max over ranks); every chunk is a replay of one captured graph per
bucket whose start position is a device scalar (``--eager-prefill``: plain
launches).  Then for each decode batch B: the captured decode
step timed over ``--steps`` steps at the largest context that fits
(``--decode-context``), tok/s = B / step time.  One JSON line per measurement.

    python bench/context_sweep.py --model 35b --contexts 2048 8192 20000 --decode-batches 1 16 64
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 bench/context_sweep.py --model 35b --fp8-experts
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="35b", choices=["27b", "35b"])
    ap.add_argument("--contexts", type=int, nargs="+", default=[2048, 8192, 20000])
    ap.add_argument("--prefill-batch", type=int, default=2)
    ap.add_argument("--bucket", type=int, default=1024, help="prefill chunk (tokens per sequence per pass)")
    ap.add_argument("--decode-batches", type=int, nargs="+", default=[1, 16, 64])
    ap.add_argument("--decode-context", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--layers", type=int, default=0, help="debug only: fewer layers (marked in the output)")
    ap.add_argument("--fp8-experts", action="store_true")
    ap.add_argument("--moe-sharding", default="ep", choices=["ep", "tp"])
    ap.add_argument("--eager-prefill", action="store_true", help="no captured prefill graph")
    a = ap.parse_args()

    from bwn.config import QWEN36_27B, QWEN36_35B_A3B
    from bwn.models.qwen36 import Qwen36Model
    from bwn.ops import check_status
    from bwn.parallel.comm import init_distributed
    from bwn.runtime.static_decode import StaticDecoder

    comm = init_distributed("nccl", timeout_s=600)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    base = QWEN36_27B if a.model == "27b" else QWEN36_35B_A3B
    cfg = base if not a.layers else base.scaled(num_layers=a.layers)
    model = Qwen36Model(cfg, comm, dev, moe_sharding=a.moe_sharding).init_random(seed=0)
    if a.fp8_experts and cfg.is_moe:
        model.quantize_fp8(include_head=False, experts=True, dense=False)
    if comm.size > 1:
        from bwn.parallel.fused import enable_fused_comm
        enable_fused_comm(model)
    name = cfg.name + (f"-{a.layers}L (debug)" if a.layers else "")

    def emit(**kv):
        if comm.rank == 0:
            print(json.dumps({"model": name, "n_gpus": comm.size, "data": "synthetic, random-init weights",
                              "experts": "fp8" if a.fp8_experts else "bf16", **kv}), flush=True)

    def timed(fn):
        comm.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = fn()
        e1.record()
        torch.cuda.synchronize()
        return out, comm.max_scalar(e0.elapsed_time(e1), dev)

    g = torch.Generator().manual_seed(7)
    B = a.prefill_batch
    for S in a.contexts:
        prompt = torch.randint(0, cfg.vocab, (B, S), generator=g).to(dev)
        cap = -(-S // a.bucket) * a.bucket + 8  # whole buckets
        pf = StaticDecoder(model, B, cap, use_graph=not a.eager_prefill)
        pf.capture_prefill(a.bucket)
        if a.eager_prefill:  # warm the kernels and the allocator on one chunk
            model.prefill(prompt[:, :min(S, a.bucket)], model.new_state(B, min(S, a.bucket) + 8), None, a.bucket)
        _, ms = timed(lambda: pf.prefill(prompt, None, a.bucket))
        check_status(f"prefill {S}")
        emit(phase="prefill", context=S, batch=B, bucket=a.bucket, ttft_ms=round(ms, 2),
             agg_tok_s=round(B * S / (ms / 1e3), 1), graph=not a.eager_prefill)
        pf.release()
        del pf
        torch.cuda.empty_cache()

    for Bd in a.decode_batches:
        dec = StaticDecoder(model, Bd, a.decode_context + a.warmup + a.steps + 8)
        dec.capture()
        prompt = torch.randint(0, cfg.vocab, (Bd, a.decode_context), generator=g)
        dec.prefill(prompt, bucket=a.bucket)
        for _ in range(a.warmup):
            dec.step_device()

        def run():
            for _ in range(a.steps):
                dec.step_device()
        _, ms = timed(run)
        check_status(f"decode B={Bd}")
        emit(phase="decode", batch=Bd, context=a.decode_context, steps=a.steps, ms_per_step=round(ms / a.steps, 4),
             tok_s=round(Bd * a.steps / (ms / 1e3), 1))
        dec.release()
        del dec
        torch.cuda.empty_cache()
    if comm.size > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
