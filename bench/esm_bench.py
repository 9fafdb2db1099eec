#!/usr/bin/env python
"""ESM-2 masked-LM fine-tuning throughput (bf16 tcgen05 GEMMs, fp32 master
weights, AdamW), synthetic protein batches (uniform over the 20 amino acids,
15% masking with the 80/10/10 split), random-init weights.

    # ESM-2 15B, tensor parallel over 8 GPUs, global batch 16 x 1024
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 bench/esm_bench.py --size 15B --tp 8 --batch 16 --seq 1024
    # ESM-2 3B, data parallel over 8 GPUs with the fused NVLS gradient reduction
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 bench/esm_bench.py --size 3B --batch 16 --seq 1024 --reducer fused
    # ESM-2 8M on the CPU (fp32)
    python bench/esm_bench.py --size 8M --batch 8 --seq 256 --cpu

Reported time per step is the max over ranks (CUDA events; wall clock on the CPU).
"""
import argparse
import json
import os
import sys
import time

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from bwn.config import ESM2_SIZES  # noqa: E402
from bwn.models.esm2 import EsmForMaskedLM  # noqa: E402
from bwn.parallel.comm import init_distributed  # noqa: E402
from bwn.train.esm_mlm import MLMConfig, MLMTrainer  # noqa: E402


def init_on_device(model: EsmForMaskedLM, seed: int, device) -> EsmForMaskedLM:
    """Random init with a device generator (identical on every rank)."""
    g = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for n, p in model.named_parameters():
            if p.dim() >= 2:
                p.normal_(0.0, 0.02, generator=g)
            elif "LayerNorm" in n or "layer_norm" in n:
                p.fill_(1.0 if n.endswith("weight") else 0.0)
            else:
                p.zero_()
    return model


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--size", default="650M", choices=sorted(ESM2_SIZES))
    ap.add_argument("--batch", type=int, default=16, help="global batch (sequences)")
    ap.add_argument("--seq", type=int, default=1024, help="tokens per sequence incl. BOS/EOS")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--reducer", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--cpu", action="store_true")
    ap.add_argument("--act-ckpt", action="store_true", help="recompute each layer's activations in backward")
    args = ap.parse_args()
    cfg = ESM2_SIZES[args.size]
    if args.cpu:
        comm = init_distributed("gloo")
        dev = torch.device("cpu")
    else:
        comm = init_distributed("nccl", timeout_s=600)
        dev = torch.device("cuda", torch.cuda.current_device())
    W = comm.size
    tp = args.tp if W > 1 else 1
    dp = W // tp
    assert args.batch % dp == 0, "global batch must split over the data-parallel ranks"
    with torch.device(dev):  # build directly on the device (a 15B fp32 model does not fit host RAM x ranks)
        model = EsmForMaskedLM(cfg)
    model = init_on_device(model, 0, dev)
    model.activation_checkpointing = args.act_ckpt
    reducer = None
    if tp > 1:
        from bwn.parallel.tensor_parallel import apply_esm_tp
        model = apply_esm_tp(model, comm)
        torch.cuda.empty_cache()
    elif dp > 1:
        from bwn.parallel.grad_reduce import GradReducer, NcclGradReducer
        reducer = (GradReducer if args.reducer == "fused" else NcclGradReducer)(model, comm, bucket_mb=64)
    tcfg = MLMConfig(model=args.size, batch=args.batch // dp, seq_len=args.seq - 2, total_steps=1000, warmup=10)
    trainer = MLMTrainer(model, tcfg, comm if dp > 1 else None, grad_reducer=reducer)
    if tp > 1:
        trainer.gen.manual_seed(1234)  # every tensor-parallel rank sees the same batch
    batches = [trainer.next_batch() for _ in range(args.warmup + args.steps)]
    for i in range(args.warmup):
        trainer.step(batches[i])
    if dev.type == "cuda":
        torch.cuda.synchronize()
    comm.barrier()
    if dev.type == "cuda":
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
    t0 = time.perf_counter()
    loss = None
    for i in range(args.steps):
        loss = trainer.step(batches[args.warmup + i])
    if dev.type == "cuda":
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / args.steps
    else:
        ms = (time.perf_counter() - t0) * 1e3 / args.steps
    ms = comm.max_scalar(ms)
    tokens = args.batch * args.seq
    flops = 6 * cfg.param_count() * tokens + 12 * cfg.num_layers * cfg.hidden * args.seq * tokens
    if comm.rank == 0:
        print(json.dumps({
            "metric": "ESM-2 MLM fine-tune throughput", "model": f"esm2-{args.size}", "n_gpus": W if not args.cpu else 0,
            "parallelism": f"tp{tp}" if tp > 1 else (f"dp{dp}-{args.reducer}" if dp > 1 else "single"),
            "global_batch": args.batch, "seq_len": args.seq, "ms_per_step": round(ms, 2),
            "samples_per_s": round(args.batch / ms * 1e3, 2), "tokens_per_s": round(tokens / ms * 1e3, 1),
            "model_tflops_per_gpu": round(flops / (ms / 1e3) / 1e12 / max(W, 1), 1) if not args.cpu else None,
            "dtype": "fp32" if args.cpu else "bf16 GEMMs, fp32 master weights", "loss": round(float(loss), 4),
            "activation_checkpointing": args.act_ckpt,
            "data": "synthetic (uniform amino acids, 15% masking 80/10/10), random-init weights"}))
    if W > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
