#!/usr/bin/env python
"""One Qwen3.6-35B-A3B MoE layer (256 experts, top-8, H 2048, I 512) under
expert parallelism over W GPUs, three ways, timed with CUDA events (max over
ranks):

* ``a2a_fused``: NVLink peer-store dispatch -> grouped tcgen05 GEMMs -> peer
  return -> weighted combine (CUDA graph);
* ``allreduce``: every rank runs its experts over all W*T tokens, then an
  all-reduce of the partial outputs (the reference's EP formulation; CUDA graph);
* ``a2a_nccl``: NCCL all_to_all_single with host split sizes (eager).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 bench/ep_bench.py --tokens 4 512
"""
import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from bwn import ops as O  # noqa: E402
from bwn.ops import check_status  # noqa: E402
from bwn.parallel.comm import init_distributed  # noqa: E402
from bwn.parallel.ep import EPAllToAll, nccl_ep_moe  # noqa: E402


def graph_us(fn, iters, comm):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(iters):
                fn()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    comm.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    del g
    return comm.max_scalar(a.elapsed_time(b) * 1e3 / iters)


def eager_us(fn, iters, comm):
    fn()
    torch.cuda.synchronize()
    comm.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return comm.max_scalar(a.elapsed_time(b) * 1e3 / iters)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, nargs="+", default=[4, 512], help="tokens per rank")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    comm = init_distributed("nccl", timeout_s=120)
    W, rank = comm.size, comm.rank
    dev = torch.device("cuda", torch.cuda.current_device())
    E, H, I, k = 256, 2048, 512, 8
    El = E // W
    g = torch.Generator(device=dev).manual_seed(rank)
    gu = (torch.randn(El, 2 * I, H, device=dev, generator=g) * 0.02).bfloat16()
    dn = (torch.randn(El, H, I, device=dev, generator=g) * 0.02).bfloat16()
    out = {}
    for T in args.tokens:
        ep = EPAllToAll(comm, H, E, k, max_tokens=T, device=dev)
        x = torch.randn(T, H, device=dev, generator=g).bfloat16()
        logits = torch.randn(T, E, device=dev, generator=g)
        w, ids = O.moe_topk_softmax(logits, k, True)
        xa = torch.randn(T * W, H, device=dev, generator=g).bfloat16()
        la = torch.randn(T * W, E, device=dev, generator=g)
        wa, ida = O.moe_topk_softmax(la, k, True)

        def fused():
            return ep.moe(x, w, ids, gu, dn)

        def allreduce():
            p = O.moe_experts(xa, wa, ida, gu, dn, rank * El)
            comm.all_reduce_(p)
            return p

        r = {"a2a_fused_us": graph_us(fused, args.iters, comm),
             "allreduce_ep_us": graph_us(allreduce, args.iters, comm),
             "a2a_nccl_us": eager_us(lambda: nccl_ep_moe(comm, x, w, ids, gu, dn, El), args.iters, comm)}
        check_status("ep bench")
        # roofline: weights of the local experts that receive rows (at most one per
        # routed pair) over HBM vs the dispatched + returned rows over NVLink
        t_w = min(El, W * T * k) * 3 * H * I * 2 / 6553e3
        t_link = 2 * T * k * H * 2 * (W - 1) / W / 770e3
        r["roofline_us"] = round(max(t_w, t_link), 2)
        r["a2a_fused_fraction_of_roofline"] = round(r["roofline_us"] / r["a2a_fused_us"], 3)
        out[f"tokens_per_rank_{T}"] = {kk: round(v, 2) for kk, v in r.items()}
        del ep
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps({"bench": "Qwen3.6-35B-A3B MoE layer, expert parallel", "world": W, "experts": E,
                          "top_k": k, "hidden": H, "moe_inter": I, **out}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
