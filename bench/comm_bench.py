#!/usr/bin/env python
"""Row-parallel GEMM -> all-reduce -> residual add -> RMSNorm at decode sizes:
NCCL baseline vs the fused NVLink kernels.  Each case is captured in a CUDA
graph of ``--iters`` back-to-back calls (as inside the decode step) and timed
with CUDA events; the reported time is the max over ranks.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 bench/comm_bench.py --rows 32 --k 2176
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
from bwn.parallel.fused import FusedComm  # noqa: E402


def timed_graph(fn, iters, comm):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(iters):
            fn()
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    comm.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / iters
    del g
    return comm.max_scalar(us)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=32)
    ap.add_argument("--hidden", type=int, default=5120)
    ap.add_argument("--k", type=int, default=2176, help="local K of the row-parallel GEMM (down_proj at TP8)")
    ap.add_argument("--iters", type=int, default=64)
    args = ap.parse_args()
    comm = init_distributed("nccl", timeout_s=120)
    dev = torch.device("cuda", torch.cuda.current_device())
    R, H, K = args.rows, args.hidden, args.k
    g = torch.Generator(device=dev).manual_seed(comm.rank)
    a = torch.randn(R, K, device=dev, generator=g).bfloat16()
    w = (torch.randn(H, K, device=dev, generator=g) * 0.02).bfloat16()
    x = torch.randn(R, H, device=dev, generator=g).bfloat16()
    nw = torch.zeros(H, device=dev)
    part = torch.randn(R, H, device=dev, generator=g).bfloat16()
    fc = FusedComm(comm, H, max_rows=max(R, 32), device=dev)
    res = {}

    def nccl_ar():
        p = part.clone()
        comm.all_reduce_(p)
        return O.add_rms_norm(p, x, nw, 1e-6)

    def nccl_gemm_ar():
        p = O.linear(a, w)
        comm.all_reduce_(p)
        return O.add_rms_norm(p, x, nw, 1e-6)

    res["gemm_only_us"] = timed_graph(lambda: O.linear(a, w), args.iters, comm)
    res["add_norm_only_us"] = timed_graph(lambda: O.add_rms_norm(part, x, nw, 1e-6), args.iters, comm)
    res["nccl_allreduce_add_norm_us"] = timed_graph(nccl_ar, args.iters, comm)
    res["fused_allreduce_add_norm_us"] = timed_graph(lambda: fc.allreduce_add_norm(part, x, nw, 1e-6), args.iters,
                                                     comm)
    res["nccl_gemm_allreduce_add_norm_us"] = timed_graph(nccl_gemm_ar, args.iters, comm)
    res["fused_gemm_allreduce_add_norm_us"] = timed_graph(lambda: fc.gemm_allreduce_add_norm(a, w, x, nw, 1e-6),
                                                          args.iters, comm)
    check_status("comm bench")
    # roofline of the fused GEMM+all-reduce: max(weight bytes / HBM, reduced bytes / NVLink)
    nvlink_gbs, hbm_gbs = 770.0, 6553.0
    t_w = H * K * 2 / (hbm_gbs * 1e3)           # us
    t_link = R * H * 4 / (nvlink_gbs * 1e3)     # fp32 partial, one pass through the switch
    res["roofline_us"] = round(max(t_w, t_link), 2)
    res["fused_fraction_of_roofline"] = round(res["roofline_us"] / res["fused_gemm_allreduce_add_norm_us"], 3)
    if comm.rank == 0:
        print(json.dumps({"bench": "row-parallel GEMM + all-reduce + add + RMSNorm", "world": comm.size,
                          "rows": R, "hidden": H, "k": K, **{k: round(v, 2) for k, v in res.items()}}))
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
