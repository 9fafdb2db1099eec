#!/usr/bin/env python
"""Single-process instance of every fused compute + collective path, for
kernel-level profiling: a process group of one rank, so the same kernels run
(peer stores land in this GPU's own symmetric buffer) without other ranks whose
flags a profiler's kernel replays would stall.  Paths that need an NVLS
multicast object (the fused all-reduce, the sequence-parallel gather) are
skipped here: a one-rank group has none, and the driver rejects a multicast
object over a single device; those kernels are timed with CUDA events at
N >= 2 (``bench/comm_bench.py``).  Each path runs ``--iters`` times.

    python bench/profile_fused.py --paths ep --ep-tokens 512
    ncu --set full --clock-control none -k regex:ep_ -c 3 python bench/profile_fused.py --paths ep
"""
import argparse
import os
import socket
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from bwn import ops as O  # noqa: E402
from bwn.ops import check_status  # noqa: E402
from bwn.parallel.comm import Comm  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=32)
    ap.add_argument("--hidden", type=int, default=5120)
    ap.add_argument("--k", type=int, default=2176)
    ap.add_argument("--sp-tokens", type=int, default=4096)
    ap.add_argument("--ep-tokens", type=int, default=512)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--paths", default="ar,sp,ep,grad")
    a = ap.parse_args()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            device_id=torch.device("cuda", 0))
    comm = Comm(dist.group.WORLD, 0, 1)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    R, H, K = a.rows, a.hidden, a.k
    paths = a.paths.split(",")

    def run(name, setup):
        """``setup`` builds the path's buffers (errors there, e.g. no multicast
        object on a one-GPU group, skip the path) and returns one iteration;
        kernel errors are not caught."""
        if name not in paths:
            return
        try:
            step = setup()
        except RuntimeError as e:
            print(f"{name}: skipped ({str(e).splitlines()[0][:160]})")
            return
        for _ in range(a.iters):
            step()
        torch.cuda.synchronize()
        check_status(name)
        print(f"{name}: ok")

    def ar():
        from bwn.parallel.fused import FusedComm
        fc = FusedComm(comm, H, max_rows=max(R, 32), device=dev)
        x = torch.randn(R, K, device=dev, generator=g).bfloat16()
        w = (torch.randn(H, K, device=dev, generator=g) * 0.02).bfloat16()
        resid = torch.randn(R, H, device=dev, generator=g).bfloat16()
        nw = torch.zeros(H, device=dev)
        part = torch.randn(R, H, device=dev, generator=g).bfloat16()

        def step():
            fc.gemm_allreduce_add_norm(x, w, resid, nw, 1e-6)
            fc.allreduce_add_norm(part, resid, nw, 1e-6)
        return step

    def sp_path():
        from bwn.parallel.sp import SeqParallel
        T = a.sp_tokens
        sp = SeqParallel(comm, H, T, device=dev)
        xs = torch.randn(T, H, device=dev, generator=g).bfloat16()
        a_in = torch.randn(T, K, device=dev, generator=g).bfloat16()
        w_row = (torch.randn(H, K, device=dev, generator=g) * 0.02).bfloat16()
        w_col = (torch.randn(4096, H, device=dev, generator=g) * 0.02).bfloat16()
        nw = torch.zeros(H, device=dev)

        def step():
            sp.row_parallel(a_in, w_row)
            sp.norm_gather(xs, nw, 1e-6)
            sp.column(w_col, T)
        return step

    def ep_path():
        from bwn.parallel.ep import EPAllToAll
        E, Hm, I, k, T = 256, 2048, 512, 8, a.ep_tokens
        ep = EPAllToAll(comm, Hm, E, k, max_tokens=T, device=dev)
        gu = (torch.randn(E, 2 * I, Hm, device=dev, generator=g) * 0.02).bfloat16()
        dn = (torch.randn(E, Hm, I, device=dev, generator=g) * 0.02).bfloat16()
        xe = torch.randn(T, Hm, device=dev, generator=g).bfloat16()
        wt, ids = O.moe_topk_softmax(torch.randn(T, E, device=dev, generator=g), k, True)
        return lambda: ep.moe(xe, wt, ids, gu, dn)

    def grad_path():
        from bwn.parallel.grad_reduce import GradReducer
        from bwn.train.esm_mlm import build_esm
        m = build_esm("650M", device=dev, seed=0)
        red = GradReducer(m, comm, bucket_mb=64)
        for p in m.parameters():
            p.grad.normal_(generator=g)
        return red.finish

    run("ar", ar)
    run("sp", sp_path)
    run("ep", ep_path)
    run("grad", grad_path)
    check_status("profile_fused")
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
