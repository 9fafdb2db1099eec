#!/usr/bin/env python
"""One eager Qwen3.6 decode step, for kernel-level profiling.

The first bwn kernels this script launches are exactly one decode step, so
``ncu --clock-control none -k regex:'gemm|deltanet|gqa|rms|embedding|argmax' -c <launches>`` captures
that step and nothing else.  Example (one GPU):

    ncu --metrics gpu__time_duration.sum --clock-control none \
        -k regex:'gemm|deltanet|gqa|rms_norm|embedding|argmax' -c 460 --csv \
        python bench/profile_decode.py --model 27b --batch 32 --ctx 2048
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from bwn.config import QWEN36_27B, QWEN36_35B_A3B  # noqa: E402
from bwn.models.qwen36 import Qwen36Model  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="27b", choices=["27b", "35b"])
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--graph-time", type=int, default=0,
                    help="capture the step as a CUDA graph and print ms/step over this many replays")
    ap.add_argument("--tp-shapes", type=int, default=1,
                    help="emulate rank 0 of a TP group of this size on one GPU (collectives become no-ops)")
    args = ap.parse_args()
    cfg = QWEN36_27B if args.model == "27b" else QWEN36_35B_A3B
    if args.layers:
        cfg = cfg.scaled(num_layers=args.layers)
    dev = torch.device("cuda", 0)
    comm = None
    if args.tp_shapes > 1:
        from bwn.parallel.comm import Comm

        class ShapeOnlyComm(Comm):
            """Rank 0 of an N-way group whose collectives do nothing (profiling only)."""

            def all_reduce_(self, x):
                return x

            def all_reduce_max_(self, x):
                return x

            def all_gather_first(self, x):  # every rank's shard equal to this one's (shapes only)
                return torch.cat([x] * self.size, 0)

            def all_gather_last(self, x):
                return torch.cat([x] * self.size, -1)

        comm = ShapeOnlyComm(None, 0, args.tp_shapes)
    m = Qwen36Model(cfg, comm, device=dev).init_random(0)
    st = m.new_state(args.batch, args.ctx + 64)
    st.k_cache.normal_()
    st.v_cache.normal_()
    st.ssm.normal_(0, 0.05)
    st.positions.fill_(args.ctx)
    tok = torch.randint(0, cfg.vocab, (args.batch,), dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    if args.graph_time:
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):  # eager warm-up on the capture stream sizes its scratch
                m.decode_step(tok, st)
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=s):
                m.decode_step(tok, st)
        torch.cuda.current_stream().wait_stream(s)
        st.positions.fill_(args.ctx)
        for _ in range(3):
            g.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        for _ in range(args.graph_time):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        print(f"tp-shapes {args.tp_shapes} batch {args.batch}: {a.elapsed_time(b) / args.graph_time:.3f} ms/step "
              f"(graph replay, collectives skipped)")
        return
    for _ in range(args.steps):
        tok = m.decode_step(tok, st)
    torch.cuda.synchronize()
    print("done")


if __name__ == "__main__":
    main()
