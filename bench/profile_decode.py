#!/usr/bin/env python
"""One eager Qwen3.6 decode step, for kernel-level profiling.

The first bwn kernels this script launches are exactly one decode step, so
``ncu -k regex:'gemm|deltanet|gqa|rms|embedding|argmax' -c <launches>`` captures
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

        comm = ShapeOnlyComm(None, 0, args.tp_shapes)
    m = Qwen36Model(cfg, comm, device=dev).init_random(0)
    st = m.new_state(args.batch, args.ctx + 64)
    st.k_cache.normal_()
    st.v_cache.normal_()
    st.ssm.normal_(0, 0.05)
    st.positions.fill_(args.ctx)
    tok = torch.randint(0, cfg.vocab, (args.batch,), dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    for _ in range(args.steps):
        tok = m.decode_step(tok, st)
    torch.cuda.synchronize()
    print("done")


if __name__ == "__main__":
    main()
