#!/usr/bin/env python
"""Time the bwn tcgen05 GEMM against cuBLAS (torch.matmul) on decode/prefill
shapes.  CUDA events, warm-up, L2 flushed between timed iterations; reports
achieved HBM bandwidth (weight bytes / time) and TFLOP/s."""
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bwn.ops as O  # noqa: E402

SHAPES = [  # (M tokens, N out, K in): Qwen3.6-27B TP=1 / TP=8 decode projections, prefill
    (32, 10240 + 6144 + 96, 5120), (32, 5120, 6144), (32, 17408 * 2, 5120), (32, 5120, 17408),
    (32, 12288 + 2048, 5120), (32, 248320, 5120),
    (32, 1280 + 768 + 12, 5120), (32, 5120, 768), (32, 4352, 5120), (32, 5120, 2176),
    (1, 17408 * 2, 5120), (2048, 17408 * 2, 5120), (4096, 5120, 17408),
]


def bench(fn, iters=20):
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    for _ in range(3):
        fn()
    ts = []
    for _ in range(iters):
        flush.fill_(0)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ts.sort()
    return ts[len(ts) // 2]


def main():
    import sys as _s
    if "--fp8" in _s.argv:
        from bwn.io.fp8 import FP8Weight
        for M, N, K in SHAPES[:10]:
            x = torch.randn(M, K, device="cuda").bfloat16()
            w = (torch.randn(N, K, device="cuda") * 0.02)
            fw = FP8Weight.from_dense(w)
            wb = w.bfloat16()
            t8 = bench(lambda: O.linear(x, fw))
            t16 = bench(lambda: O.linear(x, wb))
            print(json.dumps({"M": M, "N": N, "K": K, "w8_us": round(t8 * 1e3, 1), "bf16_us": round(t16 * 1e3, 1),
                              "w8_GBps": round(N * K / t8 / 1e6, 1), "bf16_GBps": round(2 * N * K / t16 / 1e6, 1)}))
        return
    for M, N, K in SHAPES:
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
        t_bwn = bench(lambda: O.linear(x, w))
        t_cub = bench(lambda: torch.matmul(x, w.t()))
        wb = N * K * 2
        fl = 2 * M * N * K
        print(json.dumps({"M": M, "N": N, "K": K, "bwn_us": round(t_bwn * 1e3, 1), "cublas_us": round(t_cub * 1e3, 1),
                          "bwn_GBps": round(wb / t_bwn / 1e6, 1), "cublas_GBps": round(wb / t_cub / 1e6, 1),
                          "bwn_TFLOPs": round(fl / t_bwn / 1e9, 1), "cublas_TFLOPs": round(fl / t_cub / 1e9, 1)}))


if __name__ == "__main__":
    main()
