#!/usr/bin/env python
"""EAGLE3 speculative decode on Qwen3.6 (one GPU): plain greedy decode vs
speculative steps with the 1-layer random-init EAGLE3 draft, and with an
oracle draft (the known greedy continuation, every draft accepted: the upper
bound of a verify step).  Random-init weights and uniform-random prompt ids.

    python bench/spec_bench.py --batch 1 --prompt-len 2048 --drafts 4 --steps 32
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from bwn.config import QWEN36_27B, QWEN36_35B_A3B  # noqa: E402
from bwn.models.eagle3 import Eagle3Draft, eagle3_config  # noqa: E402
from bwn.models.qwen36 import Qwen36Model  # noqa: E402
from bwn.ops import check_status  # noqa: E402
from bwn.runtime.spec_decode import SpecDecoder  # noqa: E402
from bwn.runtime.static_decode import StaticDecoder  # noqa: E402


def _time(fn, n):
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(n):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / n


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="27b", choices=["27b", "35b"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--prompt-len", type=int, default=2048)
    ap.add_argument("--drafts", type=int, default=4)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=4)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    cfg = QWEN36_27B if args.model == "27b" else QWEN36_35B_A3B
    B, S, K = args.batch, args.prompt_len, args.drafts
    N = K + 1
    gen_len = (args.steps + args.warmup + 2) * N + 8
    max_seq = S + gen_len + 16
    target = Qwen36Model(cfg, None, dev).init_random(0)
    draft = Eagle3Draft(eagle3_config(cfg), dev).init_random(1)
    prompt = torch.randint(0, cfg.vocab, (B, S), generator=torch.Generator().manual_seed(1234))

    # plain greedy decode
    dec = StaticDecoder(target, B, max_seq + args.steps + args.warmup)
    dec.capture()
    dec.prefill(prompt)
    for _ in range(args.warmup):
        dec.step_device()
    plain_ms = _time(dec.step_device, args.steps)
    check_status("plain decode")
    dec.release()
    del dec
    torch.cuda.empty_cache()

    res = {}
    # random draft: the emitted sequence is the target's greedy continuation under
    # the verify kernels; it is also the oracle for the all-accepted run
    sd = SpecDecoder(target, draft, B, max_seq, num_draft=K)
    cont = [[int(v)] for v in sd.prefill(prompt).cpu()]
    sd.capture()
    while min(len(c) for c in cont) < gen_len:
        ids, cnt = sd.step()
        for b in range(B):
            cont[b].extend(int(v) for v in ids[b, :int(cnt[b])])
    truth = torch.tensor([c[:gen_len] for c in cont])
    sd.release()
    del sd
    for mode in ("random_draft", "oracle_draft"):
        sd = SpecDecoder(target, draft, B, max_seq, num_draft=K)
        if mode == "oracle_draft":
            sd.set_oracle(truth, S)
        sd.prefill(prompt)
        sd.capture()
        for _ in range(args.warmup):
            sd.step_device()
        sd.accepted_total.zero_()
        sd.steps = 0
        ms = _time(sd.step_device, args.steps)
        acc = sd.mean_accepted()
        check_status(mode)
        res[mode] = {"ms_per_step": round(ms, 3), "accepted_drafts_per_step": round(acc, 3),
                     "tokens_per_step": round(acc + 1, 3), "tok_s": round(B * (acc + 1) / ms * 1e3, 1)}
        sd.release()
        del sd
        torch.cuda.empty_cache()
    print(json.dumps({
        "metric": "EAGLE3 speculative decode tok/s (1-layer random-init draft, greedy)",
        "model": cfg.name, "batch": B, "prompt_len": S, "drafts": K, "steps": args.steps,
        "plain_decode": {"ms_per_step": round(plain_ms, 3), "tok_s": round(B / plain_ms * 1e3, 1)},
        **res,
        "draft_weight_gb": round(draft.weight_bytes() / 1e9, 3),
        "data": "synthetic (uniform-random prompt ids, random-init target and draft)",
    }))


if __name__ == "__main__":
    main()
