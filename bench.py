#!/usr/bin/env python
"""Flagship benchmark: Qwen3.6 decode on 1-8 B200 (tensor + expert parallel).

    python bench.py --gpus N --steps K --warmup W            (N=1)
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Headline config (the reference's headline decode benchmark): Qwen3.6-35B-A3B (40 layers, hidden 2048,
[DeltaNet x3, GQA x1] x10, 256-expert top-8 MoE on every layer), bf16,
random-init weights from seed 0, TP=N for attention and EP=N for the experts,
synthetic uniform-random prompt ids, prefill 2048 then greedy decode at global
batch 32.  ``--model 27b`` runs Qwen3.6-27B instead.  The timed step is one
full decode step (all layers, LM head and sharded greedy) replayed from a CUDA
graph; W untimed warm-up steps, then K steps bracketed by barrier +
synchronize, timed with two CUDA events around the whole loop, max over ranks.
Every step streams the layers' weights and the touched experts (GBs per GPU),
far more than the 126 MB L2.

``--impl reference`` runs the reference's own 35B-A3B harness on the same
config (``bench/reference_arm.py``).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

import torch

# the reference's published decode numbers closest to each config (trn2.3xlarge)
BASELINE_TOK_S = {
    "35b": 303.9,  # 35B-A3B decode BS=32, TP=8 LNC=1, full graph (contrib/qwen3.6-35b-a3b/BENCHMARK.md:568)
    "27b": 63.1,   # 27B decode BS=16, TP=4 (contrib/qwen3.6-27b/README.md:96)
}
BASELINE_BS1_TOK_S = {
    "35b": 48.9,   # 35B-A3B decode BS=1, TP=4 LNC=2 (contrib/qwen3.6-35b-a3b/BENCHMARK.md:515)
    "27b": 28.2,   # 27B decode BS=1, TP=4 (contrib/qwen3.6-27b/README.md:94)
}
METRIC = "decode tok/s/box + p50 TPOT & prefill TTFT, Qwen3.6 TP/EP at 1/2/4/8 B200"


def reference_arm(args) -> None:
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "bench"))
    import reference_arm as RA
    RA.run(args, METRIC, BASELINE_TOK_S.get(args.model))


def count_launches(fn) -> int:
    """Number of bwn kernels one call of ``fn`` launches (each torch.ops.bwn op
    is exactly one kernel launch)."""
    import bwn.ops._ext as E

    real = E.ops
    n = [0]

    class _Proxy:
        def __getattr__(self, name):
            op = getattr(real(), name)

            def call(*a, **k):
                n[0] += 1
                return op(*a, **k)
            return call

    E.ops = lambda: _Proxy()
    import bwn.ops as O
    O.ops = E.ops
    try:
        fn()
    finally:
        E.ops = real
        O.ops = real
    return n[0]


def multi_gpu_check(model, dec, comm, dev, prefix_layers: int = 4) -> dict:
    """Decode from a copy of the live state through the product path (fused
    NVLink reductions, NVLink expert all-to-all where enabled) and through plain
    NCCL (all-reduce everywhere, the reference's formulation).  Asserted: after
    the first ``prefix_layers`` layers (every fused op, both layer types) the
    hidden states agree to bf16 accuracy (MoE: the median token, with at most
    one row in eight off by a router near-tie).  Reported: the same comparison after
    the full step, and greedy ids that differ where the top-2 logit gap
    exceeds bf16 noise -- with random weights a near-tie in an MoE router picks
    a different expert for one summation order, and 40 layers amplify it, so
    the full step is a statistic, not a pass/fail gate.  Every rank takes the
    same collective steps."""
    from bwn.models.qwen36 import Qwen36State
    st = dec.st

    def clone(s):
        return Qwen36State(conv=s.conv.clone(), ssm=s.ssm.clone(), k_cache=s.k_cache.clone(),
                           v_cache=s.v_cache.clone(), positions=s.positions.clone())

    def run(fused: bool, n_layers):
        saved = (model.fused_comm, getattr(model, "ep_a2a", None))
        if not fused:
            model.fused_comm = None
            model.ep_a2a = None
        try:
            s = clone(st)
            h = model.decode_hidden(dec.tokens.clone(), s, num_layers=n_layers)
            lg = model.logits(h) if n_layers is None else None
            del s
        finally:
            model.fused_comm, model.ep_a2a = saved
        return h, lg

    def rel(a, b):
        return comm.max_scalar(float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)), dev)

    hp1, _ = run(True, prefix_layers)
    hp2, _ = run(False, prefix_layers)
    h1, l1 = run(True, None)
    h2, l2 = run(False, None)
    torch.cuda.synchronize()
    prefix_rel, full_rel = rel(hp1, hp2), rel(h1, h2)
    # per token: a broken fused path moves every row; a router near-tie moves one
    tok = (hp1.float() - hp2.float()).norm(dim=-1) / hp2.float().norm(dim=-1).clamp_min(1e-12)
    tok_med = comm.max_scalar(float(tok.median()), dev)
    tok_over = int(comm.max_scalar(float((tok > 2e-2).sum()), dev))
    top = l2.float().topk(2, dim=-1).values
    gap = top[:, 0] - top[:, 1]
    diff = l1.argmax(-1) != l2.argmax(-1)
    noise = 0.05  # logits differ by up to ~0.02 between summation orders of bf16 partials
    beyond = int(comm.max_scalar(float((diff & (gap > noise)).sum()), dev))
    out = {"paths": "fused NVLink (+EP all-to-all) vs NCCL all-reduce",
           "prefix_layers": prefix_layers, "prefix_hidden_rel_err": round(prefix_rel, 6),
           "full_step_hidden_rel_err": round(full_rel, 6), "ids_differ": int(diff.sum()),
           "prefix_token_rel_err_median": round(tok_med, 6), "prefix_tokens_over_2e-2": tok_over,
           "ids_differ_beyond_noise": beyond, "rows": int(diff.numel())}
    if model.cfg.is_moe:
        # MoE: a token whose router sits on a near-tie may pick another expert under
        # the other summation order; the gate is the typical token and the count of
        # outliers (at most one in eight rows)
        out["ok"] = tok_med <= 2e-2 and tok_over <= max(2, out["rows"] // 8)
    else:  # no routing discontinuity: every bound holds exactly
        out["ok"] = prefix_rel <= 2e-2 and full_rel <= 2e-2 and beyond == 0
    if not out["ok"]:
        raise RuntimeError(f"multi-GPU check failed: {out}")
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="bwn", choices=["bwn", "reference"])
    ap.add_argument("--model", default="35b", choices=["27b", "35b"])
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--prompt-len", type=int, default=2048)
    ap.add_argument("--layers", type=int, default=0, help="debug only: fewer layers (result marked invalid)")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--fp8", action="store_true", help="W8A16: 128x128 block-scaled E4M3 projection weights")
    ap.add_argument("--fp8-experts", action="store_true",
                    help="MoE: block-scaled E4M3 routed experts on the fp8 grouped GEMM")
    ap.add_argument("--fused-comm", default="auto", choices=["auto", "on", "off"])
    ap.add_argument("--sp", default="auto", choices=["auto", "on", "off"],
                    help="N>1: sequence-parallel prefill (reduce-scatter/all-gather fused into the GEMM path)")
    ap.add_argument("--ep-a2a", default="auto", choices=["auto", "on", "off"],
                    help="MoE models on N>1: expert-parallel NVLink all-to-all for steps with >=16 tokens per rank")
    ap.add_argument("--moe-sharding", default="ep", choices=["ep", "tp"],
                    help="MoE models on N>1: partition experts across ranks (ep) or slice every expert (tp)")
    ap.add_argument("--profile-steps", type=int, default=int(os.environ.get("BWN_PROFILE_STEPS", "0")),
                    help="run warm-up + N decode steps only (for a profiler), then exit")
    ap.add_argument("--metrics", default=os.environ.get("BWN_METRICS", ""), help="JSONL metrics file")
    ap.add_argument("--batch1-steps", type=int, default=32,
                    help="also time batch-1 decode (latency) for this many steps; 0 skips")
    args = ap.parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return

    from bwn.config import QWEN36_27B, QWEN36_35B_A3B
    from bwn.models.qwen36 import Qwen36Model
    from bwn.ops import check_status
    from bwn.parallel.comm import init_distributed
    from bwn.runtime.static_decode import StaticDecoder
    from bwn.utils import fingerprint as F
    from bwn.utils.clocks import ClockSampler, job_gpu_ids
    from bwn.utils.env import validate
    from bwn.utils.metrics import MetricsLog

    validate()

    comm = init_distributed("nccl", timeout_s=300)
    assert comm.size == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={comm.size}"
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    base = QWEN36_27B if args.model == "27b" else QWEN36_35B_A3B
    cfg = base if not args.layers else base.scaled(num_layers=args.layers)
    B, S = args.batch, args.prompt_len
    # warm-up + timed + p50 (<= 32) + end-to-end steps, plus margin
    max_seq = S + args.warmup + args.steps * 2 + 32 + 64

    model = Qwen36Model(cfg, comm, dev, moe_sharding=args.moe_sharding).init_random(seed=0)
    if args.fp8 or args.fp8_experts:
        model.quantize_fp8(include_head=args.fp8, experts=args.fp8_experts and cfg.is_moe, dense=args.fp8)
        torch.cuda.empty_cache()
    if comm.size > 1 and args.fused_comm != "off":
        try:
            from bwn.parallel.fused import enable_fused_comm
            enable_fused_comm(model)
        except Exception as e:  # noqa: BLE001
            if args.fused_comm == "on":
                raise
            if comm.rank == 0:
                print(f"[bench] fused NVLink comm unavailable, using NCCL: {e}", file=sys.stderr)
    if cfg.is_moe and comm.size > 1 and args.ep_a2a != "off" and args.moe_sharding == "ep":
        try:
            from bwn.parallel.ep import enable_ep_all_to_all
            # prefill-sized steps; decode-sized ones (<= 64 tokens) take the fused decode MoE path
            enable_ep_all_to_all(model, max_tokens_per_rank=max(65, B * S // comm.size), min_tokens_per_rank=65)
        except Exception as e:  # noqa: BLE001
            if args.ep_a2a == "on":
                raise
            if comm.rank == 0:
                print(f"[bench] EP all-to-all unavailable: {e}", file=sys.stderr)
    if comm.size > 1 and args.sp != "off" and (B * S) % (128 * comm.size) == 0:
        try:
            from bwn.parallel.sp import enable_sequence_parallel
            enable_sequence_parallel(model, B * S)
        except Exception as e:  # noqa: BLE001
            if args.sp == "on":
                raise
            if comm.rank == 0:
                print(f"[bench] sequence-parallel prefill unavailable: {e}", file=sys.stderr)
    dec = StaticDecoder(model, B, max_seq, use_graph=not args.no_graph)
    if args.profile_steps:
        # warm-up + N decode steps and nothing else, for a profiler's timeline
        from bwn.utils.profiling import profile_steps
        dec.capture()
        ms = profile_steps(dec, args.profile_steps)
        if comm.rank == 0:
            print(json.dumps({"profile_steps": args.profile_steps, "ms_per_step": round(ms, 4)}))
        dec.release()
        return

    launches_per_step = count_launches(lambda: model.decode_step(dec.tokens, dec.st))
    dec.reset()
    dec.capture()

    # ---- prefill (TTFT) ----
    g = torch.Generator().manual_seed(1234)
    prompt = torch.randint(0, cfg.vocab, (B, S), generator=g)
    comm.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    context = "prefill"
    try:
        dec.prefill(prompt)
    except NotImplementedError:
        # decode cost depends only on the context length: fill caches/states as a
        # 2048-token prefill would (flagged in the output)
        context = "synthetic-kv"
        st = dec.st
        st.k_cache.normal_()
        st.v_cache.normal_()
        st.ssm.normal_(0, 0.05)
        st.conv.normal_()
        st.positions.fill_(S)
        dec.tokens.copy_(prompt[:, -1].to(dev))
    ev1.record()
    torch.cuda.synchronize()
    prefill_ms = comm.max_scalar(ev0.elapsed_time(ev1), dev) if context == "prefill" else None
    check_status("prefill")

    # ---- device-timed decode ----
    # One clock sampler per node (local rank 0, every GPU of the job), started
    # before the barrier so its start-up is outside the timed region; two CUDA
    # events bracket the whole K-step loop (no event between steps).
    for _ in range(args.warmup):
        dec.step_device()
    torch.cuda.synchronize()
    clk = ClockSampler(job_gpu_ids(int(os.environ.get("LOCAL_WORLD_SIZE", comm.size)))) if local == 0 else None
    if clk is not None:
        clk.__enter__()
    comm.barrier()
    torch.cuda.synchronize()
    t_ev0, t_ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_ev0.record()
    for _ in range(args.steps):
        dec.step_device()
    t_ev1.record()
    torch.cuda.synchronize()
    if clk is not None:
        clk.__exit__(None, None, None)
    comm.barrier()
    total_ms = comm.max_scalar(t_ev0.elapsed_time(t_ev1), dev)
    check_status("decode")
    # per-step TPOT distribution: a separate loop with an event between steps
    n_p = min(args.steps, 32)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(n_p + 1)]
    comm.barrier()
    torch.cuda.synchronize()
    evs[0].record()
    for i in range(n_p):
        dec.step_device()
        evs[i + 1].record()
    torch.cuda.synchronize()
    per_step = [evs[i].elapsed_time(evs[i + 1]) for i in range(n_p)]
    p50 = comm.max_scalar(statistics.median(per_step), dev)
    p_max = comm.max_scalar(max(per_step), dev)
    check_status("decode p50")

    # ---- end to end through the public per-step API (pinned H2D + D2H each step) ----
    host_tok = torch.randint(0, cfg.vocab, (B,), dtype=torch.int32)
    row0 = []
    comm.barrier()
    torch.cuda.synchronize()
    e0 = time.perf_counter()
    for _ in range(args.steps):
        host_tok = dec.step(host_tok)
        row0.append(host_tok[0])
    e_ms = (time.perf_counter() - e0) * 1e3
    e_ms = comm.max_scalar(e_ms, dev)
    check_status("e2e")
    from bwn.parallel.symm import check_canaries
    bad = check_canaries()  # outside the timed regions
    if bad:
        raise RuntimeError(f"symmetric buffers written past their end: {bad}")
    # occupancy gates on every rank (a lost state write leaves a layer empty)
    occupancy = F.check_qwen36_state(dec.st, f"decode state rank={comm.rank}")

    ms_step = total_ms / args.steps
    value = B * args.steps / (total_ms / 1e3)
    e2e_value = B * args.steps / (e_ms / 1e3)
    mg_check = multi_gpu_check(model, dec, comm, dev) if comm.size > 1 else None
    dec.release()
    del dec
    torch.cuda.empty_cache()

    # ---- batch-1 decode latency (same prompt length), its own CUDA graph ----
    batch1 = None
    if args.batch1_steps > 0:
        n1 = args.batch1_steps
        d1 = StaticDecoder(model, 1, S + n1 + 64, use_graph=not args.no_graph)
        d1.capture()
        d1.prefill(prompt[:1])
        for _ in range(3):
            d1.step_device()
        torch.cuda.synchronize()
        comm.barrier()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record()
        for _ in range(n1):
            d1.step_device()
        b1.record()
        torch.cuda.synchronize()
        ms1 = comm.max_scalar(b0.elapsed_time(b1) / n1, dev)
        check_status("batch-1 decode")
        batch1 = {"tpot_ms": round(ms1, 4), "tok_s": round(1e3 / ms1, 1), "steps": n1,
                  "vs_baseline_bs1": round((1e3 / ms1) / BASELINE_BS1_TOK_S[args.model], 2)}
        d1.release()
        del d1
    if comm.rank == 0:
        out = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "decode tokens/s (whole job)",
            "n_gpus": args.gpus,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": round(value / BASELINE_TOK_S[args.model], 3),
            "dtype": ("bf16 activations, fp8 e4m3 weights (128x128 block scales)" if args.fp8 else
                      "bf16, fp8 e4m3 routed experts (128x128 block scales)" if args.fp8_experts else "bf16"),
            "data": "synthetic (uniform-random prompt ids, random-init weights seed 0)",
            "config": {
                "model": cfg.name if not args.layers else f"{cfg.name}-{args.layers}L (INVALID: debug layer count)",
                "global_batch": B,
                "seq_len": S,
                "parallelism": f"tp{args.gpus}" + (f"+ep{args.gpus}" if cfg.is_moe else ""),
                "decode": "CUDA-graph replay, on-device greedy",
                "l2": "inputs larger than L2 (%.1f GB of weights resident per GPU; every step reads all dense "
                      "weights and each routed expert the batch picks)" % (model.weight_bytes() / 1e9),
                "fused_comm": model.fused_comm is not None,
                "ep_all_to_all": getattr(model, "ep_a2a", None) is not None,
                "prefill_sequence_parallel": getattr(model, "seq_parallel", None) is not None,
            },
            "tpot_p50_ms": round(p50, 4),
            "tpot_max_ms": round(p_max, 4),
            "context": context,
            "prefill_ttft_ms": round(prefill_ms, 2) if prefill_ms else None,
            "prefill_tok_s": round(B * S / (prefill_ms / 1e3), 1) if prefill_ms else None,
            "clocks": clk.summary() if clk is not None else None,
            "e2e": {"value": round(e2e_value, 2), "unit": "decode tokens/s (StaticDecoder.step, host round trip)",
                    "h2d_bytes_per_step": B * 4, "d2h_bytes_per_step": B * 4},
            "gpu_launches": launches_per_step * args.steps,
            "gen_hash_row0": F.gen_hash(row0),
            "batch1_decode": batch1,
            "multi_gpu_check": mg_check,
            "occupancy_min_rows": {k: min(v) for k, v in occupancy.items() if v},
        }
        print(json.dumps(out))
    if args.metrics:
        log = MetricsLog(args.metrics, comm, run={"argv": sys.argv[1:], "model": cfg.name})
        log.timing("decode_step", ms_step, batch=B)
        log.timing("decode_e2e_step", e_ms / args.steps, batch=B)
        if prefill_ms:
            log.timing("prefill", prefill_ms, batch=B, seq=S)
    if comm.size > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
