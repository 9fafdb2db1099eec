"""Static decode engine: fixed-shape decode step captured once as a CUDA graph.

This is the B200 counterpart of the reference's compiled static forward
(``torch.compile(forward, backend="neuron", fullgraph=True, dynamic=False)``,
``contrib/qwen3.6-27b/static_decode.py:1183-1185``; the stateful full-graph
decode ``decode_step_stateful``, ``contrib/qwen3.6-35b-a3b/static_decode_35b.py:1600-1616``):

* all mutable state lives in static buffers (:class:`Qwen36State`), each with
  exactly one writer per step, so graph replays need no re-binding;
* the token ids and positions live on the device; the greedy next ids are
  written back into the input buffer inside the graph, so a device-side greedy
  loop needs no host round trip (``run_decode``, ``static_decode_35b.py:3142-3153``);
* :meth:`StaticDecoder.step` is the host API: pinned H2D of the step's tokens,
  graph replay, D2H of the next ids;
* :meth:`StaticDecoder.capture_prefill` captures one prefill chunk per bucket
  size; the chunk's start position is a device scalar, so one graph serves
  every chunk offset of a bucketed prefill (the reference's per-bucket compiled
  prefill with runtime ``q_base`` / ``valid_len`` scalars,
  ``static_decode_35b.py:2646-2653``).
"""
from __future__ import annotations

import torch

from ..ops import check_status


class StaticDecoder:
    """``sampling=True`` captures a step that samples each row at its entry of
    ``self.temperature`` (Gumbel-max over the sharded head; rows at 0 are
    greedy); the default step is greedy."""

    def __init__(self, model, batch: int, max_seq: int, use_graph: bool = True, ssm_dtype=torch.float32,
                 sampling: bool = False, seed: int = 0):
        self.model = model
        self.batch = batch
        self.max_seq = max_seq
        self.st = model.new_state(batch, max_seq, ssm_dtype)
        dev = model.device
        self.tokens = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.next_ids = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.sampling = sampling
        self.temperature = torch.zeros(batch, dtype=torch.float32, device=dev)
        # the default generator of the device (graph-safe under capture); a
        # separate one on the CPU keeps host runs reproducible
        # (one stream per rank: each vocab shard draws its own noise)
        self.gen = torch.Generator().manual_seed(seed + getattr(model, "rank", 0)) if dev.type == "cpu" else None
        if dev.type == "cuda" and sampling:
            torch.cuda.manual_seed(seed + getattr(model, "rank", 0))
        self.use_graph = use_graph and dev.type == "cuda"
        self.graph: torch.cuda.CUDAGraph | None = None
        self._pf: dict[int, tuple] = {}  # bucket -> (graph, ids, valid, hidden out)
        self._host_in = torch.zeros(batch, dtype=torch.int32, pin_memory=dev.type == "cuda")
        self._host_out = torch.zeros(batch, dtype=torch.int32, pin_memory=dev.type == "cuda")

    # ---------------------------------------------------------------- state
    def reset(self) -> None:
        self.st.reset()

    def prefill(self, prompt: torch.Tensor, valid_len: torch.Tensor | None = None, bucket: int = 0) -> torch.Tensor:
        """Run the prompt ``[B, S]`` through the model; the first generated ids
        become the next decode input.  Returns the ids ``[B]`` (device).  With a
        graph captured for ``bucket`` (:meth:`capture_prefill`) every chunk is a
        replay of it."""
        if bucket in self._pf:
            ids = self._prefill_graphed(prompt, valid_len, bucket)
        else:
            ids = self.model.prefill(prompt.to(self.model.device), self.st, valid_len, bucket)
        self.tokens.copy_(ids)
        return ids

    def capture_prefill(self, bucket: int) -> None:
        """Capture one prefill chunk of ``bucket`` tokens per row as a CUDA graph.
        Its start position is read from the state on the device and its per-row
        valid lengths from a static buffer, so the same graph replays at every
        chunk offset and pads the last chunk of a prompt to the bucket.  The
        state's cache must hold whole buckets (``max_seq`` >= the prompt rounded
        up to ``bucket``).  Warms up eagerly, captures, then resets the state."""
        if not self.use_graph or bucket in self._pf:
            return
        m, B = self.model, self.batch
        dev = m.device
        ids = torch.zeros(B, bucket, dtype=torch.long, device=dev)
        valid = torch.full((B,), bucket, dtype=torch.int32, device=dev)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            m.prefill_hidden(ids, self.st, valid)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        check_status("prefill warm-up")
        self.st.reset()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = m.prefill_hidden(ids, self.st, valid)
        torch.cuda.synchronize()
        self.st.reset()
        self._pf[bucket] = (g, ids, valid, out)

    def _prefill_graphed(self, prompt: torch.Tensor, valid_len: torch.Tensor | None, bucket: int) -> torch.Tensor:
        g, ids, valid, out = self._pf[bucket]
        dev = self.model.device
        prompt = prompt.to(dev)
        B, S = prompt.shape
        if B != self.batch:
            raise ValueError(f"prefill graph was captured for batch {self.batch}, got {B}")
        if -(-S // bucket) * bucket > self.max_seq:
            raise ValueError(f"prompt of {S} tokens in {bucket}-token chunks needs max_seq >= "
                             f"{-(-S // bucket) * bucket} (have {self.max_seq})")
        vl = (valid_len.to(dev) if valid_len is not None else torch.full((B,), S, device=dev)).int()
        h = torch.zeros_like(out)
        for c0 in range(0, S, bucket):
            n = min(S, c0 + bucket) - c0
            ids[:, :n].copy_(prompt[:, c0:c0 + n])
            if n < bucket:
                ids[:, n:].zero_()
            torch.clamp(vl - c0, 0, n, out=valid)
            g.replay()
            h = torch.where((valid > 0)[:, None], out, h)
        return self.model.greedy(h)

    # ----------------------------------------------------------------- step
    def _step_body(self) -> None:
        if self.sampling:
            ids = self.model.sample(self.model.decode_hidden(self.tokens, self.st), self.temperature, self.gen)
        else:
            ids = self.model.decode_step(self.tokens, self.st)
        self.next_ids.copy_(ids)
        self.tokens.copy_(ids)

    def capture(self) -> None:
        """Warm up one step eagerly (sizes kernel scratch), capture the decode step
        as a CUDA graph, then zero the state.  Call before :meth:`prefill`."""
        if not self.use_graph:
            return
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._step_body()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        check_status("decode warm-up")
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self._step_body()
        torch.cuda.synchronize()
        self.graph = g
        self.reset()
        self.tokens.zero_()

    def release(self) -> None:
        """Drop the graphs (must happen before destroying a process group whose
        collectives they captured)."""
        self.graph = None
        self._pf.clear()

    def step_device(self) -> None:
        """One decode step entirely on the device (input = previous ids)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._step_body()

    def step(self, host_tokens: torch.Tensor | None = None) -> torch.Tensor:
        """Public per-step API: H2D copy of ``host_tokens [B]`` (if given),
        one decode step, D2H of the next ids.  Returns a host int32 tensor."""
        if host_tokens is not None:
            self._host_in.copy_(host_tokens)
            self.tokens.copy_(self._host_in, non_blocking=True)
        self.step_device()
        self._host_out.copy_(self.next_ids, non_blocking=True)
        if self.model.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        return self._host_out.clone()

    def generate(self, prompt: torch.Tensor, steps: int, bucket: int = 0) -> torch.Tensor:
        """Greedy generation: prefill then ``steps`` device-side decode steps."""
        first = self.prefill(prompt, bucket=bucket)
        out = [first.clone()]
        for _ in range(steps - 1):
            self.step_device()
            out.append(self.next_ids.clone())
        check_status("generate")
        return torch.stack(out, 1)


def main(argv=None) -> None:
    """Greedy generation from the command line (the reference harness's
    ``main``: ``--prompt-ids`` coherence runs, ``--tiny`` random models, gen
    hash, prefill fingerprint and occupancy gates; ``contrib/qwen3.6-35b-a3b/
    static_decode_35b.py:2967-3530``, ``contrib/qwen3.6-27b/static_decode.py:1060-1479``).
    One process per GPU under torchrun for tensor parallelism.

        python -m bwn.runtime.static_decode --checkpoint HF_DIR --prompt-ids 760,6511,314,9338,369 --max-new 32
        python -m bwn.runtime.static_decode --model tiny --cpu --batch 2 --prompt-len 16
    """
    import argparse
    import json
    import time

    from ..config import QWEN36_27B, QWEN36_35B_A3B, tiny_qwen36
    from ..models.qwen36 import build_qwen36, from_pretrained
    from ..parallel.comm import init_distributed
    from ..utils import fingerprint as F

    # the reference harness's flag names are accepted as aliases (--batch-size, --num-layers,
    # --num-tokens, --model-path, --bucket-chunk, --fp8-weights, --tiny, --skip-compile)
    ap = argparse.ArgumentParser(description="static greedy decode")
    ap.add_argument("--model", default="tiny", choices=["27b", "35b", "tiny", "tiny-moe"])
    ap.add_argument("--tiny", dest="model", action="store_const", const="tiny", help="= --model tiny")
    ap.add_argument("--checkpoint", "--model-path", default="", help="HF safetensors directory (config.json beside it)")
    ap.add_argument("--layers", "--num-layers", type=int, default=0, help="truncate to this many layers")
    ap.add_argument("--prompt-ids", default="", help="comma-separated prompt token ids (every row)")
    ap.add_argument("--prompt", default="", help="prompt text, through the tokenizer (every row)")
    ap.add_argument("--tokenizer", default="", help="HF tokenizer directory (default: the checkpoint's, if any)")
    ap.add_argument("--prompt-len", type=int, default=16, help="uniform-random prompt length without --prompt-ids")
    ap.add_argument("--batch", "--batch-size", type=int, default=1)
    ap.add_argument("--max-new", "--num-tokens", type=int, default=16)
    ap.add_argument("--max-seq-len", type=int, default=0, help="KV / cache length (0: prompt + new tokens + 8)")
    ap.add_argument("--bucket", "--bucket-chunk", type=int, default=0, help="prefill chunk length (0: whole prompt)")
    ap.add_argument("--skip-prefill", action="store_true",
                    help="decode from the prompt's last token over an empty cache (decode-only runs)")
    ap.add_argument("--bench", action="store_true", help="after decode, time a synced TPOT window")
    ap.add_argument("--bench-iters", type=int, default=50, help="decode steps in the --bench window")
    ap.add_argument("--prefill-bench", type=int, default=0,
                    help="time the prefill of a synthetic N-token prompt (tok/s, TTFT) and exit")
    ap.add_argument("--prefill-bench-sweep", default="", help="comma-separated further lengths after --prefill-bench")
    ap.add_argument("--graph-splits", "--prefill-splits", type=int, default=0,
                    help="accepted for the reference's command lines; a CUDA graph needs no compile partitioning")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--fp8", "--fp8-weights", action="store_true", help="W8A16 projection weights")
    ap.add_argument("--fp8-experts", action="store_true",
                    help="MoE: routed experts in fp8 (an official FP8 checkpoint's stay fp8; random ones are quantized)")
    ap.add_argument("--fused-comm", action="store_true", help="N>1: fused NVLink reductions")
    ap.add_argument("--no-graph", "--skip-compile", action="store_true", help="eager steps, no CUDA graph")
    ap.add_argument("--prefill-gen", action="store_true",
                    help="also generate by re-prefilling the growing sequence each step (the reference's PREFILL_GEN "
                         "coherence check) and report whether it matches the decode path")
    ap.add_argument("--cpu", action="store_true")
    a = ap.parse_args(argv)

    cpu = a.cpu or not torch.cuda.is_available()
    comm = init_distributed("gloo" if cpu else "nccl")
    dev = torch.device("cpu") if cpu else torch.device("cuda", torch.cuda.current_device())
    dtype = torch.float32 if cpu else torch.bfloat16
    if a.checkpoint:
        model = from_pretrained(a.checkpoint, comm, dev, dtype, fp8_experts=a.fp8_experts)
    else:
        cfg = {"27b": QWEN36_27B, "35b": QWEN36_35B_A3B, "tiny": tiny_qwen36(),
               "tiny-moe": tiny_qwen36(moe=True)}[a.model]
        if a.layers:
            cfg = cfg.scaled(num_layers=a.layers)
        model = build_qwen36(cfg, comm, dev, seed=a.seed, dtype=dtype)
    if a.fp8:
        model.quantize_fp8()
    if a.fp8_experts and not a.checkpoint and model.cfg.is_moe:
        model.quantize_fp8(include_head=False, experts=True, dense=False)
    if a.fused_comm and comm.size > 1:
        from ..parallel.fused import enable_fused_comm
        enable_fused_comm(model)
    cfg = model.cfg

    def sync():
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)

    def finish():
        if comm.size > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()

    if a.prefill_bench:  # prompt-ingest throughput at each length, then exit
        lens = [a.prefill_bench] + [int(x) for x in a.prefill_bench_sweep.split(",") if x.strip()]
        g = torch.Generator().manual_seed(a.seed)
        for n in lens:
            ids = torch.randint(0, cfg.vocab, (a.batch, n), generator=g).to(dev)
            st = model.new_state(a.batch, n + 8)
            bucket = a.bucket or n
            times = []
            for _ in range(2):  # the first pass warms the kernels and allocator
                st.reset()
                sync()
                t0 = time.perf_counter()
                for c0 in range(0, n, bucket):
                    last = model.prefill_hidden(ids[:, c0:c0 + bucket], st, None)
                model.greedy(last)
                sync()
                times.append(comm.max_scalar(time.perf_counter() - t0, None if cpu else dev))
            del st
            if comm.rank == 0:
                print(json.dumps({"model": cfg.name, "tp": comm.size, "batch": a.batch, "prefill_tokens": n,
                                  "bucket": bucket, "ttft_ms": round(times[-1] * 1e3, 2),
                                  "prefill_tok_s": round(a.batch * n / times[-1], 1),
                                  "timing": "host clock around synchronize, max over ranks"}), flush=True)
        finish()
        return

    codec = None
    if a.prompt or a.tokenizer:
        from ..serve.api import load_tokenizer
        codec = load_tokenizer(a.tokenizer or a.checkpoint)
        if codec is None:
            raise SystemExit("no tokenizer found: give --tokenizer DIR, or a --checkpoint directory with tokenizer files")
    if a.prompt:
        prompt = torch.tensor([codec.encode(a.prompt)] * a.batch, dtype=torch.long)
    elif a.prompt_ids:
        ids = [int(t) for t in a.prompt_ids.split(",") if t.strip()]
        prompt = torch.tensor([ids] * a.batch, dtype=torch.long)
    else:
        prompt = torch.randint(0, cfg.vocab, (a.batch, a.prompt_len), generator=torch.Generator().manual_seed(a.seed))
    S = prompt.shape[1]
    steps_after = a.max_new + (a.bench_iters if a.bench else 0)
    max_seq = a.max_seq_len or (S + steps_after + 8)
    if max_seq < S + steps_after:
        raise SystemExit(f"--max-seq-len {max_seq} < prompt {S} + {steps_after} decode steps")
    dec = StaticDecoder(model, a.batch, max_seq, use_graph=not a.no_graph)
    dec.capture()

    sync()
    t0 = time.perf_counter()
    logits = None
    if a.skip_prefill:  # decode-only: the prompt's last token at position 0 of an empty cache
        first = prompt[:, -1].to(dev)
    else:
        bucket = a.bucket or S
        for c0 in range(0, S, bucket):  # bucketed prefill; the last chunk's hidden gives the logits
            last = model.prefill_hidden(prompt[:, c0:c0 + bucket].to(dev), dec.st, None)
        logits = model.logits(last)
        first = model.greedy(last)
    dec.tokens.copy_(first.to(dec.tokens.dtype))
    sync()
    ttft = (time.perf_counter() - t0) * 1e3
    out = [first.cpu()]
    t1 = time.perf_counter()
    for _ in range(a.max_new - 1):
        dec.step_device()
        out.append(dec.next_ids.clone().cpu())
    sync()
    tpot = (time.perf_counter() - t1) * 1e3 / max(1, a.max_new - 1)
    bench = None
    if a.bench:  # synced TPOT window: device time of bench_iters further steps, max over ranks
        if dev.type == "cuda":
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.bench_iters):
                dec.step_device()
            e1.record()
            sync()
            ms = e0.elapsed_time(e1)
        else:
            tb = time.perf_counter()
            for _ in range(a.bench_iters):
                dec.step_device()
            ms = (time.perf_counter() - tb) * 1e3
        ms = comm.max_scalar(ms, None if cpu else dev)
        bench = {"bench_iters": a.bench_iters, "bench_tpot_ms": round(ms / a.bench_iters, 4),
                 "bench_tok_s": round(a.batch * a.bench_iters * 1e3 / ms, 1)}
    check_status("static_decode")
    gen = torch.stack(out, 1)
    occupancy = F.check_qwen36_state(dec.st, f"decode state rank={comm.rank}")
    pgen = None
    if a.prefill_gen:  # every token from a fresh prefill of prompt + tokens so far
        seq = prompt.clone()
        toks = []
        for _ in range(a.max_new):
            st = model.new_state(a.batch, S + a.max_new + 8)
            nxt = model.greedy(model.prefill_hidden(seq.to(dev), st, None)).cpu()
            toks.append(nxt)
            seq = torch.cat([seq, nxt[:, None].long()], 1)
        pgen = torch.stack(toks, 1)
    if comm.rank == 0:
        print(json.dumps({
            "model": cfg.name, "tp": comm.size, "batch": a.batch, "prompt_len": S,
            "generated_row0": gen[0].tolist(), "gen_hash_row0": F.gen_hash(gen[0]),
            **({"text_row0": codec.decode(gen[0].tolist())} if codec is not None else {}),
            "prefill_fingerprint": F.logits_fingerprint(logits.float().cpu()) if logits is not None else None,
            "ttft_ms": round(ttft, 2), "tpot_ms": round(tpot, 3),
            "occupied_ssm_layers": len(occupancy["ssm"]), "graph": dec.graph is not None,
            "skip_prefill": a.skip_prefill, **(bench or {}),
            **({"prefill_gen_hash_row0": F.gen_hash(pgen[0]), "prefill_gen_matches": bool(torch.equal(pgen, gen))}
               if pgen is not None else {})}))
    dec.release()
    finish()


if __name__ == "__main__":
    main()
