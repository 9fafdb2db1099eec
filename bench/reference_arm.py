"""Reference arm of ``bench.py``: the unmodified reference's Qwen3.6-35B-A3B
harness run on CUDA (one process per GPU, NCCL), on the same model and config
as the bwn arm.

What runs is the reference's own code, as installed under ``baseline/_ref``:

* ``load_sharded_weights`` (``contrib/qwen3.6-35b-a3b/static_decode_35b.py:2682``)
  shards the checkpoint for this rank with its own colwise / rowwise / group-aware
  / KV-replication / expert-parallel rules;
* ``StaticDecode35B`` (``:836``) with its default flags: pure-torch DeltaNet
  recurrence (``deltanet_recurrent_step``), masked-dense expert-parallel MoE,
  torch attention over the whole cache, ``functional_all_reduce`` over the
  default (NCCL) process group;
* ``decode_step`` (``:1532``) driven as its ``--bench`` loop drives it
  (``:3482-3498``): functional state threaded through, constant position.

There is no checkpoint on the box (no network), so the safetensors reader the
loader imports (``st_reader``) is served from memory: every tensor name the HF
Qwen3.6-35B-A3B layout has, with the random-init values ``bwn`` itself uses
(:func:`bwn.io.qwen36_weights.synthetic_hf_layer`, seed 0), generated on the
rank's GPU one layer at a time and handed to the loader in bf16 like a bf16
checkpoint.  Nothing else of ``bwn`` is on this path: no bwn model, kernel,
engine or extension is imported.  The KV caches and recurrent states are
filled with random values as a 2048-token prefill would leave them (the
reference's decode cost depends on the cache length, not the values), and the
position is 2048.
"""
from __future__ import annotations

import json
import os
import statistics
import sys
import tempfile
import time
import types

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "baseline", "_ref", "neuron_pytorch_native_ref", "contrib", "qwen3.6-35b-a3b")


def hf_config(cfg) -> dict:
    """The HF ``config.json`` text_config keys the reference's
    ``model_dims.load_from_config`` reads, for a :class:`bwn.config.Qwen36Config`."""
    return {"text_config": {
        "num_hidden_layers": cfg.num_layers, "full_attention_interval": cfg.full_attn_interval,
        "hidden_size": cfg.hidden, "vocab_size": cfg.vocab, "rms_norm_eps": cfg.rms_eps,
        "head_dim": cfg.head_dim, "partial_rotary_factor": cfg.partial_rotary, "rope_theta": cfg.rope_theta,
        "linear_num_key_heads": cfg.dn_k_heads, "linear_num_value_heads": cfg.dn_v_heads,
        "linear_key_head_dim": cfg.dn_k_dim, "linear_value_head_dim": cfg.dn_v_dim,
        "linear_conv_kernel_dim": cfg.conv_kernel, "num_attention_heads": cfg.q_heads,
        "num_key_value_heads": cfg.kv_heads, "attn_output_gate": True, "num_experts": cfg.num_experts,
        "num_experts_per_tok": cfg.top_k, "moe_intermediate_size": cfg.moe_inter,
        "normalize_top_k_affinities": cfg.norm_topk_prob, "shared_expert_intermediate_size": cfg.shared_inter},
        "tie_word_embeddings": cfg.tie_embeddings}


class SyntheticCheckpoint:
    """An HF-layout checkpoint held in memory: ``names()`` lists every tensor,
    ``get(name)`` generates it (one layer at a time, cached) in ``dtype``."""

    def __init__(self, cfg, seed: int, device, dtype=torch.bfloat16):
        from bwn.io.qwen36_weights import synthetic_hf_global, synthetic_hf_global_names, synthetic_hf_layer
        self.cfg, self.seed, self.device, self.dtype = cfg, seed, torch.device(device), dtype
        self._layer_fn, self._global_fn = synthetic_hf_layer, synthetic_hf_global
        self._cache_idx, self._cache = None, {}
        # the tensor names of each layer type, read off a miniature of the config
        tiny = cfg.scaled(num_layers=cfg.full_attn_interval, hidden=8, vocab=8, num_experts=min(cfg.num_experts, 2),
                          moe_inter=8, shared_inter=8, intermediate=8 if cfg.intermediate else 0, dn_k_heads=1,
                          dn_v_heads=1, q_heads=1, kv_heads=1, head_dim=8, dn_k_dim=8, dn_v_dim=8)
        suffix = {}
        for i in range(cfg.full_attn_interval):
            t = cfg.layer_type(i)
            if t not in suffix:
                suffix[t] = [k.split(".", 2)[2] for k in synthetic_hf_layer(tiny, i, seed, "cpu")]
        self._names = [f"layers.{i}.{s}" for i in range(cfg.num_layers) for s in suffix[cfg.layer_type(i)]]
        self._names += synthetic_hf_global_names(cfg)

    def names(self) -> list[str]:
        return list(self._names)

    def _cast(self, t: torch.Tensor) -> torch.Tensor:
        return t.to(self.dtype) if t.is_floating_point() else t

    def get(self, name: str) -> torch.Tensor:
        if name.startswith("layers."):
            i = int(name.split(".")[1])
            if self._cache_idx != i:
                self._cache = {}  # free the previous layer before making the next
                self._cache = self._layer_fn(self.cfg, i, self.seed, self.device)
                self._cache_idx = i
            return self._cast(self._cache[name])
        return self._cast(self._global_fn(self.cfg, name, self.seed, self.device))


def install_reader(ckpt: SyntheticCheckpoint) -> None:
    """Serve the loader's ``st_reader`` imports (``build_weight_map``,
    ``SafeReader``; ``st_reader.py:31-81``) from ``ckpt``."""
    mod = types.ModuleType("st_reader")

    class SafeReader:
        def __init__(self, path):
            self.path = path

        def get_tensor(self, key):
            return ckpt.get(key)

        def close(self):
            pass

    mod.SafeReader = SafeReader
    mod.build_weight_map = lambda path: {k: "synthetic.safetensors" for k in ckpt.names()}
    sys.modules["st_reader"] = mod


def import_reference(cfg):
    """Import the reference harness from ``baseline/_ref`` and set its model
    dims from ``cfg`` through its own ``load_from_config``."""
    if not os.path.isfile(os.path.join(REF_DIR, "static_decode_35b.py")):
        raise FileNotFoundError(f"reference not installed: {os.path.join(REF_DIR, 'static_decode_35b.py')} is missing")
    for p in (os.path.join(REF_DIR, "kernels"), REF_DIR):
        if p not in sys.path:
            sys.path.insert(0, p)
    import model_dims as D
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "config.json")
        with open(path, "w") as f:
            json.dump(hf_config(cfg), f)
        D.load_from_config(path)
    import static_decode_35b as S
    return D, S


def build_reference(cfg, rank: int, world: int, batch: int, max_seq: int, device, seed: int = 0,
                    dtype=torch.bfloat16):
    """The reference's module for this rank (``load_sharded_weights`` +
    ``StaticDecode35B``) on ``device``, and its zero decode state in the layout
    its ``main`` allocates (``static_decode_35b.py:3099-3113``)."""
    D, S = import_reference(cfg)
    ckpt = SyntheticCheckpoint(cfg, seed, device, dtype)
    install_reader(ckpt)
    weights = S.load_sharded_weights("synthetic", rank, world, num_layers=D.NUM_LAYERS)
    mod = S.StaticDecode35B(weights, max_seq, world, batch_size=batch, rank=rank)
    del weights, ckpt
    mod = mod.to(device).eval()
    td = D.tp_dims(world)
    vh = td["dn_v_heads"]
    qkv_dim = 2 * td["dn_k_heads"] * D.DN_K_DIM + vh * D.DN_V_DIM
    nkv = max(1, D.GQA_KV_HEADS // world)
    st = {
        "dn": torch.zeros(D.NUM_DELTANET, batch, vh * D.DN_K_DIM, D.DN_V_DIM, dtype=dtype, device=device),
        "conv": torch.zeros(D.NUM_DELTANET, batch, qkv_dim, D.DN_CONV_KERNEL - 1, dtype=dtype, device=device),
        "k": torch.zeros(D.NUM_GQA, batch, nkv, max_seq, D.GQA_HEAD_DIM, dtype=dtype, device=device),
    }
    st["v"] = torch.zeros_like(st["k"])
    return mod, st


def run(args, metric: str, baseline_tok_s: float) -> None:
    """``bench.py --impl reference``: prints one JSON line (rank 0)."""
    from bwn.config import QWEN36_35B_A3B
    rank0 = int(os.environ.get("RANK", "0")) == 0
    cfg = QWEN36_35B_A3B if not args.layers else QWEN36_35B_A3B.scaled(num_layers=args.layers)
    if args.model != "35b":
        if rank0:
            print(json.dumps({"impl": "reference", "metric": metric, "n_gpus": args.gpus, "unavailable":
                              "the reference's Qwen3.6-27B decode needs its NKI kernels (contrib/qwen3.6-27b/"
                              "static_decode.py:29-34, 834); its torch path exists for the 35B-A3B harness only"}))
        return
    if not os.path.isfile(os.path.join(REF_DIR, "static_decode_35b.py")):
        if rank0:
            print(json.dumps({"impl": "reference", "metric": metric, "n_gpus": args.gpus,
                              "unavailable": f"reference not installed: {REF_DIR}/static_decode_35b.py missing"}))
        return
    import datetime

    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    rank = dist.get_rank() if world > 1 else 0
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    B, S = args.batch, args.prompt_len
    max_seq = S + 64
    t_load = time.perf_counter()
    with torch.no_grad():
        mod, st = build_reference(cfg, rank, world, B, max_seq, dev)
    load_s = time.perf_counter() - t_load
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    # the state a 2048-token prefill leaves: cache rows [0, S) and recurrent states filled
    st["k"][:, :, :, :S].normal_(generator=g)
    st["v"][:, :, :, :S].normal_(generator=g)
    st["dn"].normal_(0, 0.05, generator=g)
    st["conv"].normal_(generator=g)
    position = torch.tensor(S, dtype=torch.long, device=dev)
    gt = torch.Generator().manual_seed(1234)
    ids = torch.randint(0, cfg.vocab, (B,), generator=gt).to(dev)
    state = [st["dn"], st["conv"], st["k"], st["v"]]
    del st

    def step(x):
        _, nxt, dn, cv, kk, vv = mod.decode_step(x, position, *state)
        state[:] = [dn, cv, kk, vv]
        return nxt

    from bwn.utils.clocks import ClockSampler, job_gpu_ids
    with torch.no_grad():
        for _ in range(args.warmup):
            ids = step(ids)
        torch.cuda.synchronize()
        sampler = ClockSampler(job_gpu_ids(world)) if local == 0 else None
        if sampler is not None:
            sampler.__enter__()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            ids = step(ids)
        e1.record()
        torch.cuda.synchronize()
        if sampler is not None:
            sampler.__exit__(None, None, None)
        barrier()
        total_ms = max_over_ranks(e0.elapsed_time(e1))
        # per-step TPOT distribution (events between steps; not the headline)
        n_p = min(args.steps, 16)
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(n_p + 1)]
        barrier()
        evs[0].record()
        for i in range(n_p):
            ids = step(ids)
            evs[i + 1].record()
        torch.cuda.synchronize()
        p50 = max_over_ranks(statistics.median(evs[i].elapsed_time(evs[i + 1]) for i in range(n_p)))
        # end to end: pinned H2D of the step's ids and D2H of the next ids every step
        host_in = ids.to(torch.int64).cpu().pin_memory()
        host_out = torch.empty_like(host_in).pin_memory()
        barrier()
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        for _ in range(args.steps):
            x = host_in.to(dev, non_blocking=True)
            nxt = step(x)
            host_out.copy_(nxt, non_blocking=True)
            torch.cuda.synchronize()
            host_in.copy_(host_out)
        e2e_ms = max_over_ranks((time.perf_counter() - h0) * 1e3)
    value = B * args.steps / (total_ms / 1e3)
    if rank == 0:
        out = {
            "impl": "reference",
            "metric": metric,
            "value": round(value, 2),
            "unit": "decode tokens/s (whole job)",
            "n_gpus": args.gpus,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": round(value / baseline_tok_s, 3) if baseline_tok_s else None,
            "dtype": "bf16",
            "data": "synthetic (uniform-random ids, random-init weights seed 0 in the HF layout through the "
                    "reference's own loader; caches/states filled as after a 2048-token prefill)",
            "config": {
                "model": cfg.name if not args.layers else f"{cfg.name}-{args.layers}L (INVALID: debug layer count)",
                "global_batch": B, "seq_len": S, "parallelism": f"tp{args.gpus}+ep{args.gpus}",
                "decode": "reference StaticDecode35B.decode_step, eager torch (default flags: torch DeltaNet "
                          "recurrence, masked-dense EP MoE, functional all-reduce over NCCL)",
                "l2": "inputs larger than L2 (every step streams every local expert)",
                "source": os.path.relpath(os.path.join(REF_DIR, "static_decode_35b.py"), ROOT),
            },
            "tpot_p50_ms": round(p50, 4),
            "context": "synthetic-kv",
            "clocks": sampler.summary() if sampler is not None else None,
            "e2e": {"value": round(B * args.steps / (e2e_ms / 1e3), 2),
                    "unit": "decode tokens/s (decode_step with pinned H2D of ids and D2H of next ids per step)",
                    "h2d_bytes_per_step": B * 8, "d2h_bytes_per_step": B * 8},
            "gpu_launches": 0,
            "weights_load_s": round(load_s, 1),
        }
        print(json.dumps(out))
    if world > 1:
        dist.destroy_process_group()
