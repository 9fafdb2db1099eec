"""Per-layer decode diagnostics, captures and capture comparison.

The reference exposes a diagnostic decode step whose graph outputs are the
per-layer stages of selected layers (``decode_step_diagnostics``,
``contrib/qwen3.6-35b-a3b/static_decode_35b.py:1630-1786``) and a device test
that saves per-rank captures in one run and compares them with another run's:
logits cosine >= 0.999 and relative L2 <= 0.05, greedy-id mismatches accepted
only when both runs see a near tie (``kernels/tests/test_decode_fullgraph_device.py:87-192,
255-275``).  Here:

* :func:`decode_diagnostics` walks one decode step eagerly with plain
  collectives (no fused NVLink kernels, no CUDA graph) and records, for the
  selected layers, the residual stream entering the layer (``input``), the
  token mixer's output before its projection (``mixer``), the reduced
  projection (``attn``), the residual after it (``post_attn``), the normed
  MLP / MoE input (``moe_in``), the router's ids and weights, this rank's
  routed-expert partial (``routed_local``), the reduced routed and shared
  expert outputs (``routed``, ``shared``), the reduced MLP output (``mlp``)
  and the residual leaving the layer (``output``); it advances the state
  exactly as :meth:`~bwn.models.qwen36.Qwen36Model.decode_hidden` does;
* :func:`save_capture` / :func:`load_captures` keep one file per rank;
* :func:`compare_captures` reports per-layer, per-tap cosine / relative L2 /
  max-abs and applies the logits and near-tie gates.

    python -m bwn.runtime.diagnostics capture --model 35b --layers 0,3,39 --out RUN_A   # per rank (torchrun)
    python -m bwn.runtime.diagnostics compare RUN_A RUN_B
"""
from __future__ import annotations

import glob
import json
import os

import torch

from .. import ops as O


def _reduce(model, part: torch.Tensor) -> torch.Tensor:
    if model.tp > 1:
        model.comm.all_reduce_(part)
    return part


@torch.no_grad()
def decode_diagnostics(model, tokens: torch.Tensor, st, layers=None) -> dict:
    """One decode step of ``tokens [B]`` with per-layer taps (``layers``:
    indices to record, all when ``None``).  Returns ``{"layers": {i: {tap:
    tensor}}, "hidden", "logits" (this rank's vocab shard, fp32), "next_id"}``."""
    cfg, d = model.cfg, model.d
    sel = set(range(cfg.num_layers) if layers is None else layers)
    out: dict = {"layers": {}}
    x = model.embed(tokens)
    h = O.rms_norm(x, model.layers[0]["in_norm"], cfg.rms_eps)
    di = gi = 0
    for i in range(cfg.num_layers):
        L = model.layers[i]
        rec: dict = {}
        if i in sel:
            rec["input"] = x.clone()
        if cfg.layer_type(i) == "deltanet":
            o = model._deltanet_decode(i, h, st, di)
            w = L["out_proj"]
            di += 1
        else:
            o = model._gqa_decode(i, h, st, gi)
            w = L["o_proj"]
            gi += 1
        attn = _reduce(model, O.linear(o, w))
        if i in sel:
            rec["mixer"], rec["attn"] = o.clone(), attn.clone()
        h = O.add_rms_norm(attn, x, L["post_norm"], cfg.rms_eps)
        if i in sel:
            rec["post_attn"], rec["moe_in"] = x.clone(), h.clone()
        nxt = model.layers[i + 1]["in_norm"] if i + 1 < cfg.num_layers else model.g["final_norm"]
        if cfg.is_moe:
            from ..models.moe import route
            wr, ids = route(model, L, h)
            routed_local = O.moe_experts(h, wr, ids, L["experts_gate_up"], L["experts_down"], d.expert_offset)
            sy = O.linear(O.linear_swiglu(h, L["shared_gate_up"]), L["shared_down"])
            sg = O.linear_f32(h, L["shared_gate"])
            shared = _reduce(model, (torch.sigmoid(sg.float().reshape(-1, 1)) * sy.float()).to(h.dtype))
            routed = _reduce(model, routed_local.clone())
            mlp = (routed.float() + shared.float()).to(h.dtype)
            if i in sel:
                rec.update(router_ids=ids.clone(), router_w=wr.clone(), routed_local=routed_local,
                           routed=routed, shared=shared)
        else:
            mlp = _reduce(model, O.linear(O.linear_swiglu(h, L["gate_up"]), L["down"]))
        if i in sel:
            rec["mlp"] = mlp.clone()
        h = O.add_rms_norm(mlp, x, nxt, cfg.rms_eps)
        if i in sel:
            rec["output"] = x.clone()
            out["layers"][i] = rec
    st.positions.add_(1)
    out["hidden"] = h
    out["logits"] = O.linear_f32(h, model.g["lm_head"])
    out["next_id"] = model.greedy(h)
    return out


# ------------------------------------------------------------------ captures
def _cpu(v):
    if torch.is_tensor(v):
        return v.detach().cpu()
    if isinstance(v, dict):
        return {k: _cpu(x) for k, x in v.items()}
    return v


def save_capture(cap: dict, out_dir: str, rank: int = 0, meta: dict | None = None) -> str:
    os.makedirs(out_dir, exist_ok=True)
    path = os.path.join(out_dir, f"capture_rank{rank}.pt")
    torch.save({"meta": meta or {}, **_cpu(cap)}, path)
    return path


def load_captures(run_dir: str) -> list[dict]:
    """The run's per-rank captures, in rank order."""
    paths = sorted(glob.glob(os.path.join(run_dir, "capture_rank*.pt")),
                   key=lambda p: int(p.rsplit("rank", 1)[1].split(".")[0]))
    if not paths:
        raise FileNotFoundError(f"no capture_rank*.pt under {run_dir}")
    return [torch.load(p, map_location="cpu", weights_only=False) for p in paths]


def global_logits(caps: list[dict], width: int | None = None) -> torch.Tensor:
    """Full-vocabulary logits: the vocab shards of every rank concatenated (or
    rank 0's when it already holds ``width`` columns)."""
    first = caps[0]["logits"].float()
    if width is not None and first.shape[-1] == width:
        return first
    return torch.cat([c["logits"].float() for c in caps], dim=-1)


def near_tie_mismatches(ref_logits, ref_ids, cand_logits, cand_ids, tol: float):
    """Rows whose greedy ids differ are accepted only when both runs rank the
    two ids within ``tol`` of each other.  Returns ``(rejected_rows, details)``
    with ``details = [(row, ref_id, cand_id, ref_margin, cand_margin, accepted)]``."""
    rejected, details = [], []
    for row in (cand_ids != ref_ids).nonzero().reshape(-1).tolist():
        r, c = int(ref_ids[row]), int(cand_ids[row])
        rm = float(ref_logits[row, r] - ref_logits[row, c])
        cm = float(cand_logits[row, c] - cand_logits[row, r])
        ok = abs(rm) <= tol and abs(cm) <= tol
        if not ok:
            rejected.append(row)
        details.append((row, r, c, rm, cm, ok))
    return rejected, details


def similarity(a: torch.Tensor, b: torch.Tensor) -> dict:
    a, b = a.float().reshape(-1), b.float().reshape(-1)
    diff = a - b
    na, nb = torch.linalg.vector_norm(a), torch.linalg.vector_norm(b)
    cos = float((a @ b) / (na * nb).clamp_min(1e-30)) if a.numel() else 1.0
    if float(na) == 0.0 and float(nb) == 0.0:
        cos = 1.0
    return {"cosine": cos, "rel_l2": float(torch.linalg.vector_norm(diff) / na.clamp_min(1e-12)),
            "max_abs": float(diff.abs().max()) if diff.numel() else 0.0}


# taps that every rank holds in full (the others are this rank's shard)
REPLICATED_TAPS = ("input", "attn", "post_attn", "moe_in", "router_ids", "router_w", "routed", "shared", "mlp",
                   "output")


def compare_captures(ref: list[dict], cand: list[dict], cos_min: float = 0.999, rel_l2_max: float = 0.05,
                     tie_tol: float = 0.125) -> dict:
    """Compare two runs' per-rank captures (``ref`` is the expected run).
    With equal rank counts every tap is compared rank by rank; otherwise (e.g.
    TP1 against TP8) rank 0's replicated taps are.  Router ids compare as
    sets per token, everything else by cosine / relative L2 (relative to the
    reference); the logits gate uses the global logits."""
    same = len(ref) == len(cand)
    pairs = list(zip(ref, cand)) if same else [(ref[0], cand[0])]
    taps = {}
    first_bad = None
    for rank, (r, c) in enumerate(pairs):
        for i in sorted(set(r["layers"]) & set(c["layers"])):
            for tap in sorted(set(r["layers"][i]) & set(c["layers"][i])):
                if not same and tap not in REPLICATED_TAPS:
                    continue
                a, b = r["layers"][i][tap], c["layers"][i][tap]
                key = f"rank{rank}/layer{i}/{tap}"
                if tap == "router_ids":
                    taps[key] = {"match": float((a.sort(-1).values == b.sort(-1).values).float().mean())}
                else:
                    taps[key] = similarity(a, b)
                    if first_bad is None and taps[key]["cosine"] < cos_min:
                        first_bad = key
    cl = global_logits(cand)
    rl = global_logits(ref, cl.shape[-1])
    logits = similarity(rl, cl)
    rejected, details = near_tie_mismatches(rl, ref[0]["next_id"], cl, cand[0]["next_id"], tie_tol)
    ok = logits["cosine"] >= cos_min and logits["rel_l2"] <= rel_l2_max and not rejected
    return {"ok": ok, "logits": logits, "id_mismatches": details, "rejected_rows": rejected,
            "first_diverging_tap": first_bad, "taps": taps}


def capture_run(a) -> str:
    """Build the model (random init from ``--seed``; one rank per process under
    torchrun), prefill a seeded prompt, run one tapped decode step and save
    this rank's capture."""
    from ..config import QWEN36_27B, QWEN36_35B_A3B, tiny_qwen36
    from ..models.qwen36 import build_qwen36
    from ..parallel.comm import init_distributed
    cpu = a.cpu or not torch.cuda.is_available()
    comm = init_distributed("gloo" if cpu else "nccl")
    dev = torch.device("cpu") if cpu else torch.device("cuda", torch.cuda.current_device())
    cfg = {"27b": QWEN36_27B, "35b": QWEN36_35B_A3B, "tiny": tiny_qwen36(), "tiny-moe": tiny_qwen36(moe=True)}[a.model]
    if a.layers_total:
        cfg = cfg.scaled(num_layers=a.layers_total)
    model = build_qwen36(cfg, comm, dev, seed=a.seed, dtype=torch.float32 if cpu else torch.bfloat16,
                         moe_sharding=a.moe_sharding)
    gen = torch.Generator().manual_seed(a.seed + 1)
    prompt = torch.randint(0, cfg.vocab, (a.batch, a.prompt_len), generator=gen).to(dev)
    st = model.new_state(a.batch, a.prompt_len + 8)
    ids = model.greedy(model.prefill_hidden(prompt, st))
    layers = [int(v) for v in a.layers.split(",")] if a.layers else None
    cap = decode_diagnostics(model, ids.int(), st, layers)
    meta = {"model": cfg.name, "world": comm.size, "rank": comm.rank, "seed": a.seed, "batch": a.batch,
            "prompt_len": a.prompt_len, "moe_sharding": a.moe_sharding, "device": str(dev)}
    path = save_capture(cap, a.out, comm.rank, meta)
    if comm.size > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return path


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="per-rank decode captures and their comparison")
    sub = ap.add_subparsers(dest="cmd", required=True)
    k = sub.add_parser("capture")
    k.add_argument("--model", default="tiny", choices=["27b", "35b", "tiny", "tiny-moe"])
    k.add_argument("--layers-total", type=int, default=0, help="truncate the model to this many layers")
    k.add_argument("--layers", default="", help="comma-separated layers to tap (all when empty)")
    k.add_argument("--batch", type=int, default=2)
    k.add_argument("--prompt-len", type=int, default=16)
    k.add_argument("--seed", type=int, default=0)
    k.add_argument("--moe-sharding", default="ep", choices=["ep", "tp"])
    k.add_argument("--cpu", action="store_true")
    k.add_argument("--out", required=True)
    c = sub.add_parser("compare")
    c.add_argument("reference")
    c.add_argument("candidate")
    c.add_argument("--cos-min", type=float, default=0.999)
    c.add_argument("--rel-l2-max", type=float, default=0.05)
    c.add_argument("--tie-tol", type=float, default=0.125)
    c.add_argument("--report-only", action="store_true")
    a = ap.parse_args(argv)
    if a.cmd == "capture":
        print(json.dumps({"saved": capture_run(a)}))
        return 0
    rep = compare_captures(load_captures(a.reference), load_captures(a.candidate), a.cos_min, a.rel_l2_max,
                           a.tie_tol)
    print(json.dumps({k: v for k, v in rep.items() if k != "taps"}))
    return 0 if rep["ok"] or a.report_only else 1


if __name__ == "__main__":
    raise SystemExit(main())
