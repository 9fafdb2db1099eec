"""Run fingerprints and state guards.

* :func:`gen_hash` -- the reference's ``gen hash``: the first 12 hex digits of
  the MD5 of ``str(list_of_ids)`` (``contrib/qwen3.6-35b-a3b/static_decode_35b.py:3513-3520``),
  kept byte-identical so hashes can be compared across implementations.
* :func:`logits_fingerprint` -- sum, norm, top-5 and finiteness of prefill
  logits (``static_decode_35b.py:3222-3246``).
* :func:`state_stats` -- sum / norm / non-zero count of carried state tensors.
* :func:`snapshot_state` / :func:`assert_state_advanced`: every per-layer
  state buffer must change on every decode step (each DeltaNet layer's
  recurrent state and conv ring slot, each attention layer's K/V row at the
  step's position) -- the static-buffer form of the reference's in-place
  mutation lesson.
* Guards (``static_decode_35b.py:549-659``): :func:`assert_disjoint` rejects two
  in-place-mutated buffers whose bytes overlap; :func:`assert_occupancy` rejects
  a per-layer state slice with no non-zero row after a step (a dropped write
  that greedy ids and finiteness do not reveal).  With CUDA graphs over static
  buffers, per-layer slices of one stacked tensor are legal (each kernel writes
  its own slice), so the distinctness guard compares byte ranges rather than
  storages.
"""
from __future__ import annotations

import hashlib
import os

import torch


def gen_hash(ids) -> str:
    ids = [int(i) for i in (ids.tolist() if isinstance(ids, torch.Tensor) else ids)]
    return hashlib.md5(str(ids).encode()).hexdigest()[:12]


def logits_fingerprint(logits: torch.Tensor, k: int = 5) -> dict:
    lf = logits.float()
    row = lf.reshape(-1, lf.shape[-1])[0]
    return {
        "sum": float(lf.sum()),
        "norm": float(torch.linalg.vector_norm(lf)),
        "top5": [int(v) for v in torch.topk(row, min(k, row.numel())).indices],
        "finite": bool(torch.isfinite(lf).all()),
    }


def state_stats(t: torch.Tensor) -> dict:
    tf = t.float()
    return {"sum": float(tf.sum()), "norm": float(torch.linalg.vector_norm(tf)),
            "nz": int((t != 0).sum()), "numel": t.numel(), "finite": bool(torch.isfinite(tf).all())}


def _span(t: torch.Tensor) -> tuple[int, int]:
    """Byte range ``[lo, hi)`` a (possibly strided) tensor can touch."""
    if t.numel() == 0:
        p = t.data_ptr()
        return p, p
    lo = t.data_ptr()
    hi = lo + sum((s - 1) * st for s, st in zip(t.shape, t.stride())) * t.element_size() + t.element_size()
    return lo, hi


def assert_disjoint(tensors, what: str = "buffers") -> int:
    """Precondition: no two mutated buffers overlap in memory."""
    spans = sorted((_span(t) + (i,)) for i, t in enumerate(tensors) if t.numel())
    for (lo0, hi0, i0), (lo1, hi1, i1) in zip(spans, spans[1:]):
        if lo1 < hi0:
            raise RuntimeError(f"{what}: buffers {i0} and {i1} overlap (bytes 0x{lo1:x}..0x{min(hi0, hi1):x}); "
                               "each in-place-updated buffer needs its own memory")
    return len(spans)


def nonzero_rows(t: torch.Tensor) -> int:
    return int((t.reshape(-1, t.shape[-1]) != 0).any(dim=-1).sum())


def assert_occupancy(per_layer, what: str, min_rows: int = 1, env: str = "BWN_OCCUPANCY_CHECK") -> list[int]:
    """Postcondition: every per-layer slice holds at least ``min_rows`` non-zero rows."""
    if os.environ.get(env, "1") != "1":
        return []
    parts = list(per_layer) if isinstance(per_layer, (list, tuple)) else [per_layer[i] for i in range(per_layer.shape[0])]
    rows = [nonzero_rows(t) for t in parts]
    empty = [i for i, n in enumerate(rows) if n < min_rows]
    if empty:
        raise RuntimeError(f"{what}: layers {empty} of {len(parts)} hold fewer than {min_rows} non-zero rows "
                           f"(per-layer non-zero rows {rows}): their state writes were lost")
    return rows


def check_qwen36_state(st, what: str = "decode state", kv_rows_used: bool = True) -> dict:
    """Distinctness + occupancy gates over a :class:`~bwn.models.qwen36.Qwen36State`."""
    bufs = [st.conv[i] for i in range(st.conv.shape[0])] + [st.ssm[i] for i in range(st.ssm.shape[0])]
    bufs += [st.k_cache[i] for i in range(st.k_cache.shape[0])] + [st.v_cache[i] for i in range(st.v_cache.shape[0])]
    bufs.append(st.positions)
    assert_disjoint(bufs, what)
    out = {"ssm": assert_occupancy(st.ssm, what + " ssm"), "conv": assert_occupancy(st.conv, what + " conv")}
    if kv_rows_used:
        out["k"] = assert_occupancy(st.k_cache, what + " k_cache")
        out["v"] = assert_occupancy(st.v_cache, what + " v_cache")
    return out


def snapshot_state(st) -> dict:
    """Copies of the state slices one decode step must write (taken before the step)."""
    pos = st.positions.long()
    b = torch.arange(pos.shape[0], device=pos.device)
    R = st.conv.shape[2]
    return {"pos": pos.clone(), "ssm": st.ssm.clone(), "conv": st.conv[:, b, pos % R].clone(),
            "k": _kv_rows(st.k_cache, b, pos).clone(), "v": _kv_rows(st.v_cache, b, pos).clone()}


def _kv_rows(cache: torch.Tensor, b: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    """``cache [L, B, KVH, S, D]`` -> the row at each sequence's position, ``[L, B, KVH, D]``."""
    return cache.transpose(2, 3)[:, b, pos]


def assert_state_advanced(before: dict, st, what: str = "decode step") -> None:
    """Postcondition of one decode step: the positions moved by one, and for
    every sequence each DeltaNet layer's recurrent state and conv-ring slot and
    each attention layer's K/V row at the step's position changed."""
    pos = before["pos"]
    if not torch.equal(st.positions.long(), pos + 1):
        raise RuntimeError(f"{what}: positions did not advance by one")
    b = torch.arange(pos.shape[0], device=pos.device)
    R = st.conv.shape[2]
    now = {"ssm": st.ssm, "conv": st.conv[:, b, pos % R], "k": _kv_rows(st.k_cache, b, pos),
           "v": _kv_rows(st.v_cache, b, pos)}
    for name, cur in now.items():
        old = before[name]
        # [L, B, ...]: per layer and sequence, did anything change
        same = (cur == old).reshape(cur.shape[0], cur.shape[1], -1).all(-1)
        if bool(same.any()):
            lay, seq = [int(v) for v in same.nonzero()[0]]
            raise RuntimeError(f"{what}: {name} of layer {lay} (sequence {seq}) was not written")
