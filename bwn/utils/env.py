"""Environment overrides, declared and validated in one place.

The reference reads ~60 module-level env flags at import, with import-time
mutual-exclusion guards (``contrib/qwen3.6-35b-a3b/static_decode_35b.py:50-498``).
bwn keeps model dims in typed configs and run options on the command line; the
few A/B levers that must reach code far from the CLI are env flags declared
here, each with a type, a default and a check, and :func:`validate` rejects
unknown ``BWN_*`` names and illegal combinations before anything runs.
"""
from __future__ import annotations

import os
from dataclasses import dataclass


@dataclass(frozen=True)
class Flag:
    name: str
    kind: type
    default: object
    help: str
    choices: tuple | None = None


FLAGS = {f.name: f for f in (
    Flag("BWN_PDL", int, 1, "programmatic dependent launch between bwn kernels (read by the C++ launcher)", (0, 1)),
    Flag("BWN_FUSED_COMM", str, "auto", "fused NVLink compute+collective kernels", ("auto", "on", "off")),
    Flag("BWN_NO_REDUCE", int, 0, "cost probe: turn every tensor-parallel all-reduce into a no-op (wrong results)", (0, 1)),
    Flag("BWN_PROFILE_STEPS", int, 0, "run warm-up, then N constant-token decode steps for a profiler, then exit"),
    Flag("BWN_NVTX", int, 0, "emit NVTX ranges per layer and per op", (0, 1)),
    Flag("BWN_OCCUPANCY_CHECK", int, 1, "per-layer state occupancy gates after generation", (0, 1)),
    Flag("BWN_DEBUG", int, 0, "build kernels with device-side bounds checks (build-time)", (0, 1)),
    Flag("BWN_METRICS", str, "", "path of a JSONL metrics file"),
    Flag("BWN_WAIT_LIMIT_MS", int, 2000, "bound on every device-side wait before it reports a timeout"),
    Flag("BWN_GQA_TC", int, 1, "GQA decode on the tcgen05 kernel (0: CUDA-core kernel)", (0, 1)),
    Flag("BWN_GEMM_SMALL_RING", int, 1, "decode GEMMs with short K ranges on a 4-stage ring (two CTAs per SM, so the "
         "next kernel's weight prefetch overlaps)", (0, 1)),
    Flag("BWN_GEMM_MAX_SPLITS", int, 16, "upper bound of the decode GEMMs' split-K factor (1..16)"),
    Flag("BWN_MOE_SHARDING", str, "ep", "MoE expert layout across TP ranks: partition experts (ep) or slice each "
         "expert's intermediate width (tp)", ("ep", "tp")),
    Flag("BWN_PREFILL_TRACE", int, 0, "per-layer finite / max-abs trace of prefill (1: print, 2: also raise at the "
         "first non-finite layer)", (0, 1, 2)),
    Flag("BWN_SHARD_EMBED", int, 0, "vocab-parallel token embedding (vocab/tp rows per rank, one all-reduce per "
         "lookup) instead of a replicated table", (0, 1)),
    Flag("BWN_F1_ONE_KERNEL", int, 1, "row-parallel GEMM, NVLS all-reduce, residual add and RMSNorm in one launch "
         "(0: the reduction as a second kernel)", (0, 1)),
    Flag("BWN_DN_TC", int, 1, "chunked DeltaNet prefill on the tcgen05 kernel (0: the CUDA-core kernel)", (0, 1)),
    Flag("BWN_MQA_TC", int, 1, "prefill-sized DeepSeek MQA on the tcgen05 kernel (0: the CUDA-core kernel)", (0, 1)),
    Flag("BWN_HC_GEMM", int, 1, "DeepSeek hc_pre mixes as one tensor-core GEMM (0: the fused per-token GEMV, fp32)", (0, 1)),
    Flag("BWN_MOE_FUSED", int, 1, "decode-sized MoE blocks in four launches (fused routing + gather, shared expert "
         "folded into the grouped GEMMs, combine fused with the add-norm or the NVLink slot store)", (0, 1)),
    Flag("BWN_MOE_SHARED_ONLY", int, 0, "cost probe: skip the routed experts, keep the shared expert (wrong results)",
         (0, 1)),
)}


def get(name: str):
    f = FLAGS[name]
    raw = os.environ.get(name)
    if raw is None or raw == "":
        return f.default
    try:
        v = f.kind(raw)
    except ValueError as e:
        raise ValueError(f"{name}={raw!r}: expected {f.kind.__name__}") from e
    if f.choices is not None and v not in f.choices:
        raise ValueError(f"{name}={raw!r}: expected one of {f.choices}")
    return v


def validate(environ=None) -> dict:
    """Parse every declared flag; reject unknown ``BWN_*`` names and conflicts."""
    env = os.environ if environ is None else environ
    unknown = sorted(k for k in env if k.startswith("BWN_") and k not in FLAGS)
    if unknown:
        raise ValueError(f"unknown bwn flags {unknown}; known: {sorted(FLAGS)}")
    saved = dict(os.environ)
    try:
        if environ is not None:
            os.environ.clear()
            os.environ.update(environ)
        vals = {k: get(k) for k in FLAGS}
    finally:
        if environ is not None:
            os.environ.clear()
            os.environ.update(saved)
    if vals["BWN_NO_REDUCE"] and vals["BWN_FUSED_COMM"] == "on":
        raise ValueError("BWN_NO_REDUCE=1 skips collectives; it cannot be combined with BWN_FUSED_COMM=on")
    if vals["BWN_PROFILE_STEPS"] < 0 or vals["BWN_WAIT_LIMIT_MS"] <= 0:
        raise ValueError("BWN_PROFILE_STEPS must be >= 0 and BWN_WAIT_LIMIT_MS > 0")
    return vals


def describe() -> str:
    return "\n".join(f"{f.name:22s} default={f.default!r:8} {f.help}" for f in FLAGS.values())


if __name__ == "__main__":  # python -m bwn.utils.env: list the flags, then validate the current environment
    print(describe())
    validate()
