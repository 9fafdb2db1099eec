"""``python -m bwn``: one launcher for the framework's commands.

    python -m bwn                      # list the commands
    python -m bwn decode --tiny --cpu  # = python -m bwn.runtime.static_decode --tiny --cpu
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m bwn serve --model 35b

Each command is the module named beside it, run with the remaining arguments
(so ``torchrun ... -m bwn <command>`` launches it once per rank).  The
reference's equivalents are separate scripts per model directory
(``static_decode.py``, ``static_decode_35b.py``, ``run_deepseek_v4_tp.py``,
``train_esm.py``, ``train_esm_fsdp.py``, ``run_esm.py``,
``preprocess_weights.py``, the vLLM serve scripts).
"""
from __future__ import annotations

import runpy
import sys

COMMANDS = {
    "decode": ("bwn.runtime.static_decode", "Qwen3.6 greedy generation, prefill / decode benchmarks"),
    "serve": ("bwn.serve.server", "OpenAI-compatible HTTP server (continuous, static or EAGLE3 scheduler)"),
    "deepseek": ("bwn.models.deepseek_v4", "DeepSeek V4 Flash runner (TP / EP / hybrid groups)"),
    "deepseek-weights": ("bwn.io.deepseek_weights", "DeepSeek checkpoint -> per-rank files (fp8 kept or bf16)"),
    "esm-train": ("bwn.train.esm_mlm", "ESM-2 MLM fine-tuning (DP or TP, checkpoints, eval)"),
    "esm-fsdp": ("bwn.train.esm_fsdp", "ESM-2 MLM fine-tuning with FSDP2"),
    "esm-infer": ("bwn.train.esm_infer", "ESM-2 masked-residue prediction"),
    "diagnostics": ("bwn.runtime.diagnostics", "per-layer decode captures and their comparison"),
    "env": ("bwn.utils.env", "list and validate the BWN_* flags"),
}


def usage() -> str:
    w = max(map(len, COMMANDS))
    lines = ["usage: python -m bwn <command> [args]   (torchrun ... -m bwn <command> for several GPUs)", ""]
    lines += [f"  {k:<{w}}  {desc}   [{mod}]" for k, (mod, desc) in COMMANDS.items()]
    return "\n".join(lines)


def main(argv: list[str] | None = None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if not argv or argv[0] in ("-h", "--help", "help"):
        print(usage())
        return 0
    cmd = COMMANDS.get(argv[0])
    if cmd is None:
        print(f"unknown command {argv[0]!r}\n\n{usage()}", file=sys.stderr)
        return 2
    sys.argv = [cmd[0]] + argv[1:]
    runpy.run_module(cmd[0], run_name="__main__", alter_sys=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
