"""The static-decode command (the reference harness's main): generated ids,
gen hash and prefill fingerprint are the same for whole and bucketed prefill
and for one process and two tensor-parallel gloo ranks; a checkpoint
directory with --prompt-ids runs the same path."""
import json
import os
import socket
import subprocess
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENV = dict(os.environ, PYTHONPATH=ROOT, OMP_NUM_THREADS="2")
BASE = ["-m", "bwn.runtime.static_decode", "--model", "tiny", "--cpu", "--batch", "2", "--prompt-len", "12",
        "--max-new", "6"]


def _run(args):
    r = subprocess.run([sys.executable] + args, env=ENV, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])


def test_whole_bucketed_and_two_ranks_agree():
    one = _run(BASE + ["--prefill-gen"])
    assert one["prefill_gen_matches"] and one["prefill_gen_hash_row0"] == one["gen_hash_row0"]
    assert one["prefill_fingerprint"]["finite"] and len(one["generated_row0"]) == 6
    assert _run(BASE + ["--bucket", "5"])["gen_hash_row0"] == one["gen_hash_row0"]
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    two = _run(["-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
                "--master-port", str(port)] + BASE)
    assert two["tp"] == 2 and two["gen_hash_row0"] == one["gen_hash_row0"]
    assert two["prefill_fingerprint"]["top5"] == one["prefill_fingerprint"]["top5"]


def test_checkpoint_with_prompt_ids(tmp_path):
    from bwn.config import qwen36_from_hf, qwen36_to_hf, tiny_qwen36
    from bwn.io import qwen36_weights as W
    from bwn.io.safetensors import save_file
    cfg = tiny_qwen36()
    sd = dict(W.synthetic_hf_globals(cfg, 2, "cpu"))
    for i in range(cfg.num_layers):
        sd.update(W.synthetic_hf_layer(cfg, i, 2, "cpu"))
    save_file({"model." + k if k != "lm_head.weight" else k: v.contiguous() for k, v in sd.items()},
              str(tmp_path / "model.safetensors"))
    (tmp_path / "config.json").write_text(json.dumps(qwen36_to_hf(cfg)))
    assert qwen36_from_hf(str(tmp_path)) == cfg
    out = _run(["-m", "bwn.runtime.static_decode", "--checkpoint", str(tmp_path), "--cpu", "--prompt-ids",
                "7,11,13,17,19", "--max-new", "4"])
    assert out["prompt_len"] == 5 and len(out["generated_row0"]) == 4
    assert torch.tensor(out["generated_row0"]).max() < cfg.vocab


def _run_all(args):
    r = subprocess.run([sys.executable] + args, env=ENV, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    return [json.loads(ln) for ln in r.stdout.splitlines() if ln.startswith("{")]


def test_reference_flag_names_and_bench_modes():
    """The reference harness's command line runs as is: --tiny, --batch-size,
    --num-tokens, --bucket-chunk, --skip-compile name the same settings; --bench
    adds a TPOT window after the generated tokens; --skip-prefill decodes from
    the last prompt token; --prefill-bench (+ sweep) reports prompt-ingest
    throughput per length and exits."""
    ref = _run(BASE)
    alias = _run(["-m", "bwn.runtime.static_decode", "--tiny", "--cpu", "--batch-size", "2", "--prompt-len", "12",
                  "--num-tokens", "6", "--bucket-chunk", "5", "--skip-compile", "--bench", "--bench-iters", "3"])
    assert alias["gen_hash_row0"] == ref["gen_hash_row0"] and alias["batch"] == 2
    assert alias["bench_iters"] == 3 and alias["bench_tpot_ms"] > 0 and alias["bench_tok_s"] > 0
    skip = _run(BASE + ["--skip-prefill"])
    assert skip["skip_prefill"] and skip["prefill_fingerprint"] is None and len(skip["generated_row0"]) == 6
    lines = _run_all(["-m", "bwn.runtime.static_decode", "--tiny", "--cpu", "--prefill-bench", "32",
                      "--prefill-bench-sweep", "16,48", "--bucket-chunk", "16"])
    assert [ln["prefill_tokens"] for ln in lines] == [32, 16, 48]
    assert all(ln["prefill_tok_s"] > 0 and ln["bucket"] == 16 for ln in lines)


def test_text_prompt_through_tokenizer(tmp_path):
    """--prompt text goes through the tokenizer: the same tokens as the ids it
    encodes to, and the generated ids decoded as text_row0."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    tk = Tokenizer(models.WordLevel({f"w{i}": i for i in range(512)}, unk_token="w0"))
    tk.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tk.decoder = decoders.WordPiece(prefix="##")
    PreTrainedTokenizerFast(tokenizer_object=tk, unk_token="w0").save_pretrained(str(tmp_path))
    common = ["-m", "bwn.runtime.static_decode", "--tiny", "--cpu", "--max-new", "4"]
    by_text = _run(common + ["--tokenizer", str(tmp_path), "--prompt", "w5 w9 w13"])
    by_ids = _run(common + ["--prompt-ids", "5,9,13"])
    assert by_text["prompt_len"] == 3 and by_text["gen_hash_row0"] == by_ids["gen_hash_row0"]
    assert by_text["text_row0"] == " ".join(f"w{i}" for i in by_text["generated_row0"])
