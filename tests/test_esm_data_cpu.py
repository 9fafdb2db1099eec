"""ESM-2 fine-tuning data path and training command on CPU: FASTA parsing,
the seeded train/eval split, fixed-shape tokenization, and the training
command end to end (evaluation, checkpoint, resume; two gloo ranks through
``torch.distributed.run``), mirroring ``contrib/esm2/train_esm.py``."""
import json
import os
import socket
import subprocess
import sys

import torch

from bwn.config import ESM2_SIZES, ESM_ALPHABET
from bwn.train.esm_data import SequenceBatches, encode, load_fasta, split_dataset

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG = ESM2_SIZES["8M"]


def _fasta(tmp_path, n=12):
    lines = []
    for i in range(n):
        lines += [f">seq{i} some description", "MKTVRQERLK", "SIVRILERSK" * (1 + i % 3), ""]
    lines += [">short", "MKT"]  # below 10 residues: dropped
    p = tmp_path / "seqs.fasta"
    p.write_text("\n".join(lines) + "\n")
    return str(p)


def test_load_fasta_joins_lines_and_drops_short(tmp_path):
    seqs = load_fasta(_fasta(tmp_path))
    assert len(seqs) == 12
    assert seqs[0] == "MKTVRQERLK" + "SIVRILERSK"
    assert seqs[1] == "MKTVRQERLK" + "SIVRILERSK" * 2
    assert all(len(s) >= 10 for s in seqs)


def test_split_is_seeded_disjoint_and_nonempty():
    seqs = [f"S{i:03d}" * 4 for i in range(50)]
    tr, ev = split_dataset(seqs, 0.1, seed=42)
    assert len(ev) == 5 and len(tr) == 45
    assert sorted(tr + ev) == sorted(seqs)
    assert split_dataset(seqs, 0.1, seed=42) == (tr, ev)
    assert split_dataset(seqs, 0.1, seed=7) != (tr, ev)
    tr1, ev1 = split_dataset(seqs[:3], 0.1)
    assert len(ev1) == 1 and len(tr1) == 2


def test_encode_truncates_keeps_eos_and_pads():
    ids, am = encode(["ACDEFGHIKL", "AC*D"], CFG, 8)
    assert ids.shape == (2, 8)
    row = [ESM_ALPHABET[i] for i in ids[0].tolist()]
    assert row == ["<cls>", "A", "C", "D", "E", "F", "G", "<eos>"]
    row = [ESM_ALPHABET[i] for i in ids[1].tolist()]
    assert row == ["<cls>", "A", "C", "<unk>", "D", "<eos>", "<pad>", "<pad>"]
    assert am.tolist() == [[1] * 8, [1] * 6 + [0, 0]]


def test_batches_fixed_shape_and_seeded():
    seqs = ["MKTVRQERLK" * (1 + i) for i in range(7)]
    a = SequenceBatches(seqs, CFG, 3, 32, seed=1)
    b = SequenceBatches(seqs, CFG, 3, 32, seed=1)
    for _ in range(3):
        (ia, ma), (ib, mb) = a.sample(), b.sample()
        assert ia.shape == (3, 32) and torch.equal(ia, ib) and torch.equal(ma, mb)
    st = a.state_dict()
    nxt = a.sample()
    a.load_state_dict(st)
    assert torch.equal(a.sample()[0], nxt[0])
    assert sum(x.shape[0] for x, _ in a.sequential()) == 6  # two full batches of 3


def _run(args, env=None, timeout=300):
    e = dict(os.environ, PYTHONPATH=REPO, OMP_NUM_THREADS="2")
    e.update(env or {})
    r = subprocess.run(args, capture_output=True, text=True, timeout=timeout, env=e, cwd=REPO)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return [json.loads(line) for line in r.stdout.splitlines() if line.startswith("{")]


def test_training_command_evaluates_saves_and_resumes(tmp_path):
    fasta = _fasta(tmp_path, 20)
    ck = str(tmp_path / "ck")
    base = [sys.executable, "-m", "bwn.train.esm_mlm", "--cpu", "--model-size", "8M", "--fasta", fasta,
            "--max-seq-len", "40", "--batch-size", "2", "--eval-every", "2", "--save-every", "3",
            "--checkpoint-dir", ck, "--warmup-steps", "2"]
    ev = _run(base + ["--num-steps", "4"])
    kinds = [e["event"] for e in ev]
    assert kinds[0] == "start" and kinds[-1] == "done"
    assert ev[0]["train_sequences"] == 18 and ev[0]["eval_sequences"] == 2
    assert sum(k == "eval" for k in kinds) == 2
    assert all(e["perplexity"] > 1.0 for e in ev if e["event"] == "eval")
    saved = torch.load(os.path.join(ck, "checkpoint.pt"), weights_only=False)
    assert saved["step"] == 4 and saved["rngs"][0]["data"] is not None
    ev2 = _run(base + ["--num-steps", "6", "--resume", ck])
    assert ev2[0]["event"] == "resumed" and ev2[0]["step"] == 4
    assert ev2[-1]["steps"] == 2
    assert torch.load(os.path.join(ck, "checkpoint.pt"), weights_only=False)["step"] == 6


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _torchrun(n, port):
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", str(n),
            "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "bwn.train.esm_mlm", "--cpu"]


def test_training_command_two_ranks(tmp_path):
    port = _free_port()
    for mode in ("dp", "tp"):
        ck = str(tmp_path / mode)
        ev = _run(_torchrun(2, port) + ["--model-size", "8M", "--max-seq-len", "32", "--batch-size", "2",
                                        "--num-steps", "3", "--eval-every", "0", "--save-every", "0",
                                        "--checkpoint-dir", ck, "--parallel", mode])
        assert ev[0]["parallel"] == f"{mode}2"
        assert ev[-1]["event"] == "done"
        assert sorted(os.listdir(ck)) == ["checkpoint.pt"]  # one portable file in both modes


def _losses(events):
    return {e["step"]: e["loss"] for e in events if e["event"] == "step"}


def test_resume_continues_the_loss_trajectory(tmp_path):
    """A run stopped after 3 steps and resumed in a new process reproduces the
    uninterrupted run's losses exactly (same world size: model, AdamW moments,
    schedule and every generator restored)."""
    fasta = _fasta(tmp_path, 20)
    base = [sys.executable, "-m", "bwn.train.esm_mlm", "--cpu", "--model-size", "8M", "--fasta", fasta,
            "--max-seq-len", "40", "--batch-size", "2", "--eval-every", "0", "--log-every", "1",
            "--warmup-steps", "2"]
    full = _losses(_run(base + ["--num-steps", "6", "--save-every", "0", "--checkpoint-dir", str(tmp_path / "x")]))
    ck = str(tmp_path / "ck")
    first = _losses(_run(base + ["--num-steps", "6", "--stop-after", "3", "--save-every", "0", "--checkpoint-dir", ck]))
    rest = _losses(_run(base + ["--num-steps", "6", "--save-every", "0", "--checkpoint-dir", ck, "--resume", ck]))
    assert sorted(first) == [0, 1, 2] and sorted(rest) == [3, 4, 5]
    assert {**first, **rest} == full


def test_checkpoint_reshards_from_tp2_to_one_rank(tmp_path):
    """Saved by two tensor-parallel ranks, resumed by a single process: the
    losses continue the two-rank run's trajectory up to reduction-order rounding."""
    common = ["--model-size", "8M", "--max-seq-len", "32", "--batch-size", "2", "--eval-every", "0",
              "--log-every", "1", "--warmup-steps", "2"]
    ref = _losses(_run(_torchrun(2, _free_port()) + common + ["--parallel", "tp", "--num-steps", "4",
                                                            "--save-every", "0", "--checkpoint-dir",
                                                            str(tmp_path / "r")]))
    ck = str(tmp_path / "ck")
    _run(_torchrun(2, _free_port()) + common + ["--parallel", "tp", "--num-steps", "4", "--stop-after", "2",
                                              "--save-every", "0", "--checkpoint-dir", ck])
    saved = torch.load(os.path.join(ck, "checkpoint.pt"), weights_only=False)
    q = saved["model"]["esm.encoder.layer.0.attention.self.query.weight"]
    assert q.shape == (CFG.hidden, CFG.hidden)  # stored unsharded
    assert "esm.encoder.layer.0.attention.self.query.weight" in saved["moments"]
    rest = _losses(_run([sys.executable, "-m", "bwn.train.esm_mlm", "--cpu"] + common +
                        ["--parallel", "tp", "--num-steps", "4", "--save-every", "0", "--checkpoint-dir", ck,
                         "--resume", ck]))
    assert sorted(rest) == [2, 3]
    for s in (2, 3):
        assert abs(rest[s] - ref[s]) < 2e-3, (s, rest[s], ref[s])
