"""``python -m bwn``: lists the commands, runs one with its arguments, and
refuses an unknown one."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENV = dict(os.environ, PYTHONPATH=ROOT, OMP_NUM_THREADS="2")


def _run(args):
    return subprocess.run([sys.executable, "-m", "bwn"] + args, env=ENV, cwd=ROOT, capture_output=True, text=True,
                          timeout=300)


def test_launcher_lists_dispatches_and_refuses():
    from bwn.__main__ import COMMANDS
    r = _run([])
    assert r.returncode == 0 and all(k in r.stdout for k in COMMANDS)
    r = _run(["decode", "--tiny", "--cpu", "--prompt-len", "8", "--num-tokens", "3"])
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])
    assert len(out["generated_row0"]) == 3
    assert _run(["env"]).returncode == 0
    r = _run(["no-such-command"])
    assert r.returncode == 2 and "unknown command" in r.stderr
