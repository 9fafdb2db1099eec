"""ESM-2 FSDP (fully_shard per layer) on two gloo ranks: gradients of the
sharded model equal the single-process gradients of the concatenated batch."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        from bwn.models.esm2 import mlm_loss
        from bwn.train.esm_fsdp import hf_mlm_loss, mask_all_chosen, shard_esm_fsdp
        from bwn.train.esm_mlm import build_esm, mask_tokens, synthetic_batch

        ref = build_esm("8M", seed=0)
        fs = shard_esm_fsdp(build_esm("8M", seed=0), 2, device_type="cpu")
        g = torch.Generator().manual_seed(5)
        ids, am = synthetic_batch(ref.cfg, 4, 16, g)
        ids2, labels, lm = mask_tokens(ids, ref.cfg, g)
        mlm_loss(ref(ids2, am), labels, lm, "tokens").backward()
        half = slice(rank * 2, rank * 2 + 2)
        mlm_loss(fs(ids2[half], am[half]), labels[half], lm[half], "tokens").backward()
        err = 0.0
        for (n, a), (_, b) in zip(ref.named_parameters(), fs.named_parameters()):
            gb = b.grad.full_tensor() if hasattr(b.grad, "full_tensor") else b.grad
            err = max(err, float((a.grad - gb).abs().max()))
        mi, lab = mask_all_chosen(ids, ref.cfg, torch.Generator().manual_seed(1))
        assert bool(((lab != -100) == (mi == ref.cfg.mask_token_id)).all())
        assert torch.isfinite(hf_mlm_loss(ref(mi, am), lab))
        q.put((rank, err))
    except Exception:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc()))
    dist.destroy_process_group()


def test_esm_fsdp_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=180) for _ in range(2))
    for p in ps:
        p.join(30)
    for r in (0, 1):
        assert isinstance(res[r], float), res[r]
        assert res[r] < 1e-5, res


def test_fsdp_command_two_ranks(tmp_path):
    """The FSDP training command on two gloo ranks under torchrun."""
    import json
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "bwn.train.esm_fsdp",
                        "--model-size", "8M", "--cpu", "--num-steps", "3", "--max-seq-len", "32"],
                       env=dict(os.environ, PYTHONPATH=root, OMP_NUM_THREADS="2"), cwd=root, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    ev = [json.loads(ln) for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert ev[0]["world"] == 2 and ev[-1]["event"] == "done" and ev[-1]["steps"] == 3
    assert all(e["loss"] > 0 for e in ev if e["event"] == "step")
