"""Bucketed, backward-overlapped gradient reduction (NCCL/gloo baseline
reducer) on two gloo ranks: averaged gradients equal the single-process
gradients of the concatenated batch."""
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
        from bwn.parallel.comm import Comm
        from bwn.parallel.grad_reduce import NcclGradReducer
        from bwn.train.esm_mlm import build_esm, mask_tokens, synthetic_batch

        comm = Comm(None, rank, 2)
        ref = build_esm("8M", seed=0)
        dp = build_esm("8M", seed=0)
        red = NcclGradReducer(dp, comm, bucket_mb=1.0)
        assert len(red.buckets) > 2
        g = torch.Generator().manual_seed(5)
        ids, am = synthetic_batch(ref.cfg, 4, 16, g)
        ids, labels, lm = mask_tokens(ids, ref.cfg, g)
        loss = mlm_loss(ref(ids, am), labels, lm, "tokens")
        loss.backward()
        half = slice(rank * 2, rank * 2 + 2)
        for step in range(2):  # twice: bucket storage reused, zeroed in place
            for p in dp.parameters():
                p.grad.zero_()
            l2 = mlm_loss(dp(ids[half], am[half]), labels[half], lm[half], "tokens")
            l2.backward()
            red.finish()
        err = max(float((a.grad - b.grad).abs().max()) for a, b in zip(ref.parameters(), dp.parameters()))
        q.put((rank, err))
    except Exception:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc()))
    dist.destroy_process_group()


def test_bucketed_grad_reduce_two_ranks():
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
