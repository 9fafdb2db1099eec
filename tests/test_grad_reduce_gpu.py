"""Fused NVLS gradient reduction (2 GPUs): data-parallel ESM-2 gradients after
the bucketed, backward-overlapped reduction equal the single-GPU gradients of
the concatenated batch (bf16 on the wire), for the fused and NCCL reducers."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist

        from bwn.models.esm2 import mlm_loss
        from bwn.ops import check_status
        from bwn.parallel.comm import init_distributed
        from bwn.parallel.grad_reduce import GradReducer, NcclGradReducer
        from bwn.train.esm_mlm import build_esm, mask_tokens, synthetic_batch

        comm = init_distributed("nccl", timeout_s=60)
        dev = torch.device("cuda", rank)
        ref = build_esm("8M", device=dev, seed=0)
        g = torch.Generator().manual_seed(5)
        ids, am = synthetic_batch(ref.cfg, 4, 64, g)
        ids, labels, lm = mask_tokens(ids, ref.cfg, g)
        ids, am, labels, lm = (t.to(dev) for t in (ids, am, labels, lm))
        mlm_loss(ref(ids, am), labels, lm, "tokens").backward()
        half = slice(rank * 2, rank * 2 + 2)
        errs = {}
        for name, cls in (("fused", GradReducer), ("nccl", NcclGradReducer)):
            dp = build_esm("8M", device=dev, seed=0)
            red = cls(dp, comm, bucket_mb=1.0)
            for _ in range(2):
                for p in dp.parameters():
                    p.grad.zero_()
                mlm_loss(dp(ids[half], am[half]), labels[half], lm[half], "tokens").backward()
                red.finish()
            torch.cuda.synchronize()
            check_status(name)
            num = max(float((a.grad - b.grad).abs().max()) for a, b in zip(ref.parameters(), dp.parameters()))
            den = max(float(a.grad.abs().max()) for a in ref.parameters())
            errs[name] = num / den
        from bwn.parallel.symm import check_canaries
        assert not check_canaries(), "a symmetric buffer was written past its end"
        q.put((rank, errs))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        import traceback
        q.put((rank, "ERR " + traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_grad_reduce_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(60)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
        assert res[r]["fused"] < 2e-2 and res[r]["nccl"] < 1e-2, res
