"""ESM-2 tensor parallelism (colwise q/k/v + intermediate, rowwise output
projections) on two gloo ranks: the loss and every gradient equal the
single-process model's."""
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
        from bwn.parallel.tensor_parallel import apply_esm_tp
        from bwn.train.esm_mlm import build_esm, mask_tokens, synthetic_batch

        comm = Comm(None, rank, 2)
        ref = build_esm("8M", seed=0)
        tp = apply_esm_tp(build_esm("8M", seed=0), comm)
        g = torch.Generator().manual_seed(5)
        ids, am = synthetic_batch(ref.cfg, 2, 20, g)
        ids, labels, lm = mask_tokens(ids, ref.cfg, g)
        losses = []
        for m in (ref, tp):
            loss = mlm_loss(m(ids, am), labels, lm, "masked")
            loss.backward()
            losses.append(float(loss))
        errs = [abs(losses[0] - losses[1])]
        n = 2
        for lr, lt in zip(ref.esm.encoder.layer, tp.esm.encoder.layer):
            w_full = lr.intermediate.dense.weight.grad
            rows = w_full.shape[0] // n
            errs.append(float((w_full[rank * rows:(rank + 1) * rows] - lt.intermediate.dense.weight.grad).abs().max()))
            w_full = lr.output.dense.weight.grad
            cols = w_full.shape[1] // n
            errs.append(float((w_full[:, rank * cols:(rank + 1) * cols] - lt.output.dense.weight.grad).abs().max()))
            errs.append(float((lr.output.dense.bias.grad - lt.output.dense.bias.grad).abs().max()))
            w_full = lr.attention.self.query.weight.grad
            rows = w_full.shape[0] // n
            errs.append(float((w_full[rank * rows:(rank + 1) * rows] - lt.attention.self.query.weight.grad).abs().max()))
        errs.append(float((ref.esm.embeddings.word_embeddings.weight.grad
                           - tp.esm.embeddings.word_embeddings.weight.grad).abs().max()))
        q.put((rank, max(errs)))
    except Exception:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc()))
    dist.destroy_process_group()


def test_esm_tp2_matches_single():
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
        assert res[r] < 1e-4, res
