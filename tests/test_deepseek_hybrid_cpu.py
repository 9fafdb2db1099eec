"""DeepSeek V4 hybrid layout (TP groups of consecutive ranks, EP groups strided
by the TP size) on four gloo ranks equals the single-process model."""
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


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from bwn.config import tiny_deepseek_v4
        from bwn.models.deepseek_v4 import DeepSeekV4Model, synthetic_checkpoint
        from bwn.parallel.comm import hybrid_groups

        cfg = tiny_deepseek_v4()
        sd = synthetic_checkpoint(cfg, 0)
        tp_comm, ep_comm = hybrid_groups(2)
        assert tp_comm.size == 2 and ep_comm.size == 2
        ref = DeepSeekV4Model(cfg, None, "cpu", torch.float32).load(sd)
        hyb = DeepSeekV4Model(cfg, tp_comm, "cpu", torch.float32, ep_comm=ep_comm).load(sd)
        toks = torch.randint(0, cfg.vocab, (2, 10), generator=torch.Generator().manual_seed(3))
        outs = []
        for m in (ref, hyb):
            st = m.new_state(2, 32)
            B, S = toks.shape
            pos = torch.arange(S, dtype=torch.int32).repeat(B)
            bidx = torch.arange(B, dtype=torch.int32).repeat_interleave(S)
            outs.append(m.forward_tokens(toks.reshape(-1), pos, bidx, st, S))
        q.put((rank, float((outs[0] - outs[1]).abs().max() / outs[0].abs().max())))
    except Exception:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc()))
    dist.destroy_process_group()


def test_deepseek_hybrid_tp2_ep2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, 4, port, q)) for r in range(4)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(4))
    for p in ps:
        p.join(30)
    for r in range(4):
        assert isinstance(res[r], float), res[r]
        assert res[r] < 1e-4, res
