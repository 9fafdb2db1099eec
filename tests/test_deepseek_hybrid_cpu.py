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


class _FakeFused:
    """Stands in for bwn.parallel.fused.FusedComm on gloo: same interface, the
    reduction through the process group; counts the calls."""

    def __init__(self, comm):
        self.comm, self.calls = comm, {"gemm_allreduce_hc_post": 0, "allreduce_hc_post": 0}

    def fits(self, rows):
        return rows <= 256

    def gemm_allreduce_hc_post(self, a, w, resid, post, comb):
        from bwn.ops import reference as R
        self.calls["gemm_allreduce_hc_post"] += 1
        return R.hc_post(self.comm.all_reduce_(a.float() @ w.float().t()).to(resid.dtype), resid, post, comb)

    def allreduce_hc_post(self, part, resid, post, comb):
        from bwn.ops import reference as R
        self.calls["allreduce_hc_post"] += 1
        return R.hc_post(self.comm.all_reduce_(part.clone()), resid, post, comb)


def _fused_rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(2)
        from bwn.config import tiny_deepseek_v4
        from bwn.models.deepseek_v4 import DeepSeekV4Model, synthetic_checkpoint
        from bwn.parallel.comm import Comm
        cfg = tiny_deepseek_v4()
        sd = synthetic_checkpoint(cfg, 0)
        comm = Comm(None, rank, world)
        plain = DeepSeekV4Model(cfg, comm, "cpu", torch.float32).load(sd)
        fused = DeepSeekV4Model(cfg, comm, "cpu", torch.float32).load(sd)
        fused.fused_comm = _FakeFused(comm)
        toks = torch.randint(0, cfg.vocab, (2, 6), generator=torch.Generator().manual_seed(5))
        outs = []
        for m in (plain, fused):
            st = m.new_state(2, 16)
            pos = torch.arange(6, dtype=torch.int32).repeat(2)
            bidx = torch.arange(2, dtype=torch.int32).repeat_interleave(6)
            outs.append(m.forward_tokens(toks.reshape(-1), pos, bidx, st, 6))
        q.put((rank, float((outs[0] - outs[1]).abs().max()), fused.fused_comm.calls, cfg.num_layers))
    except Exception:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc(), None, 0))
    dist.destroy_process_group()


def test_deepseek_fused_comm_hooks_two_ranks():
    """With a fused communicator attached, each layer reduces its attention
    output projection and its MoE partial through it, folded with the
    hyper-connection post-mix, with the same result."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_fused_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=240) for _ in range(2)]
    for p in ps:
        p.join(30)
    for rank, err, calls, layers in res:
        assert not isinstance(err, str), err
        assert err < 1e-4, (rank, err)
        assert calls == {"gemm_allreduce_hc_post": layers, "allreduce_hc_post": layers}, calls
