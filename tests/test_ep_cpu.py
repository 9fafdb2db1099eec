"""Expert-parallel MoE baseline (host all-to-all with split sizes) on two gloo
ranks equals the single-process MoE with every expert local, with bf16 and
with block-scaled fp8 experts."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bwn.ops import reference as R


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _weights(E, H, I):
    g = torch.Generator().manual_seed(0)
    gu = torch.randn(E, 2 * I, H, generator=g) * 0.05
    dn = torch.randn(E, H, I, generator=g) * 0.05
    return gu, dn


def _tokens(rank, T, H, E, k):
    g = torch.Generator().manual_seed(10 + rank)
    x = torch.randn(T, H, generator=g)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).int()
    w = torch.rand(T, k, generator=g)
    return x, ids, w / w.sum(1, keepdim=True)


def _rank(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    from bwn.parallel.comm import Comm
    from bwn.parallel.ep import nccl_ep_moe
    from bwn.ops import interleave_gate_up
    E, H, I, k, T = 8, 32, 16, 3, 6
    gu, dn = _weights(E, H, I)
    x, ids, w = _tokens(rank, T, H, E, k)
    El = E // 2
    gu_i = torch.stack([interleave_gate_up(gu[e, :I], gu[e, I:]) for e in range(E)])
    local_gu, local_dn = gu_i[rank * El:(rank + 1) * El], dn[rank * El:(rank + 1) * El]
    out = nccl_ep_moe(Comm(None, rank, 2), x, w, ids, local_gu, local_dn, El)
    ref = R.moe_experts(x, w, ids, gu_i, dn, 0)
    err = float((out.float() - ref.float()).abs().max())
    # block-scaled fp8 experts: each rank holds its slice of the quantized set
    from bwn.io.fp8 import FP8Experts
    gate, up = gu[:, :I].contiguous(), gu[:, I:].contiguous()
    f_gu, f_dn = FP8Experts.quantize_gate_up(gate, up), FP8Experts.quantize(dn)
    out8 = nccl_ep_moe(Comm(None, rank, 2), x, w, ids, f_gu.select(rank * El, (rank + 1) * El),
                       f_dn.select(rank * El, (rank + 1) * El), El)
    gq = f_gu.dequant().to(torch.bfloat16).float().reshape(E, I // 16, 2, 16, H)
    ref8 = R.moe_experts(x, w, ids, torch.cat([gq[:, :, 0].reshape(E, I, H), gq[:, :, 1].reshape(E, I, H)], 1),
                         f_dn.dequant().to(torch.bfloat16).float(), 0)
    q.put((rank, max(err, float((out8.float() - ref8.float()).abs().max()))))
    dist.destroy_process_group()


def test_nccl_ep_baseline_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in ps:
        p.join(30)
    assert res[0] < 1e-4 and res[1] < 1e-4, res
