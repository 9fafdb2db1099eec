"""Multi-GPU tests (2+ GPUs): tensor-parallel decode with NCCL vs the fused
NVLink kernels vs the single-GPU model, spawned as one process per GPU."""
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


def _worker(rank, world, port, moe, q, sharding=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        import torch.distributed as dist

        from bwn.config import tiny_qwen36
        from bwn.io import qwen36_weights as W
        from bwn.models.qwen36 import build_qwen36
        from bwn.ops import check_status
        from bwn.parallel.comm import init_distributed
        from bwn.parallel.fused import enable_fused_comm

        comm = init_distributed("nccl", timeout_s=60)
        dev = torch.device("cuda", rank)
        cfg = tiny_qwen36(moe=moe).scaled(q_heads=8, kv_heads=2, dn_k_heads=2, dn_v_heads=4)
        if sharding == "tp":  # each rank's slice of an expert: gate/up rows a multiple of 128 (grouped GEMM tiles)
            cfg = cfg.scaled(moe_inter=64 * world, shared_inter=64 * world)
        hf = dict(W.synthetic_hf_globals(cfg, 3, "cpu"))
        for i in range(cfg.num_layers):
            hf.update(W.synthetic_hf_layer(cfg, i, 3, "cpu"))
        ref = build_qwen36(cfg, device=dev, hf_state=hf)          # tp=1 replica on every rank
        tp = build_qwen36(cfg, comm=comm, device=dev, hf_state=hf, moe_sharding=sharding)  # tp=world
        tpf = build_qwen36(cfg, comm=comm, device=dev, hf_state=hf, moe_sharding=sharding)
        enable_fused_comm(tpf)
        B = 4
        toks = torch.randint(0, cfg.vocab, (B, 24), generator=torch.Generator().manual_seed(0)).to(dev)
        outs = []
        for m in (ref, tp, tpf):
            st = m.new_state(B, 64)
            ids = [m.prefill(toks, st)]
            for _ in range(4):
                ids.append(m.decode_step(ids[-1], st))
            torch.cuda.synchronize()
            check_status("tp decode")
            outs.append(torch.stack(ids, 1).cpu())
        from bwn.parallel.symm import check_canaries
        assert not check_canaries(), "a symmetric buffer was written past its end"
        q.put((rank, [o.tolist() for o in outs]))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, "ERR " + traceback.format_exc()))


@pytest.mark.parametrize("moe,sharding", [(False, None), (True, None), (True, "ep"), (True, "tp")])
def test_tp_decode_fused_vs_nccl(moe, sharding):
    """Dense and MoE; the MoE with experts partitioned across ranks ("ep") and
    with every expert sliced across ranks ("tp", the batch-1 latency layout)."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, moe, q, sharding)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
        ref, tp, tpf = res[r]
        # greedy ids agree across TP degrees and comm paths (tiny model, bf16)
        agree = sum(a == b for ra, rb in zip(ref, tp) for a, b in zip(ra, rb))
        total = sum(len(x) for x in ref)
        assert agree >= total - 2, (ref, tp)
        agree_f = sum(a == b for ra, rb in zip(tp, tpf) for a, b in zip(ra, rb))
        assert agree_f >= total - 2, (tp, tpf)
