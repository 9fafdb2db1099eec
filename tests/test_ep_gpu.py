"""Expert-parallel all-to-all over NVLink peer memory (2 GPUs, one process
each): the dispatch -> grouped expert GEMMs -> return -> combine block equals
the MoE with every expert local, eagerly, repeatedly (buffer reuse) and
replayed from a CUDA graph."""
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

        from bwn import ops as O
        from bwn.ops import check_status
        from bwn.parallel.comm import init_distributed
        from bwn.parallel.ep import EPAllToAll, nccl_ep_moe

        comm = init_distributed("nccl", timeout_s=60)
        dev = torch.device("cuda", rank)
        E, H, I, k, T = 16, 256, 64, 4, 24
        El = E // world
        g = torch.Generator().manual_seed(0)
        gu = torch.stack([O.interleave_gate_up(torch.randn(I, H, generator=g) * 0.05,
                                               torch.randn(I, H, generator=g) * 0.05) for _ in range(E)])
        dn = torch.randn(E, H, I, generator=g) * 0.05
        gu, dn = gu.bfloat16().to(dev), dn.bfloat16().to(dev)
        loc_gu, loc_dn = gu[rank * El:(rank + 1) * El].contiguous(), dn[rank * El:(rank + 1) * El].contiguous()
        ep = EPAllToAll(comm, H, E, k, max_tokens=T, device=dev)
        errs = []
        for it in range(3):
            gt = torch.Generator().manual_seed(100 * it + rank)
            x = torch.randn(T, H, generator=gt).bfloat16().to(dev)
            ids = torch.stack([torch.randperm(E, generator=gt)[:k] for _ in range(T)]).int().to(dev)
            w = torch.rand(T, k, generator=gt).to(dev)
            sy = torch.randn(T, H, generator=gt).bfloat16().to(dev)
            sg = torch.randn(T, 1, generator=gt).to(dev)
            out = ep.moe(x, w, ids, loc_gu, loc_dn, shared=(sy, sg))
            ref = O.moe_experts(x, w, ids, gu, dn, 0, shared=(sy, sg))
            base = nccl_ep_moe(comm, x, w, ids, loc_gu, loc_dn, El, shared=(sy, sg))
            torch.cuda.synchronize()
            check_status("ep")
            errs.append(float((out.float() - ref.float()).abs().max() / ref.float().abs().max()))
            errs.append(float((base.float() - ref.float()).abs().max() / ref.float().abs().max()))
        # CUDA graph replay of the whole block
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(7 + rank)).bfloat16().to(dev)
        ids = torch.stack([torch.randperm(E, generator=torch.Generator().manual_seed(9 + rank + 2 * i))[:k]
                           for i in range(T)]).int().to(dev)
        w = torch.rand(T, k, generator=torch.Generator().manual_seed(3)).to(dev)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ep.moe(x, w, ids, loc_gu, loc_dn)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                out_g = ep.moe(x, w, ids, loc_gu, loc_dn)
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        check_status("ep graph")
        ref = O.moe_experts(x, w, ids, gu, dn, 0)
        errs.append(float((out_g.float() - ref.float()).abs().max() / ref.float().abs().max()))
        del graph
        from bwn.parallel.symm import check_canaries
        assert not check_canaries(), "a symmetric buffer was written past its end"
        q.put((rank, errs))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        import traceback
        q.put((rank, "ERR " + traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_all_to_all_two_gpus():
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
        assert max(res[r]) < 2e-2, res[r]


def _model_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist

        from bwn.config import tiny_qwen36
        from bwn.io import qwen36_weights as Wt
        from bwn.models.qwen36 import build_qwen36
        from bwn.ops import check_status
        from bwn.parallel.comm import init_distributed
        from bwn.parallel.ep import enable_ep_all_to_all

        comm = init_distributed("nccl", timeout_s=60)
        dev = torch.device("cuda", rank)
        cfg = tiny_qwen36(moe=True).scaled(q_heads=8, kv_heads=2, dn_k_heads=2, dn_v_heads=4)
        hf = dict(Wt.synthetic_hf_globals(cfg, 3, "cpu"))
        for i in range(cfg.num_layers):
            hf.update(Wt.synthetic_hf_layer(cfg, i, 3, "cpu"))
        ref = build_qwen36(cfg, device=dev, hf_state=hf)
        ep_model = build_qwen36(cfg, comm=comm, device=dev, hf_state=hf)
        enable_ep_all_to_all(ep_model, max_tokens_per_rank=64, min_tokens_per_rank=8)
        B, S = 4, 24
        toks = torch.randint(0, cfg.vocab, (B, S), generator=torch.Generator().manual_seed(0)).to(dev)
        hs = []
        for m in (ref, ep_model):
            st = m.new_state(B, 64)
            hs.append(m.prefill_hidden(toks, st).float())
        torch.cuda.synchronize()
        check_status("ep model")
        rel = float((hs[0] - hs[1]).norm() / hs[0].norm())
        from bwn.parallel.symm import check_canaries
        assert not check_canaries(), "a symmetric buffer was written past its end"
        q.put((rank, rel))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        import traceback
        q.put((rank, "ERR " + traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_qwen36_moe_prefill_with_ep_all_to_all():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_model_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(60)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
        assert res[r] < 3e-2, res


def _sp_worker(rank, world, port, moe, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist

        from bwn.config import tiny_qwen36
        from bwn.io import qwen36_weights as Wt
        from bwn.models.qwen36 import build_qwen36
        from bwn.models.qwen36_prefill import prefill_hidden_sp
        from bwn.ops import check_status
        from bwn.parallel.comm import init_distributed
        from bwn.parallel.ep import enable_ep_all_to_all
        from bwn.parallel.sp import SeqParallel

        comm = init_distributed("nccl", timeout_s=60)
        dev = torch.device("cuda", rank)
        cfg = tiny_qwen36(moe=moe).scaled(q_heads=8, kv_heads=2, dn_k_heads=2, dn_v_heads=4)
        hf = dict(Wt.synthetic_hf_globals(cfg, 3, "cpu"))
        for i in range(cfg.num_layers):
            hf.update(Wt.synthetic_hf_layer(cfg, i, 3, "cpu"))
        ref = build_qwen36(cfg, device=dev, hf_state=hf)
        m = build_qwen36(cfg, comm=comm, device=dev, hf_state=hf)
        B, S = 4, 128
        if moe:
            enable_ep_all_to_all(m, max_tokens_per_rank=B * S // world, min_tokens_per_rank=8)
        sp = SeqParallel(comm, cfg.hidden, B * S, device=dev)
        toks = torch.randint(0, cfg.vocab, (B, S), generator=torch.Generator().manual_seed(0)).to(dev)
        st0, st1 = ref.new_state(B, 160), m.new_state(B, 160)
        h0 = ref.prefill_hidden(toks, st0).float()
        errs = []
        for _ in range(2):  # twice: buffers and epochs reused
            st1 = m.new_state(B, 160)
            h1 = prefill_hidden_sp(m, toks, st1, sp).float()
            torch.cuda.synchronize()
            check_status("sp prefill")
            errs.append(float((h0 - h1).norm() / h0.norm()))
        # decode after the sequence-parallel prefill continues correctly
        t0 = ref.greedy(h0.bfloat16())
        d0 = ref.decode_step(t0, st0).float()
        d1 = m.decode_step(t0, st1).float()
        errs.append(float((d0 != d1).float().mean()))
        from bwn.parallel.symm import check_canaries
        assert not check_canaries(), "a symmetric buffer was written past its end"
        q.put((rank, errs))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        import traceback
        q.put((rank, "ERR " + traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("moe", [False, True])
def test_sequence_parallel_prefill(moe):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_sp_worker, args=(r, 2, port, moe, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(60)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
        assert max(res[r][:2]) < 3e-2 and res[r][2] <= 0.25, res
