"""Multi-rank serving in lockstep on two gloo ranks: rank 0's worker takes the
requests, the follower replays admissions and steps, and the tensor-parallel
engine's answers equal single-rank greedy generation."""
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


PROMPTS = [([5, 9, 13], 5), ([7, 7, 2, 1, 30], 4), ([100, 3], 6), ([11], 3), ([40, 41, 42, 43], 5)]


def _rank(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        torch.set_num_threads(2)
        from bwn.config import tiny_qwen36
        from bwn.models.qwen36 import build_qwen36
        from bwn.parallel.comm import Comm
        from bwn.serve.continuous import ContinuousEngine
        from bwn.serve.engine import Request
        from bwn.serve.lockstep import LockstepEngine, control_group, follow
        cfg = tiny_qwen36()
        model = build_qwen36(cfg, Comm(None, rank, 2), seed=4, dtype=torch.float32)
        engine = ContinuousEngine(model, 2, 32, use_graph=False)
        ctrl = control_group()
        if rank != 0:
            follow(engine, ctrl)
            q.put((rank, "followed"))
            return
        from bwn.runtime.static_decode import StaticDecoder
        from bwn.serve.server import ContinuousWorker
        one = build_qwen36(cfg, Comm.single(), seed=4, dtype=torch.float32)
        want = [StaticDecoder(one, 1, 32, use_graph=False).generate(torch.tensor([p]), n)[0].tolist()
                for p, n in PROMPTS]
        worker = ContinuousWorker(LockstepEngine(engine, ctrl))
        futs = [worker.submit(Request(p, n)) for p, n in PROMPTS]
        got = [f.result(timeout=120).tokens for f in futs]
        worker.stop()
        q.put((rank, got == want))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def test_lockstep_serving_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(2))
    for p in ps:
        p.join(60)
    assert res[0] is True, res[0]
    assert res[1] == "followed", res[1]


def _batch_rank(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        torch.set_num_threads(2)
        from bwn.config import tiny_qwen36
        from bwn.models.eagle3 import Eagle3Draft, eagle3_config
        from bwn.models.qwen36 import build_qwen36
        from bwn.parallel.comm import Comm
        from bwn.serve.engine import Request
        from bwn.serve.lockstep import LockstepBatchEngine, control_group, follow
        from bwn.serve.spec import SpecEngine
        cfg = tiny_qwen36()
        model = build_qwen36(cfg, Comm(None, rank, 2), seed=4, dtype=torch.float32)
        draft = Eagle3Draft(eagle3_config(cfg), "cpu", torch.float32).init_random(0)
        engine = SpecEngine(model, draft, 2, 48, 3, use_graph=False)
        ctrl = control_group()
        if rank != 0:
            follow(engine, ctrl)
            q.put((rank, "followed"))
            return
        from bwn.runtime.static_decode import StaticDecoder
        from bwn.serve.server import BatchingWorker
        one = build_qwen36(cfg, Comm.single(), seed=4, dtype=torch.float32)
        want = [StaticDecoder(one, 1, 48, use_graph=False).generate(torch.tensor([p]), n)[0].tolist()
                for p, n in PROMPTS]
        worker = BatchingWorker(LockstepBatchEngine(engine, ctrl), batch_window_ms=1)
        got = [worker.submit(Request(p, n)).result(timeout=120).tokens for p, n in PROMPTS]
        worker.stop()
        q.put((rank, got == want))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def test_lockstep_speculative_serving_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_batch_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(2))
    for p in ps:
        p.join(60)
    assert res[0] is True, res[0]
    assert res[1] == "followed", res[1]
