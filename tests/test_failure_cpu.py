"""Failure detection without a GPU fault: host-side rank failures among CPU
processes (gloo / TCPStore), and the launcher's handling of a dead worker."""
import datetime
import os
import socket
import subprocess
import sys
import time

import torch.distributed as dist
import torch.multiprocessing as mp

from bwn.runtime.health import Heartbeat, PeerFailure, ProtocolError, guarded

HERE = os.path.dirname(os.path.abspath(__file__))


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _store(rank, port):
    return dist.TCPStore("127.0.0.1", port, 2, rank == 0, timeout=datetime.timedelta(seconds=20))


def _scenario(rank, port, mode, q):
    try:
        st = _store(rank, port)
        hb = Heartbeat(st, rank, 2, stale_s=1.5)
        for step in range(4):
            if rank == 1 and step == 2:
                if mode == "raise":
                    try:
                        guarded(hb, step, lambda: (_ for _ in ()).throw(ValueError("bad batch")))
                    except ValueError:
                        pass
                    time.sleep(3)
                    q.put((rank, "ok"))
                    return
                if mode == "die":
                    os._exit(0)
                if mode == "corrupt":
                    hb.beat(step)
                    time.sleep(0.5)
                    hb.beat(0)      # sequence number goes backwards
                    time.sleep(3)
                    q.put((rank, "ok"))
                    return
            guarded(hb, step, lambda: None)
            hb.wait_peers(step)
        q.put((rank, "finished"))
    except PeerFailure as e:
        q.put((rank, "PeerFailure:" + str(e)))
    except ProtocolError as e:
        q.put((rank, "ProtocolError:" + str(e)))


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_scenario, args=(r, port, mode, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = {}
    t0 = time.time()
    while len(out) < (1 if mode == "die" else 2) and time.time() - t0 < 60:
        try:
            r, v = q.get(timeout=1)
            out[r] = v
        except Exception:
            pass
    for p in ps:
        p.join(10)
        if p.is_alive():
            p.kill()
    return out


def test_peer_error_reported_before_next_launch():
    out = _run("raise")
    assert out[0].startswith("PeerFailure") and "bad batch" in out[0]


def test_dead_peer_detected_by_stale_heartbeat():
    out = _run("die")
    assert out[0].startswith("PeerFailure") and "no progress" in out[0]


def test_corrupted_sequence_number():
    out = _run("corrupt")
    assert out[0].startswith("ProtocolError")


def _barrier_rank(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        time.sleep(8)  # never joins the barrier in time
        q.put((1, "slept"))
        return
    t0 = time.time()
    try:
        dist.barrier()
        q.put((0, "passed"))
    except Exception as e:  # noqa: BLE001
        q.put((0, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))


def test_process_group_timeout_ends_a_missing_rank_wait():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_barrier_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    t0 = time.time()
    while 0 not in res and time.time() - t0 < 60:
        try:
            r, v = q.get(timeout=1)
            res[r] = v
        except Exception:
            pass
    for p in ps:
        p.join(15)
        if p.is_alive():
            p.kill()
    assert res[0].startswith("error after"), res


def test_launcher_stops_job_when_a_worker_dies():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()), os.path.join(HERE, "_worker_exit.py")]
    t0 = time.time()
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=100)
    assert r.returncode != 0
    assert time.time() - t0 < 90
    assert "rank 0 was never stopped" not in r.stdout
