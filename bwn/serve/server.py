"""HTTP server with the OpenAI API (``/v1/completions``,
``/v1/chat/completions``, ``/v1/models``, streaming; :mod:`bwn.serve.api`) plus
``/health`` and ``/metrics``.

Prompts are token ids, or text when a tokenizer is loaded (``--tokenizer``,
by default the checkpoint directory's).  Three schedulers:

* ``static`` (:class:`BatchingWorker`): a worker thread drains the queue into
  batches of at most ``max_batch`` requests (waiting up to ``batch_window_ms``
  for a batch to fill) and runs each batch to completion through
  :class:`~bwn.serve.engine.GenerationEngine`;
* ``continuous`` (:class:`ContinuousWorker`): requests join and leave the
  running batch between decode steps (:class:`~bwn.serve.continuous.ContinuousEngine`);
* ``spec``: EAGLE3 speculative decoding on batches of equal-length prompts
  (:class:`~bwn.serve.spec.SpecEngine` behind the batching worker).

    python -m bwn.serve.server --model tiny --port 8000 --scheduler continuous
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m bwn.serve.server --model 27b   # rank 0 serves HTTP
"""
from __future__ import annotations

import argparse
import queue
import threading
import time
from concurrent.futures import Future

from .api import build_app, load_tokenizer  # noqa: F401 - build_app is this module's app factory too
from .engine import GenerationEngine, Request


class LatencyStats:
    """Per-request TTFT (prefill) and TPOT (decode time per token after the
    first) for ``/metrics``: running sums and counts, and quantiles over the
    last ``window`` requests."""

    def __init__(self, window: int = 1000):
        from collections import deque
        self.lock = threading.Lock()
        self.vals = {"ttft_ms": deque(maxlen=window), "tpot_ms": deque(maxlen=window)}
        self.sums = {"ttft_ms": 0.0, "tpot_ms": 0.0}
        self.count = 0

    def record(self, res) -> None:
        tpot = res.decode_ms / max(1, len(res.tokens) - 1)
        with self.lock:
            for k, v in (("ttft_ms", res.prefill_ms), ("tpot_ms", tpot)):
                self.vals[k].append(v)
                self.sums[k] += v
            self.count += 1

    def prometheus(self) -> str:
        out = []
        with self.lock:
            for k, vals in self.vals.items():
                out.append(f"# TYPE bwn_{k} summary\n")
                srt = sorted(vals)
                for q in (0.5, 0.9, 0.99):
                    if srt:
                        out.append(f'bwn_{k}{{quantile="{q}"}} {srt[min(len(srt) - 1, int(q * len(srt)))]:.4f}\n')
                out.append(f"bwn_{k}_sum {self.sums[k]:.4f}\nbwn_{k}_count {self.count}\n")
        return "".join(out)


class BatchingWorker:
    def __init__(self, engine: GenerationEngine, batch_window_ms: float = 5.0):
        self.engine = engine
        self.window = batch_window_ms / 1e3
        self.q: queue.Queue = queue.Queue()
        self.stats = {"requests": 0, "batches": 0, "tokens": 0}
        self.latency = LatencyStats()
        self._stop = False
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def submit(self, req: Request) -> Future:
        fut: Future = Future()
        self.q.put((req, fut))
        return fut

    def _loop(self):
        while not self._stop:
            try:
                first = self.q.get(timeout=0.1)
            except queue.Empty:
                continue
            batch = [first]
            deadline = time.perf_counter() + self.window
            while len(batch) < self.engine.max_batch:
                left = deadline - time.perf_counter()
                if left <= 0:
                    break
                try:
                    batch.append(self.q.get(timeout=left))
                except queue.Empty:
                    break
            try:
                res = self.engine.generate([r for r, _ in batch])
                for (_, fut), out in zip(batch, res):
                    self.latency.record(out)
                    fut.set_result(out)
                self.stats["requests"] += len(batch)
                self.stats["batches"] += 1
                self.stats["tokens"] += sum(len(o.tokens) for o in res)
            except Exception as e:  # noqa: BLE001
                for _, fut in batch:
                    fut.set_exception(e)

    def stop(self):
        self._stop = True
        self.thread.join(timeout=5)
        if hasattr(self.engine, "stop"):  # followers of a multi-rank engine leave their loop
            self.engine.stop()


class ContinuousWorker:
    """One thread owns the engine: it admits queued requests, runs decode steps
    while any slot is busy, and completes each request's future when it finishes."""

    def __init__(self, engine, idle_poll_s: float = 0.05):
        self.engine = engine
        self.poll = idle_poll_s
        self.q: queue.Queue = queue.Queue()
        self.futs: dict[int, Future] = {}
        self.stats = {"requests": 0, "steps": 0, "tokens": 0}
        self.latency = LatencyStats()
        self._stop = False
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def submit(self, req: Request) -> Future:
        fut: Future = Future()
        self.q.put((req, fut))
        return fut

    def _drain(self, block: bool):
        try:
            item = self.q.get(timeout=self.poll) if block else self.q.get_nowait()
        except queue.Empty:
            return False
        while item is not None:
            req, fut = item
            try:
                self.futs[self.engine.add(req)] = fut
            except ValueError as e:
                fut.set_exception(e)
            try:
                item = self.q.get_nowait()
            except queue.Empty:
                item = None
        return True

    def _loop(self):
        while not self._stop:
            if self.engine.idle():
                self._drain(block=True)
                continue
            self._drain(block=False)
            try:
                finished = self.engine.step()
            except Exception as e:  # noqa: BLE001 - fail every request in flight, keep serving
                for fut in self.futs.values():
                    fut.set_exception(e)
                self.futs.clear()
                self.engine.abort_all()
                continue
            self.stats["steps"] += 1
            for rid, res in finished:
                self.stats["requests"] += 1
                self.stats["tokens"] += len(res.tokens)
                self.latency.record(res)
                self.futs.pop(rid).set_result(res)

    def gauges(self) -> dict:
        e = getattr(self.engine, "e", self.engine)  # a lockstep handle wraps the engine
        return {"running_requests": sum(s is not None for s in e.slots), "waiting_requests": len(e.waiting)}

    def stop(self):
        self._stop = True
        self.thread.join(timeout=5)
        if hasattr(self.engine, "stop"):  # followers of a multi-rank engine leave their loop
            self.engine.stop()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny", choices=["tiny", "27b", "35b"])
    ap.add_argument("--checkpoint", default="", help="HF safetensors directory (random init when empty)")
    ap.add_argument("--max-batch", type=int, default=8)
    ap.add_argument("--max-seq", type=int, default=4096)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--scheduler", default="continuous", choices=["continuous", "static", "spec"])
    ap.add_argument("--draft", default="", help="spec: EAGLE3 draft safetensors directory (random 1-layer when empty)")
    ap.add_argument("--num-draft", type=int, default=3, help="spec: draft tokens per step")
    ap.add_argument("--sampling", action="store_true", help="continuous scheduler: honour request temperatures")
    ap.add_argument("--tokenizer", default="", help="HF tokenizer directory (default: the checkpoint's, if any)")
    ap.add_argument("--served-model-name", default="", help="model id in responses (default: --model)")
    a = ap.parse_args()
    import torch
    import uvicorn

    from ..config import QWEN36_27B, QWEN36_35B_A3B, tiny_qwen36
    from ..models.qwen36 import Qwen36Model, from_pretrained
    from ..parallel.comm import init_distributed
    comm = init_distributed()  # torchrun: one rank per GPU, the model sharded over them
    dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    if a.checkpoint:
        model = from_pretrained(a.checkpoint, comm, dev)
    else:
        cfg = {"tiny": tiny_qwen36(), "27b": QWEN36_27B, "35b": QWEN36_35B_A3B}[a.model]
        model = Qwen36Model(cfg, comm, dev).init_random(0)
    if comm.size > 1 and dev.type == "cuda":
        from ..parallel.fused import enable_fused_comm
        try:
            enable_fused_comm(model)
        except RuntimeError as e:
            print(f"[server] fused NVLink comm unavailable, using NCCL: {e}")
    use_graph = dev.type == "cuda"
    if a.scheduler == "spec":
        from ..models.eagle3 import Eagle3Draft, eagle3_config
        from .spec import SpecEngine
        draft = Eagle3Draft(eagle3_config(model.cfg), dev, model.dtype)
        if a.draft:
            from ..io.checkpoint import Checkpoint
            ck = Checkpoint(a.draft, prefix="")
            draft.load({k: ck.raw(k) for k in ck.wm})
        else:
            draft.init_random(0)
        engine = SpecEngine(model, draft, a.max_batch, a.max_seq, a.num_draft, use_graph=use_graph)
    elif a.scheduler == "continuous":
        from .continuous import ContinuousEngine
        engine = ContinuousEngine(model, a.max_batch, a.max_seq, use_graph=use_graph, sampling=a.sampling)
    else:
        engine = GenerationEngine(model, a.max_batch, a.max_seq, use_graph=use_graph)
    if comm.size > 1:  # every rank runs the engine; rank 0 serves HTTP and leads
        from .lockstep import LockstepBatchEngine, LockstepEngine, control_group, follow
        ctrl = control_group()
        if comm.rank != 0:
            follow(engine, ctrl)
            return
        engine = (LockstepEngine if a.scheduler == "continuous" else LockstepBatchEngine)(engine, ctrl)
    worker = ContinuousWorker(engine) if a.scheduler == "continuous" else BatchingWorker(engine)
    codec = load_tokenizer(a.tokenizer or a.checkpoint)
    if a.tokenizer and codec is None:
        raise SystemExit(f"no tokenizer files in {a.tokenizer}")
    try:
        uvicorn.run(build_app(worker, a.served_model_name or a.model, codec), host=a.host, port=a.port)
    finally:
        worker.stop()


if __name__ == "__main__":
    main()
