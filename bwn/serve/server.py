"""HTTP completion server (``/v1/completions``, ``/health``, ``/metrics``).

Requests carry token ids (``prompt``: list of ints; a tokenizer is outside the
framework).  A worker thread drains the queue into batches of at most
``max_batch`` requests (waiting up to ``batch_window_ms`` for a batch to fill)
and runs them through :class:`~bwn.serve.engine.GenerationEngine`.

    python -m bwn.serve.server --model tiny --port 8000
"""
from __future__ import annotations

import argparse
import queue
import threading
import time
from concurrent.futures import Future

from pydantic import BaseModel

from .engine import GenerationEngine, Request


class CompletionIn(BaseModel):
    prompt: list[int]
    max_tokens: int = 16
    stop: list[int] = []


class BatchingWorker:
    def __init__(self, engine: GenerationEngine, batch_window_ms: float = 5.0):
        self.engine = engine
        self.window = batch_window_ms / 1e3
        self.q: queue.Queue = queue.Queue()
        self.stats = {"requests": 0, "batches": 0, "tokens": 0}
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


def build_app(worker: BatchingWorker, model_name: str = "bwn"):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import PlainTextResponse

    app = FastAPI(title="bwn")

    @app.get("/health")
    def health():
        return {"status": "ok", "model": model_name}

    @app.post("/v1/completions")
    def completions(body: CompletionIn):
        if not body.prompt:
            raise HTTPException(400, "prompt must hold at least one token id")
        try:
            out = worker.submit(Request(body.prompt, body.max_tokens, body.stop)).result(timeout=600)
        except ValueError as e:
            raise HTTPException(400, str(e)) from e
        return {"object": "text_completion", "model": model_name,
                "choices": [{"index": 0, "tokens": out.tokens, "finish_reason": out.finish_reason}],
                "usage": {"prompt_tokens": len(body.prompt), "completion_tokens": len(out.tokens)},
                "timing_ms": {"prefill": round(out.prefill_ms, 3), "decode": round(out.decode_ms, 3)}}

    @app.get("/metrics", response_class=PlainTextResponse)
    def metrics():
        s = worker.stats
        return "".join(f"bwn_{k}_total {v}\n" for k, v in s.items())

    return app


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny", choices=["tiny", "27b", "35b"])
    ap.add_argument("--checkpoint", default="", help="HF safetensors directory (random init when empty)")
    ap.add_argument("--max-batch", type=int, default=8)
    ap.add_argument("--max-seq", type=int, default=4096)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    a = ap.parse_args()
    import torch
    import uvicorn

    from ..config import QWEN36_27B, QWEN36_35B_A3B, tiny_qwen36
    from ..models.qwen36 import Qwen36Model, from_pretrained
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    if a.checkpoint:
        model = from_pretrained(a.checkpoint, None, dev)
    else:
        cfg = {"tiny": tiny_qwen36(), "27b": QWEN36_27B, "35b": QWEN36_35B_A3B}[a.model]
        model = Qwen36Model(cfg, None, dev).init_random(0)
    worker = BatchingWorker(GenerationEngine(model, a.max_batch, a.max_seq, use_graph=dev == "cuda"))
    uvicorn.run(build_app(worker, a.model), host=a.host, port=a.port)


if __name__ == "__main__":
    main()
