"""Generation engine (static batches, right-padded prompts, stop ids) and the
HTTP completion server, on the tiny Qwen3.6 model on the CPU."""
import torch

from bwn.config import tiny_qwen36
from bwn.models.qwen36 import build_qwen36
from bwn.serve.engine import GenerationEngine, Request


def _greedy(model, prompt, n):
    st = model.new_state(1, len(prompt) + n + 8)
    tok = model.prefill(torch.tensor([prompt]), st)
    out = [int(tok[0])]
    for _ in range(n - 1):
        tok = model.decode_step(tok, st)
        out.append(int(tok[0]))
    return out


def test_engine_matches_single_sequence_greedy():
    model = build_qwen36(tiny_qwen36(layers=4), device="cpu", dtype=torch.float32)
    eng = GenerationEngine(model, max_batch=4, max_seq=128, use_graph=False, pad_to=16)
    prompts = [[5, 9, 13, 2, 7], [100, 3], [42] * 11]
    res = eng.generate([Request(p, 6) for p in prompts])
    for p, r in zip(prompts, res):
        assert r.tokens == _greedy(model, p, 6) and r.finish_reason == "length"
    # a second batch reuses the decoder state
    r2 = eng.generate([Request(prompts[1], 3)])[0]
    assert r2.tokens == _greedy(model, prompts[1], 3)
    # stop id
    want = _greedy(model, prompts[0], 6)
    r3 = eng.generate([Request(prompts[0], 6, stop=[want[2]])])[0]
    assert r3.tokens == want[:want.index(want[2]) + 1] and r3.finish_reason == "stop"


def test_http_server():
    from fastapi.testclient import TestClient

    from bwn.serve.server import BatchingWorker, build_app
    model = build_qwen36(tiny_qwen36(layers=4), device="cpu", dtype=torch.float32)
    worker = BatchingWorker(GenerationEngine(model, 2, 128, use_graph=False, pad_to=16), batch_window_ms=2)
    client = TestClient(build_app(worker, "tiny"))
    assert client.get("/health").json()["status"] == "ok"
    r = client.post("/v1/completions", json={"prompt": [5, 9, 13], "max_tokens": 4})
    assert r.status_code == 200
    body = r.json()
    assert body["choices"][0]["tokens"] == _greedy(model, [5, 9, 13], 4)
    assert client.post("/v1/completions", json={"prompt": [], "max_tokens": 4}).status_code == 400
    assert "bwn_requests_total 1" in client.get("/metrics").text
    worker.stop()
