"""Generation engine (static batches, right-padded prompts, stop ids) and the
HTTP completion server, on the tiny Qwen3.6 model on the CPU."""
import pytest
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


def test_continuous_batching_matches_solo_generation():
    """Five requests of different lengths through two slots: requests join and
    leave the running batch between steps, and each one's tokens equal its
    generation alone; idle slots stay inside their caches although the run is
    longer than max_seq."""
    from bwn.config import tiny_qwen36
    from bwn.models.qwen36 import build_qwen36
    from bwn.runtime.static_decode import StaticDecoder
    from bwn.serve.continuous import ContinuousEngine
    from bwn.serve.engine import Request
    cfg = tiny_qwen36()
    m = build_qwen36(cfg, seed=11, dtype=torch.float32)
    g = torch.Generator().manual_seed(4)
    reqs = [Request(torch.randint(0, cfg.vocab, (n,), generator=g).tolist(), max_tokens=t)
            for n, t in [(5, 6), (9, 3), (3, 8), (7, 1), (4, 5)]]
    solo = []
    for q in reqs:
        d = StaticDecoder(m, 1, 32, use_graph=False)
        solo.append(d.generate(torch.tensor([q.prompt]), q.max_tokens)[0].tolist())
    eng = ContinuousEngine(m, max_batch=2, max_seq=24, use_graph=False)
    res = eng.run(reqs)
    assert [r.tokens for r in res] == solo
    assert all(r.finish_reason == "length" for r in res)
    assert eng.stats["admitted"] == 5 and eng.stats["finished"] == 5
    # a stop id ends a request early and frees its slot
    stop_at = solo[2][2]
    res2 = eng.run([Request(reqs[2].prompt, max_tokens=8, stop=[stop_at])])
    assert res2[0].tokens == solo[2][:solo[2].index(stop_at) + 1] and res2[0].finish_reason == "stop"
    # one long request beside an idle slot: more steps than max_seq rows would allow an idle row
    eng2 = ContinuousEngine(m, max_batch=2, max_seq=24, use_graph=False)
    long = Request(reqs[0].prompt, max_tokens=18)
    ref = StaticDecoder(m, 1, 32, use_graph=False).generate(torch.tensor([long.prompt]), 18)[0].tolist()
    assert eng2.run([long])[0].tokens == ref
    assert int(eng2.dec.st.positions[1]) <= 1  # pinned to 0 before every step
    with pytest.raises(ValueError):
        eng2.add(Request([1] * 20, max_tokens=10))


def test_http_server_continuous_scheduler():
    """Concurrent HTTP requests through the continuous scheduler: each answer
    equals the request's solo greedy tokens; a request that cannot fit is a 400."""
    from concurrent.futures import ThreadPoolExecutor

    from fastapi.testclient import TestClient

    from bwn.serve.continuous import ContinuousEngine
    from bwn.serve.server import ContinuousWorker, build_app
    model = build_qwen36(tiny_qwen36(layers=4), device="cpu", dtype=torch.float32)
    worker = ContinuousWorker(ContinuousEngine(model, 2, 64, use_graph=False))
    client = TestClient(build_app(worker, "tiny"))
    prompts = [([5, 9, 13], 4), ([7, 7, 2, 1, 30], 6), ([100], 3), ([3, 4], 5)]
    with ThreadPoolExecutor(4) as ex:
        rs = list(ex.map(lambda pt: client.post("/v1/completions", json={"prompt": pt[0], "max_tokens": pt[1]}),
                         prompts))
    for (p, t), r in zip(prompts, rs):
        assert r.status_code == 200
        assert r.json()["choices"][0]["tokens"] == _greedy(model, p, t)
    assert client.post("/v1/completions", json={"prompt": [1] * 60, "max_tokens": 10}).status_code == 400
    assert "bwn_requests_total 4" in client.get("/metrics").text
    worker.stop()


def test_continuous_sampling_engine():
    """With sampling on, temperature-0 requests still equal solo greedy
    generation and sampled requests are reproducible from the engine seed."""
    from bwn.runtime.static_decode import StaticDecoder
    from bwn.serve.continuous import ContinuousEngine
    from bwn.serve.engine import Request
    cfg = tiny_qwen36()
    m = build_qwen36(cfg, seed=11, dtype=torch.float32)
    p0, p1 = [5, 9, 13, 2], [7, 7, 1]
    solo = StaticDecoder(m, 1, 32, use_graph=False).generate(torch.tensor([p0]), 5)[0].tolist()

    def run(seed):
        eng = ContinuousEngine(m, max_batch=2, max_seq=24, use_graph=False, sampling=True, seed=seed)
        return eng.run([Request(p0, 5), Request(p1, 6, temperature=1.5)])

    a, b = run(3), run(3)
    assert a[0].tokens == solo
    assert a[1].tokens == b[1].tokens and len(a[1].tokens) == 6
    assert all(0 <= t < cfg.vocab for t in a[1].tokens)
    with pytest.raises(ValueError):
        ContinuousEngine(m, 2, 24, use_graph=False).add(Request(p0, 3, temperature=1.0))


def test_speculative_engine_matches_greedy():
    """EAGLE3 speculative serving (random 1-layer draft, 4 drafts per step):
    requests of mixed prompt lengths are grouped, and every request's tokens
    equal its plain greedy generation, also when the decoder is reused."""
    from bwn.models.eagle3 import Eagle3Draft, eagle3_config
    from bwn.runtime.static_decode import StaticDecoder
    from bwn.serve.engine import Request
    from bwn.serve.spec import SpecEngine
    cfg = tiny_qwen36()
    m = build_qwen36(cfg, seed=11, dtype=torch.float32)
    draft = Eagle3Draft(eagle3_config(cfg), "cpu", torch.float32).init_random(1)
    g = torch.Generator().manual_seed(9)
    reqs = [Request(torch.randint(0, cfg.vocab, (n,), generator=g).tolist(), max_tokens=t)
            for n, t in [(6, 7), (6, 4), (9, 5), (6, 9)]]
    solo = [StaticDecoder(m, 1, 48, use_graph=False).generate(torch.tensor([q.prompt]), q.max_tokens)[0].tolist()
            for q in reqs]
    eng = SpecEngine(m, draft, max_batch=2, max_seq=48, num_draft=4, use_graph=False)
    assert [r.tokens for r in eng.generate(reqs)] == solo
    assert [r.tokens for r in eng.generate(reqs[:2])] == solo[:2]  # decoder reuse after reset
    assert eng.stats["batches"] == 4 and eng.stats["steps"] > 0  # (6,6) (6) (9), then (6,6)


def test_http_server_spec_scheduler():
    from fastapi.testclient import TestClient

    from bwn.models.eagle3 import Eagle3Draft, eagle3_config
    from bwn.serve.server import BatchingWorker, build_app
    from bwn.serve.spec import SpecEngine
    cfg = tiny_qwen36(layers=4)
    model = build_qwen36(cfg, device="cpu", dtype=torch.float32)
    draft = Eagle3Draft(eagle3_config(cfg), "cpu", torch.float32).init_random(0)
    worker = BatchingWorker(SpecEngine(model, draft, 2, 64, 3, use_graph=False), batch_window_ms=2)
    client = TestClient(build_app(worker, "tiny-eagle3"))
    r = client.post("/v1/completions", json={"prompt": [5, 9, 13], "max_tokens": 6})
    assert r.status_code == 200 and r.json()["choices"][0]["tokens"] == _greedy(model, [5, 9, 13], 6)
    assert client.post("/v1/completions", json={"prompt": [5], "max_tokens": 3, "temperature": 1.0}).status_code == 400
    worker.stop()


def test_serve_bench_runs(capsys):
    import importlib.util
    import json
    import os
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "bench", "serve_bench.py")
    spec = importlib.util.spec_from_file_location("serve_bench", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.main(["--model", "tiny", "--cpu", "--concurrency", "1", "2", "--prompt-len", "8", "--max-tokens", "4"])
    lines = [json.loads(ln) for ln in capsys.readouterr().out.splitlines() if ln.startswith("{")]
    assert [x["concurrency"] for x in lines] == [1, 2]
    assert all(x["output_tok_s"] > 0 and x["requests"] == 4 for x in lines)
