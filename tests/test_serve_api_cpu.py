"""The OpenAI-compatible HTTP API on the tiny Qwen3.6 model (CPU): text
prompts through a local HF tokenizer, chat templates, stop strings, EOS,
server-sent-event streaming from the continuous and the static scheduler."""
import json

import pytest
import torch

from bwn.config import tiny_qwen36
from bwn.models.qwen36 import build_qwen36
from bwn.serve.engine import GenerationEngine

VOCAB = 512


def _greedy(model, prompt, n):
    st = model.new_state(1, len(prompt) + n + 8)
    tok = model.prefill(torch.tensor([prompt]), st)
    out = [int(tok[0])]
    for _ in range(n - 1):
        tok = model.decode_step(tok, st)
        out.append(int(tok[0]))
    return out


def _tokenizer(path, eos_id=VOCAB - 1):
    """A word-level tokenizer: token ``w<i>`` is id i, words joined by spaces;
    the chat template writes ``<role> <content>`` per message, then ``w1``."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    vocab = {f"w{i}": i for i in range(VOCAB)}
    tk = Tokenizer(models.WordLevel(vocab, unk_token="w0"))
    tk.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tk.decoder = decoders.WordPiece(prefix="##")
    f = PreTrainedTokenizerFast(tokenizer_object=tk, eos_token=f"w{eos_id}", unk_token="w0")
    f.chat_template = ("{% for m in messages %}{{ m['role'] }} {{ m['content'] }} {% endfor %}"
                       "{% if add_generation_prompt %}w1 {% endif %}")
    f.save_pretrained(str(path))
    from bwn.serve.api import load_tokenizer
    return load_tokenizer(str(path))


def _text(ids):
    return " ".join(f"w{i}" for i in ids)


def _sse(resp):
    lines = [ln[len("data: "):] for ln in resp.text.split("\n") if ln.startswith("data: ")]
    assert lines[-1] == "[DONE]"
    return [json.loads(x) for x in lines[:-1]]


@pytest.fixture(scope="module")
def model():
    return build_qwen36(tiny_qwen36(layers=4), device="cpu", dtype=torch.float32)


def _continuous_client(model, codec):
    from fastapi.testclient import TestClient

    from bwn.serve.continuous import ContinuousEngine
    from bwn.serve.server import ContinuousWorker, build_app
    worker = ContinuousWorker(ContinuousEngine(model, 2, 64, use_graph=False))
    return TestClient(build_app(worker, "tiny", codec)), worker


def test_text_prompt_stop_strings_and_eos(model, tmp_path):
    prompt = [5, 9, 13]
    want = _greedy(model, prompt, 6)
    codec = _tokenizer(tmp_path / "tok", eos_id=want[3])
    client, worker = _continuous_client(model, codec)
    try:
        assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"
        # the tokenizer's EOS stops generation unless ignore_eos
        k = want.index(want[3]) + 1  # generation stops at the first EOS
        r = client.post("/v1/completions", json={"prompt": _text(prompt), "max_tokens": 6}).json()
        assert r["choices"][0]["tokens"] == want[:k] and r["choices"][0]["finish_reason"] == "stop"
        assert r["choices"][0]["text"] == _text(want[:k - 1])  # EOS is a special token: not in the text
        assert r["usage"] == {"prompt_tokens": 3, "completion_tokens": k, "total_tokens": 3 + k}
        r = client.post("/v1/completions", json={"prompt": _text(prompt), "max_tokens": 6, "ignore_eos": True}).json()
        assert r["choices"][0]["tokens"] == want and r["choices"][0]["finish_reason"] == "length"
        # a single-token stop string, and a two-token one (stops where the output first ends with it)
        r = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 6, "ignore_eos": True,
                                                 "stop": [f"w{want[1]}"]}).json()
        assert r["choices"][0]["tokens"] == want[:want.index(want[1]) + 1]
        seq = want[2:4]
        end = next(i + 2 for i in range(len(want) - 1) if want[i:i + 2] == seq)
        r = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 6, "ignore_eos": True,
                                                 "stop": _text(seq)}).json()
        assert r["choices"][0]["tokens"] == want[:end] and r["choices"][0]["finish_reason"] == "stop"
        assert client.post("/v1/completions", json={"prompt": prompt, "stop": " "}).status_code == 400
    finally:
        worker.stop()


def test_streaming_continuous(model, tmp_path):
    prompt = [7, 7, 2, 1, 30]
    want = _greedy(model, prompt, 5)
    client, worker = _continuous_client(model, _tokenizer(tmp_path / "tok"))
    try:
        r = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 5, "stream": True})
        assert r.status_code == 200 and r.headers["content-type"].startswith("text/event-stream")
        chunks = _sse(r)
        assert [c["choices"][0]["tokens"] for c in chunks[:-1]] == [[t] for t in want]
        assert "".join(c["choices"][0]["text"] for c in chunks) == " ".join(f"w{t}" for t in want)
        assert chunks[-1]["choices"][0]["finish_reason"] == "length"
        chunks = _sse(client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 5, "stream": True,
                                                           "stream_options": {"include_usage": True}}))
        assert chunks[-1]["choices"] == [] and chunks[-1]["usage"] == {
            "prompt_tokens": 5, "completion_tokens": 5, "total_tokens": 10}
        # a request that cannot fit is refused with a 400 before any event is sent
        r = client.post("/v1/completions", json={"prompt": [1] * 60, "max_tokens": 10, "stream": True})
        assert r.status_code == 400 and "max_seq" in r.json()["detail"]
    finally:
        worker.stop()


def test_streaming_static_scheduler_without_tokenizer(model):
    from fastapi.testclient import TestClient

    from bwn.serve.server import BatchingWorker, build_app
    worker = BatchingWorker(GenerationEngine(model, 2, 128, use_graph=False, pad_to=16), batch_window_ms=2)
    client = TestClient(build_app(worker, "tiny"))
    try:
        want = _greedy(model, [5, 9, 13], 4)
        chunks = _sse(client.post("/v1/completions", json={"prompt": [5, 9, 13], "max_tokens": 4, "stream": True}))
        assert sum((c["choices"][0]["tokens"] for c in chunks), []) == want
        assert chunks[-1]["choices"][0]["finish_reason"] == "length"
        assert all(c["choices"][0]["text"] is None for c in chunks)
        # text and chat need a tokenizer
        assert client.post("/v1/completions", json={"prompt": "w5 w9"}).status_code == 400
        assert client.post("/v1/chat/completions",
                           json={"messages": [{"role": "user", "content": "hi"}]}).status_code == 400
    finally:
        worker.stop()


def test_chat_completions(model, tmp_path):
    codec = _tokenizer(tmp_path / "tok")
    msgs = [{"role": "w2", "content": "w5 w6"}, {"role": "w3", "content": "w40"}]
    prompt = [2, 5, 6, 3, 40, 1]
    assert codec.chat(msgs) == prompt
    want = _greedy(model, prompt, 4)
    client, worker = _continuous_client(model, codec)
    try:
        r = client.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 4}).json()
        assert r["object"] == "chat.completion"
        assert r["choices"][0]["message"] == {"role": "assistant", "content": _text(want)}
        assert r["usage"]["prompt_tokens"] == len(prompt)
        chunks = _sse(client.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 4, "stream": True}))
        assert chunks[0]["choices"][0]["delta"]["role"] == "assistant"
        assert "".join(c["choices"][0]["delta"].get("content", "") for c in chunks) == _text(want)
        assert chunks[-1]["choices"][0]["finish_reason"] == "length"
        r = client.post("/v1/chat/completions", json={"messages": msgs, "max_completion_tokens": 2, "n": 2}).json()
        assert [c["message"]["content"] for c in r["choices"]] == [_text(want[:2])] * 2
        assert r["usage"]["completion_tokens"] == 4
    finally:
        worker.stop()


def test_metrics_latency_summaries(model):
    client, worker = _continuous_client(model, None)
    try:
        for p in ([5, 9, 13], [7, 2]):
            assert client.post("/v1/completions", json={"prompt": p, "max_tokens": 3}).status_code == 200
        text = client.get("/metrics").text
        assert "bwn_requests_total 2" in text
        assert "bwn_ttft_ms_count 2" in text and "bwn_tpot_ms_count 2" in text
        assert 'bwn_ttft_ms{quantile="0.5"}' in text
        assert "bwn_running_requests 0" in text and "bwn_waiting_requests 0" in text
    finally:
        worker.stop()


def test_stop_sequences_in_static_engine(model):
    from bwn.serve.engine import Request
    r = Request([1], 8, stop=[3], stop_seqs=[[4, 5]])
    assert not r.stopped([]) and r.stopped([9, 3]) and r.stopped([1, 4, 5]) and not r.stopped([4, 5, 6])
    want = _greedy(model, [5, 9, 13], 6)
    seq = want[3:5]
    end = next(i + 2 for i in range(len(want) - 1) if want[i:i + 2] == seq)
    eng = GenerationEngine(model, 2, 128, use_graph=False, pad_to=16)
    res = eng.generate([Request([5, 9, 13], 6, stop_seqs=[seq]), Request([5, 9, 13], 6)])
    assert res[0].tokens == want[:end] and res[0].finish_reason == "stop"
    assert res[1].tokens == want and res[1].finish_reason == "length"


def test_prompt_lists_give_one_choice_each(model, tmp_path):
    client, worker = _continuous_client(model, _tokenizer(tmp_path / "tok"))
    try:
        ps = [[5, 9, 13], [7, 2]]
        r = client.post("/v1/completions", json={"prompt": ps, "max_tokens": 3, "ignore_eos": True}).json()
        assert [c["index"] for c in r["choices"]] == [0, 1]
        assert [c["tokens"] for c in r["choices"]] == [_greedy(model, p, 3) for p in ps]
        assert r["usage"]["prompt_tokens"] == 5 and r["usage"]["completion_tokens"] == 6
        r = client.post("/v1/completions", json={"prompt": ["w5 w9 w13", "w7 w2"], "max_tokens": 3,
                                                 "ignore_eos": True}).json()
        assert [c["tokens"] for c in r["choices"]] == [_greedy(model, p, 3) for p in ps]
        assert client.post("/v1/completions", json={"prompt": ps, "stream": True}).status_code == 400
        r = client.post("/v1/completions", json={"prompt": ps, "max_tokens": 2, "n": 2, "ignore_eos": True}).json()
        assert [c["tokens"] for c in r["choices"]] == [_greedy(model, p, 2) for p in ps for _ in range(2)]
        # each prompt counted once in usage whatever n; n is capped
        assert r["usage"]["prompt_tokens"] == 5 and r["usage"]["completion_tokens"] == 8
        assert client.post("/v1/completions", json={"prompt": ps, "n": 1000}).status_code == 400
    finally:
        worker.stop()
