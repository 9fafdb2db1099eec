"""OpenAI-compatible HTTP surface of the server.

The reference serves its models through a vLLM fork, whose OpenAI API is what
its users call (``contrib/qwen3.6-27b/deploy/serve_qwen35.sh``,
``serve_eagle3.sh``; ``contrib/qwen3.6-35b-a3b/VLLM_NEURON_ASSESSMENT.md``).
This module gives the same endpoints over the bwn engines:

* ``POST /v1/completions``: ``prompt`` as token ids or text, or a list of
  them (``n`` choices each); ``max_tokens``,
  ``temperature``, ``stop`` (token ids, or strings: generation stops once the
  output ends with the string's tokens),
  ``stop_token_ids``, ``ignore_eos``, ``stream`` (server-sent events, one
  chunk per token as the continuous engine produces it, then ``[DONE]``);
* ``POST /v1/chat/completions``: ``messages`` rendered by the tokenizer's chat
  template; the reply as ``message`` (or ``delta`` chunks when streaming);
* ``GET /v1/models``, ``GET /health``, ``GET /metrics`` (Prometheus text).

Text needs a tokenizer: a local HF tokenizer directory (usually the checkpoint
directory) loaded with ``transformers`` offline.  Without one the server takes
and returns token ids only.  Every choice carries ``tokens`` (the generated
ids) beside ``text``.
"""
from __future__ import annotations

import itertools
import json
import queue
import time

from pydantic import BaseModel

from .engine import Request

_ids = itertools.count()


class CompletionIn(BaseModel):
    prompt: list[int] | str | list[str] | list[list[int]]
    max_tokens: int = 16
    n: int = 1  # completions per prompt (distinct only when sampled)
    stop: list[int] | list[str] | str | None = None
    stop_token_ids: list[int] = []
    temperature: float = 0.0
    ignore_eos: bool = False
    stream: bool = False
    stream_options: dict | None = None  # {"include_usage": true}: a last chunk with usage
    model: str | None = None


class ChatMessage(BaseModel):
    role: str
    content: str


class ChatIn(BaseModel):
    messages: list[ChatMessage]
    max_tokens: int = 16
    max_completion_tokens: int | None = None  # the newer name of max_tokens; wins when given
    n: int = 1
    stop: list[int] | list[str] | str | None = None
    stop_token_ids: list[int] = []
    temperature: float = 0.0
    ignore_eos: bool = False
    stream: bool = False
    stream_options: dict | None = None  # {"include_usage": true}: a last chunk with usage
    model: str | None = None


class TextCodec:
    """Token ids <-> text through a local HF tokenizer."""

    def __init__(self, tokenizer):
        self.tok = tokenizer
        eos = getattr(tokenizer, "eos_token_id", None)
        self.eos = [] if eos is None else ([int(e) for e in eos] if isinstance(eos, (list, tuple)) else [int(eos)])

    def encode(self, text: str) -> list[int]:
        return [int(i) for i in self.tok.encode(text, add_special_tokens=False)]

    def decode(self, ids: list[int]) -> str:
        return self.tok.decode(ids, skip_special_tokens=True)

    def chat(self, messages: list[dict]) -> list[int]:
        out = self.tok.apply_chat_template(messages, add_generation_prompt=True, tokenize=True)
        if hasattr(out, "keys"):  # a BatchEncoding
            out = out["input_ids"]
        return [int(i) for i in out]

    def stop_tokens(self, s: str) -> list[int]:
        ids = self.encode(s)
        if not ids:
            raise ValueError(f"stop string {s!r} encodes to no tokens")
        return ids


def load_tokenizer(path: str) -> TextCodec | None:
    """The HF tokenizer saved in ``path`` (``tokenizer.json`` /
    ``tokenizer_config.json``), or None when the directory has none."""
    import os
    if not path or not any(os.path.exists(os.path.join(path, f))
                           for f in ("tokenizer.json", "tokenizer_config.json", "tokenizer.model")):
        return None
    from transformers import AutoTokenizer
    return TextCodec(AutoTokenizer.from_pretrained(path, local_files_only=True))


class _Incremental:
    """Streams text deltas: the decode of every id so far, minus what was sent
    (a multi-token character appears once it is complete)."""

    def __init__(self, codec: TextCodec | None):
        self.codec, self.ids, self.sent = codec, [], ""

    def push(self, tok: int) -> str | None:
        self.ids.append(tok)
        if self.codec is None:
            return None
        text = self.codec.decode(self.ids)
        if text.endswith("�"):  # an incomplete byte sequence: wait for the next token
            return ""
        delta, self.sent = text[len(self.sent):], text
        return delta


def _usage(body, n_prompt: int):
    """The usage reporter of a streamed request that asked for it, else None."""
    if not (body.stream_options or {}).get("include_usage"):
        return None
    return lambda res: {"prompt_tokens": n_prompt, "completion_tokens": len(res.tokens),
                        "total_tokens": n_prompt + len(res.tokens)}


def build_app(worker, model_name: str = "bwn", codec: TextCodec | None = None, max_n: int = 16):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import PlainTextResponse, StreamingResponse

    app = FastAPI(title="bwn")

    def stop_ids(body) -> tuple[list[int], list[list[int]]]:
        """(stop ids, stop sequences): a stop string of one token is a stop
        id; a longer one stops when the output ends with its encoding."""
        out, seqs = list(body.stop_token_ids), []
        stops = [body.stop] if isinstance(body.stop, (str, int)) else (body.stop or [])
        for s in stops:
            if isinstance(s, int):
                out.append(s)
            elif codec is None:
                raise HTTPException(400, "stop strings need a tokenizer (--tokenizer)")
            else:
                try:
                    ids = codec.stop_tokens(s)
                except ValueError as e:
                    raise HTTPException(400, str(e)) from e
                (out.append(ids[0]) if len(ids) == 1 else seqs.append(ids))
        if codec is not None and not body.ignore_eos:
            out += [e for e in codec.eos if e not in out]
        return out, seqs

    def submit(prompt: list[int], body, stream: bool):
        """Validate and queue one request; returns (future, token queue)."""
        if not prompt:
            raise HTTPException(400, "prompt must hold at least one token id")
        eng = getattr(worker, "engine", None)
        eng = getattr(eng, "e", eng)  # a lockstep handle wraps the engine
        max_seq = getattr(eng, "max_seq", None)
        if max_seq is not None and len(prompt) + body.max_tokens > max_seq:  # refused before any stream starts
            raise HTTPException(400, f"prompt ({len(prompt)}) + {body.max_tokens} new tokens exceed "
                                     f"max_seq {max_seq}")
        q: queue.Queue = queue.Queue()
        stop, seqs = stop_ids(body)
        req = Request(prompt, body.max_tokens, stop, body.temperature, on_token=q.put if stream else None,
                      stop_seqs=seqs)
        return worker.submit(req), q

    def wait(fut):
        try:
            return fut.result(timeout=600)
        except ValueError as e:
            raise HTTPException(400, str(e)) from e

    def run(prompt: list[int], body, stream: bool):
        fut, q = submit(prompt, body, stream)
        return (fut, q) if stream else (wait(fut), None)

    def to_ids(p) -> list[int]:
        if isinstance(p, str):
            if codec is None:
                raise HTTPException(400, "text prompts need a tokenizer (--tokenizer); send token ids")
            return codec.encode(p)
        return p

    def events(fut, q, chunk, usage_of=None):
        """SSE body: one chunk per token while the engine produces them, the
        rest (engines that finish a request at once) after it completes, then
        a final chunk with the finish reason and ``[DONE]``."""
        inc = _Incremental(codec)
        n = 0
        while True:
            try:
                tok = q.get(timeout=0.05)
            except queue.Empty:
                if fut.done():
                    break
                continue
            n += 1
            yield "data: " + json.dumps(chunk([tok], inc.push(tok), None)) + "\n\n"
        try:
            res = fut.result()
        except Exception as e:  # noqa: BLE001 - headers are sent: report in the stream
            yield "data: " + json.dumps({"error": {"message": str(e)}}) + "\n\n"
            yield "data: [DONE]\n\n"
            return
        while not q.empty():  # tokens queued after the last poll
            q.get_nowait()
        rest = res.tokens[n:]
        for tok in rest:
            yield "data: " + json.dumps(chunk([tok], inc.push(tok), None)) + "\n\n"
        yield "data: " + json.dumps(chunk([], "" if codec else None, res.finish_reason)) + "\n\n"
        if usage_of is not None:  # stream_options.include_usage: usage in a chunk without choices
            last = chunk([], None, None)
            last["choices"], last["usage"] = [], usage_of(res)
            yield "data: " + json.dumps(last) + "\n\n"
        yield "data: [DONE]\n\n"

    @app.get("/health")
    def health():
        return {"status": "ok", "model": model_name}

    @app.get("/v1/models")
    def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "bwn"}]}

    @app.post("/v1/completions")
    def completions(body: CompletionIn):
        """One prompt (ids or text), or a list of prompts: one choice each,
        queued together so the engine batches them."""
        many = isinstance(body.prompt, list) and bool(body.prompt) and not isinstance(body.prompt[0], int)
        prompts = [to_ids(p) for p in body.prompt] if many else [to_ids(body.prompt)]
        if not 1 <= body.n <= max_n:
            raise HTTPException(400, f"n must be in [1, {max_n}]")
        cid, created = f"cmpl-{next(_ids)}", int(time.time())
        if body.stream:
            if many or body.n > 1:
                raise HTTPException(400, "streaming takes a single prompt and n = 1")
            fut, q = run(prompts[0], body, True)

            def chunk(toks, text, fin):
                return {"id": cid, "object": "text_completion", "created": created, "model": model_name,
                        "choices": [{"index": 0, "text": text, "tokens": toks, "finish_reason": fin}]}
            return StreamingResponse(events(fut, q, chunk, _usage(body, len(prompts[0]))),
                                     media_type="text/event-stream")
        n_in = sum(map(len, prompts))  # each prompt counted once, whatever n (as chat and OpenAI count)
        prompts = [p for p in prompts for _ in range(body.n)]  # choice i*n + j: prompt i, sample j
        futs = [submit(p, body, False)[0] for p in prompts]
        outs = [wait(f) for f in futs]
        n_out = sum(len(o.tokens) for o in outs)
        return {"id": cid, "object": "text_completion", "created": created, "model": model_name,
                "choices": [{"index": i, "text": codec.decode(o.tokens) if codec else None,
                             "tokens": o.tokens, "finish_reason": o.finish_reason} for i, o in enumerate(outs)],
                "usage": {"prompt_tokens": n_in, "completion_tokens": n_out, "total_tokens": n_in + n_out},
                "timing_ms": {"prefill": round(max(o.prefill_ms for o in outs), 3),
                              "decode": round(max(o.decode_ms for o in outs), 3)}}

    @app.post("/v1/chat/completions")
    def chat(body: ChatIn):
        if codec is None:
            raise HTTPException(400, "chat needs a tokenizer with a chat template (--tokenizer)")
        try:
            prompt = codec.chat([m.model_dump() for m in body.messages])
        except Exception as e:  # noqa: BLE001 - a template that cannot render these messages
            raise HTTPException(400, f"chat template: {e}") from e
        if body.max_completion_tokens is not None:
            body = body.model_copy(update={"max_tokens": body.max_completion_tokens})
        if not 1 <= body.n <= max_n or (body.stream and body.n > 1):
            raise HTTPException(400, f"n must be in [1, {max_n}], and 1 when streaming")
        cid, created = f"chatcmpl-{next(_ids)}", int(time.time())
        if body.stream:
            out, q = run(prompt, body, True)
            first = [True]

            def chunk(toks, text, fin):
                delta = {"content": text} if text else {}
                if first[0]:
                    delta["role"], first[0] = "assistant", False
                return {"id": cid, "object": "chat.completion.chunk", "created": created, "model": model_name,
                        "choices": [{"index": 0, "delta": delta, "tokens": toks, "finish_reason": fin}]}
            return StreamingResponse(events(out, q, chunk, _usage(body, len(prompt))), media_type="text/event-stream")
        outs = [wait(f) for f in [submit(prompt, body, False)[0] for _ in range(body.n)]]
        n_out = sum(len(o.tokens) for o in outs)
        return {"id": cid, "object": "chat.completion", "created": created, "model": model_name,
                "choices": [{"index": i, "message": {"role": "assistant", "content": codec.decode(o.tokens)},
                             "tokens": o.tokens, "finish_reason": o.finish_reason} for i, o in enumerate(outs)],
                "usage": {"prompt_tokens": len(prompt), "completion_tokens": n_out,
                          "total_tokens": len(prompt) + n_out}}

    @app.get("/metrics", response_class=PlainTextResponse)
    def metrics():
        """Prometheus text: counters, request latency summaries (TTFT, TPOT),
        and the continuous scheduler's running / waiting gauges."""
        out = "".join(f"bwn_{k}_total {v}\n" for k, v in worker.stats.items())
        if hasattr(worker, "latency"):
            out += worker.latency.prometheus()
        if hasattr(worker, "gauges"):
            out += "".join(f"bwn_{k} {v}\n" for k, v in worker.gauges().items())
        return out

    return app
