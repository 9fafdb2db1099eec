"""Static decode engine: fixed-shape decode step captured once as a CUDA graph.

This is the B200 counterpart of the reference's compiled static forward
(``torch.compile(forward, backend="neuron", fullgraph=True, dynamic=False)``,
``contrib/qwen3.6-27b/static_decode.py:1183-1185``; the stateful full-graph
decode ``decode_step_stateful``, ``contrib/qwen3.6-35b-a3b/static_decode_35b.py:1600-1616``):

* all mutable state lives in static buffers (:class:`Qwen36State`), each with
  exactly one writer per step, so graph replays need no re-binding;
* the token ids and positions live on the device; the greedy next ids are
  written back into the input buffer inside the graph, so a device-side greedy
  loop needs no host round trip (``run_decode``, ``static_decode_35b.py:3142-3153``);
* :meth:`StaticDecoder.step` is the host API: pinned H2D of the step's tokens,
  graph replay, D2H of the next ids.
"""
from __future__ import annotations

import torch

from ..ops import check_status


class StaticDecoder:
    def __init__(self, model, batch: int, max_seq: int, use_graph: bool = True, ssm_dtype=torch.float32):
        self.model = model
        self.batch = batch
        self.max_seq = max_seq
        self.st = model.new_state(batch, max_seq, ssm_dtype)
        dev = model.device
        self.tokens = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.next_ids = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.use_graph = use_graph and dev.type == "cuda"
        self.graph: torch.cuda.CUDAGraph | None = None
        self._host_in = torch.zeros(batch, dtype=torch.int32, pin_memory=dev.type == "cuda")
        self._host_out = torch.zeros(batch, dtype=torch.int32, pin_memory=dev.type == "cuda")

    # ---------------------------------------------------------------- state
    def reset(self) -> None:
        self.st.reset()

    def prefill(self, prompt: torch.Tensor, valid_len: torch.Tensor | None = None, bucket: int = 0) -> torch.Tensor:
        """Run the prompt ``[B, S]`` through the model; the first generated ids
        become the next decode input.  Returns the ids ``[B]`` (device)."""
        ids = self.model.prefill(prompt.to(self.model.device), self.st, valid_len, bucket)
        self.tokens.copy_(ids)
        return ids

    # ----------------------------------------------------------------- step
    def _step_body(self) -> None:
        ids = self.model.decode_step(self.tokens, self.st)
        self.next_ids.copy_(ids)
        self.tokens.copy_(ids)

    def capture(self) -> None:
        """Warm up one step eagerly (sizes kernel scratch), capture the decode step
        as a CUDA graph, then zero the state.  Call before :meth:`prefill`."""
        if not self.use_graph:
            return
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._step_body()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        check_status("decode warm-up")
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self._step_body()
        torch.cuda.synchronize()
        self.graph = g
        self.reset()
        self.tokens.zero_()

    def release(self) -> None:
        """Drop the graph (must happen before destroying a process group whose
        collectives it captured)."""
        self.graph = None

    def step_device(self) -> None:
        """One decode step entirely on the device (input = previous ids)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._step_body()

    def step(self, host_tokens: torch.Tensor | None = None) -> torch.Tensor:
        """Public per-step API: H2D copy of ``host_tokens [B]`` (if given),
        one decode step, D2H of the next ids.  Returns a host int32 tensor."""
        if host_tokens is not None:
            self._host_in.copy_(host_tokens)
            self.tokens.copy_(self._host_in, non_blocking=True)
        self.step_device()
        self._host_out.copy_(self.next_ids, non_blocking=True)
        if self.model.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        return self._host_out.clone()

    def generate(self, prompt: torch.Tensor, steps: int, bucket: int = 0) -> torch.Tensor:
        """Greedy generation: prefill then ``steps`` device-side decode steps."""
        first = self.prefill(prompt, bucket=bucket)
        out = [first.clone()]
        for _ in range(steps - 1):
            self.step_device()
            out.append(self.next_ids.clone())
        check_status("generate")
        return torch.stack(out, 1)
