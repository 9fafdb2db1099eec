"""CUDA prefill ops (chunked DeltaNet, prefix-aware flash attention)."""
from __future__ import annotations


def deltanet_prefill(*args, **kwargs):
    raise NotImplementedError("bwn: CUDA chunked DeltaNet prefill kernel not built yet")


def gqa_prefill(*args, **kwargs):
    raise NotImplementedError("bwn: CUDA flash prefill kernel not built yet")
