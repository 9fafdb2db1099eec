"""Dependency-free safetensors reading and writing.

File format: an 8-byte little-endian header length ``n``, ``n`` bytes of JSON
mapping each tensor name to ``{dtype, shape, data_offsets: [begin, end]}``
(offsets relative to the first byte after the header), then the raw bytes.
The reference reads the same format with a copying reader
(``contrib/qwen3.6-35b-a3b/st_reader.py:31-81``); this one maps the file
copy-on-write so a tensor is a zero-copy view until it is moved to the GPU,
and it can also write files (used by the weight preprocessors and tests).

FP8 tensors (``F8_E4M3``, ``F8_E5M2``) and the E8M0 scale type are returned as
raw ``uint8`` bytes: the bwn FP8 kernels take E4M3FN bytes directly, and the
decoders in :mod:`bwn.io.fp8` work from the bit layout.
"""
from __future__ import annotations

import json
import mmap
import os
import struct

import torch

DTYPES = {
    "F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8,
    "U8": torch.uint8, "BOOL": torch.bool,
    "F8_E4M3": torch.uint8, "F8_E5M2": torch.uint8, "F8_E8M0": torch.uint8,
}
_TAGS = {torch.float64: "F64", torch.float32: "F32", torch.float16: "F16", torch.bfloat16: "BF16",
         torch.int64: "I64", torch.int32: "I32", torch.int16: "I16", torch.int8: "I8",
         torch.uint8: "U8", torch.bool: "BOOL"}
if hasattr(torch, "float8_e4m3fn"):
    _TAGS[torch.float8_e4m3fn] = "F8_E4M3"
    _TAGS[torch.float8_e5m2] = "F8_E5M2"


class SafeReader:
    """Lazy reader over one ``.safetensors`` file (kept mapped until :meth:`close`)."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        head = self._f.read(8)
        if len(head) != 8:
            raise ValueError(f"{path}: truncated safetensors header")
        n = struct.unpack("<Q", head)[0]
        self.header = json.loads(self._f.read(n).decode("utf-8"))
        self.metadata = self.header.pop("__metadata__", None) or {}
        self._base = 8 + n
        size = os.fstat(self._f.fileno()).st_size
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_COPY) if size > self._base else None
        for k, m in self.header.items():
            b0, b1 = m["data_offsets"]
            if not (0 <= b0 <= b1 <= size - self._base):
                raise ValueError(f"{path}: tensor {k!r} lies outside the file")

    def keys(self) -> list[str]:
        return list(self.header)

    def __contains__(self, name: str) -> bool:
        return name in self.header

    def dtype_tag(self, name: str) -> str:
        return self.header[name]["dtype"]

    def shape(self, name: str) -> list[int]:
        return list(self.header[name]["shape"])

    def get(self, name: str) -> torch.Tensor:
        m = self.header[name]
        tag = m["dtype"]
        if tag not in DTYPES:
            raise TypeError(f"unsupported safetensors dtype {tag!r} for {name!r}")
        dt = DTYPES[tag]
        b0, b1 = m["data_offsets"]
        shape = m["shape"]
        if b1 == b0:
            return torch.empty(shape, dtype=dt)
        t = torch.frombuffer(self._mm, dtype=torch.uint8, count=b1 - b0, offset=self._base + b0)
        return t.view(dt).reshape(shape)

    def close(self):
        if self._mm is not None:
            self._mm = None  # views keep the mapping alive until they are freed
        self._f.close()


def save_file(tensors: dict[str, torch.Tensor], path: str, metadata: dict | None = None,
              dtype_tags: dict[str, str] | None = None):
    """Write ``tensors`` (moved to CPU, made contiguous) as one safetensors file.
    ``dtype_tags`` overrides the tag of a ``uint8`` tensor that holds FP8 bytes."""
    header: dict = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    blobs = []
    off = 0
    for name in sorted(tensors):
        t = tensors[name].detach().to("cpu").contiguous()
        tag = (dtype_tags or {}).get(name) or _TAGS.get(t.dtype)
        if tag is None:
            raise TypeError(f"cannot store dtype {t.dtype} ({name!r})")
        nb = t.numel() * t.element_size()
        header[name] = {"dtype": tag, "shape": list(t.shape), "data_offsets": [off, off + nb]}
        blobs.append(t)
        off += nb
    hj = json.dumps(header, separators=(",", ":")).encode("utf-8")
    hj += b" " * ((8 - len(hj) % 8) % 8)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for t in blobs:
            if t.numel():
                f.write(t.reshape(-1).view(torch.uint8).numpy().tobytes())
    os.replace(tmp, path)


def weight_map(ckpt_dir: str) -> dict[str, str]:
    """``{tensor name: file name}`` over a checkpoint directory, from
    ``model.safetensors.index.json`` when present, else by scanning every file."""
    idx = os.path.join(ckpt_dir, "model.safetensors.index.json")
    if os.path.exists(idx):
        with open(idx) as f:
            return dict(json.load(f)["weight_map"])
    wm: dict[str, str] = {}
    for fn in sorted(os.listdir(ckpt_dir)):
        if fn.endswith(".safetensors"):
            r = SafeReader(os.path.join(ckpt_dir, fn))
            for k in r.keys():
                wm[k] = fn
            r.close()
    if not wm:
        raise FileNotFoundError(f"no .safetensors files in {ckpt_dir}")
    return wm


def save_sharded(tensors: dict[str, torch.Tensor], ckpt_dir: str, max_shard_bytes: int = 4 << 30,
                 dtype_tags: dict[str, str] | None = None):
    """Write an HF-style sharded checkpoint (``model-0000i-of-0000n.safetensors``
    plus ``model.safetensors.index.json``)."""
    os.makedirs(ckpt_dir, exist_ok=True)
    shards: list[dict[str, torch.Tensor]] = [{}]
    size = 0
    for name in sorted(tensors):
        nb = tensors[name].numel() * tensors[name].element_size()
        if shards[-1] and size + nb > max_shard_bytes:
            shards.append({})
            size = 0
        shards[-1][name] = tensors[name]
        size += nb
    wm = {}
    for i, sh in enumerate(shards):
        fn = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(ckpt_dir, fn), dtype_tags={k: v for k, v in (dtype_tags or {}).items() if k in sh})
        wm.update({k: fn for k in sh})
    with open(os.path.join(ckpt_dir, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": wm}, f, indent=1)
