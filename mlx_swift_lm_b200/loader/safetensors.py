"""Safetensors checkpoint reading / writing on top of the native parallel reader.

Parity: MLXLMCommon/Load.swift:522-649 (``loadWeights``: shard discovery
``safetensorWeightURLs`` :426, parallel span reads ``loadModelCheckpoint``
:196-280, bf16 conversion :733) and the safetensors save used for prompt
caches (KVCache.swift:2248).
"""
from __future__ import annotations

import glob
import json
import os
import sys

import numpy as np
import torch

_LIBDIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "_lib")
if _LIBDIR not in sys.path:
    sys.path.insert(0, _LIBDIR)
import _b200host  # noqa: E402

_DT = {
    "F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
    "BOOL": torch.bool, "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2,
    "U32": torch.int32, "U16": torch.int16, "U64": torch.int64,
}
_DT_NAME = {v: k for k, v in _DT.items() if k not in ("U32", "U16", "U64")}


class SafetensorsFile:
    def __init__(self, path: str):
        self.path = path
        hdr, self.data_start = _b200host.st_read_header(path)
        self.header = json.loads(hdr)
        self.metadata = self.header.pop("__metadata__", {}) or {}

    def keys(self):
        return list(self.header.keys())

    def info(self, name):
        h = self.header[name]
        return h["dtype"], h["shape"], h["data_offsets"]

    def read(self, names=None, pin: bool = False, threads: int = 0) -> dict[str, torch.Tensor]:
        names = list(names if names is not None else self.header.keys())
        out, spans = {}, []
        for n in names:
            dt, shape, (a, b) = self.info(n)
            t = torch.empty(shape, dtype=_DT[dt], pin_memory=pin)
            if b > a:
                spans.append((self.data_start + a, b - a, t.data_ptr()))
            out[n] = t
        if spans:
            _b200host.st_read_spans(self.path, spans, threads)
        return out


def load_safetensors(path_or_dir: str, pin: bool = False) -> tuple[dict[str, torch.Tensor], dict]:
    """All tensors of a file or of every *.safetensors shard in a directory."""
    files = [path_or_dir] if os.path.isfile(path_or_dir) else sorted(
        glob.glob(os.path.join(path_or_dir, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no .safetensors files under {path_or_dir}")
    tensors, meta = {}, {}
    for f in files:
        sf = SafetensorsFile(f)
        tensors.update(sf.read(pin=pin))
        meta.update(sf.metadata)
    return tensors, meta


def save_safetensors(path: str, tensors: dict[str, torch.Tensor], metadata: dict | None = None):
    header, payload, off = {}, [], 0
    keep = []
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        keep.append(t)
        nbytes = t.numel() * t.element_size()
        header[name] = {"dtype": _DT_NAME[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + nbytes]}
        payload.append((t.data_ptr(), nbytes))
        off += nbytes
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    _b200host.st_write(path, json.dumps(header, separators=(",", ":")), payload)


def as_uint32(t: torch.Tensor) -> np.ndarray:
    """View an (int32-typed) packed tensor as uint32."""
    return t.numpy().view(np.uint32)
