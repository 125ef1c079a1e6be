"""Prism Hadamard checkpoints (``model_type: prism_hadamard_qwen35``).

Parity: MLXLMCommon/PrismHadamardCheckpoint.swift - the packed-artifact
declaration in ``config.json`` (:16-60: schema 2, base ``qwen3_5``, grouped
GDN activation layout, ``mlx-vlm-qwen3_5`` tensor names, ``hadamard.json``
metadata, text only without MTP or experts, 2-bit affine group-128 packing,
module records with block 512 / 1024 / 2048 / 4096 and exactly one embedding),
the tensor checks of ``PrismHadamardCheckpoint.init`` (:72-115: fp32 layer
normalisers, the transform manifest against the tensors, packed shapes,
signs equal to the metadata) and the module install (:117-140: linears become
Hadamard-transformed quantised linears, the embedding a quantised embedding
with the inverse transform).

Transform (``normalized-sylvester-walsh-hadamard`` over the input's last
dimension, explicit signs): a transformed linear computes
``((x * signs) H) W^T`` with H the orthonormal Sylvester Hadamard matrix of
the block size applied per block; the embedding returns ``(e H) * signs`` for
the dequantised row e (the inverse, since H is symmetric and orthonormal).

Here a linear is a :class:`~..ops.rotation.RotatedWeight` whose rotation is a
:class:`~..ops.rotation.HadamardTransform` (``b200_block_hadamard``) in
front of the dequantising GEMM; the 2-bit codes ride in 4-bit records. The
embedding table is inverse-transformed once at load into a dense table (a
lookup touches only its rows); a tied head uses the packed table with the
forward transform.
"""
from __future__ import annotations

import json
import os
import re

import torch

MODEL_TYPE = "prism_hadamard_qwen35"
BLOCKS = (512, 1024, 2048, 4096)
_PATH_PART = re.compile(r"^[A-Za-z0-9_]+$")


class PrismCheckpointError(ValueError):
    def __init__(self, detail: str):
        self.detail = detail
        super().__init__(f"Invalid Prism Hadamard checkpoint: {detail}")


def is_prism(hf: dict) -> bool:
    return hf.get("model_type") == MODEL_TYPE


def parse_config(hf: dict) -> dict:
    """Validate the artifact declaration; returns {modules, has_vision}."""
    try:
        comp, qz, text = hf["components"], hf["quantization"], hf["text_config"]
        ok = (hf["schema_version"] == 2 and hf["model_type"] == MODEL_TYPE and hf["base_model_type"] == "qwen3_5"
              and hf["gdn_activation_layout"] == "grouped" and hf["tensor_namespace"] == "mlx-vlm-qwen3_5"
              and hf["hadamard_config"] == "hadamard.json" and comp["text"] and not comp["mtp"]
              and (text.get("mtp_num_hidden_layers") or 0) == 0 and (text.get("num_experts") or 0) == 0
              and qz["bits"] == 2 and qz["group_size"] == 128 and qz["mode"] == "affine")
        modules = hf["modules"]
    except (KeyError, TypeError) as e:
        raise PrismCheckpointError("unsupported architecture/packing contract") from e
    if not ok:
        raise PrismCheckpointError("unsupported architecture/packing contract")

    def valid(r):
        parts = r.get("path", "").split(".")
        return (all(_PATH_PART.match(p) for p in parts) and r.get("block") in BLOCKS and r.get("dtype") == "float16"
                and r.get("embedding") == (r["path"] == "model.embed_tokens"))

    paths = [r.get("path") for r in modules]
    if (not modules or len(modules) > 10_000 or len(set(paths)) != len(paths) or not all(valid(r) for r in modules)
            or sum(1 for r in modules if r["embedding"]) != 1):
        raise PrismCheckpointError("invalid packed module declarations")
    return {"modules": modules, "has_vision": bool(comp.get("vision"))}


class HadamardMetadata:
    """``hadamard.json``: block size, per-width sign vectors, the forward and
    inverse weight manifests and the grouped-GDN flag."""

    def __init__(self, d: dict):
        try:
            self.block = int(d["prism.hadamard.block_size"])
            self.weight_names = list(d["prism.hadamard.weight_names"])
            self.inverse_weight_names = list(d["prism.hadamard.inverse_weight_names"])
            widths = [int(w) for w in d["prism.hadamard.sign_widths"]]
            values = [float(v) for v in d["prism.hadamard.sign_values"]]
            self.gdn_v_grouped = bool(d.get("prism.hadamard.gdn_v_grouped", False))
            kind = d.get("prism.hadamard.transform", "normalized-sylvester-walsh-hadamard")
            axis = d.get("prism.hadamard.axis", "input-last-dimension")
            mode = d.get("prism.hadamard.sign_mode", "explicit")
        except (KeyError, TypeError, ValueError) as e:
            raise PrismCheckpointError("unsafe transform metadata") from e
        if (kind != "normalized-sylvester-walsh-hadamard" or axis != "input-last-dimension" or mode != "explicit"
                or self.block not in BLOCKS or sum(widths) != len(values)
                or any(v not in (-1.0, 1.0) for v in values)):
            raise PrismCheckpointError("unsafe transform metadata")
        self._cache = {}
        self.signs, o = {}, 0
        for w in widths:
            self.signs[w] = torch.tensor(values[o:o + w], dtype=torch.float32)
            o += w

    @classmethod
    def read(cls, directory: str) -> "HadamardMetadata":
        path = os.path.realpath(os.path.join(directory, "hadamard.json"))
        if not os.path.isfile(path) or not 0 < os.path.getsize(path) <= 8 * 1024 * 1024:
            raise PrismCheckpointError("unsafe transform metadata")
        with open(path) as f:
            return cls(json.load(f))

    def transform(self, width: int):
        """The transform of inputs of `width` channels (one shared object per
        width, so the fused projections of a layer transform x once)."""
        from ..ops.rotation import HadamardTransform

        if width in self._cache:
            return self._cache[width]
        if width not in self.signs:
            raise PrismCheckpointError(f"no transform signs for width {width}")
        if width % self.block:
            raise PrismCheckpointError(f"width {width} is not a multiple of the Hadamard block {self.block}")
        self._cache[width] = HadamardTransform(self.block, self.signs[width])
        return self._cache[width]


def validate(info: dict, meta: HadamardMetadata, tensors: dict):
    """Tensor checks: fp32 normalisers, manifests against the tensors, packed
    shapes / dtypes, signs equal to the metadata."""
    pre = "language_model."
    norms = [v for k, v in tensors.items() if k.startswith(pre + "model.layers.")
             and (k.endswith(".input_layernorm.weight") or k.endswith(".post_attention_layernorm.weight"))]
    if not norms or any(v.dtype != torch.float32 for v in norms):
        raise PrismCheckpointError("schema-2 native state requires the published FP32 normalizers")
    mods = info["modules"]
    forward = {f"{pre}{r['path']}.weight" for r in mods if not r["embedding"]}
    inverse = {f"{pre}{r['path']}.weight" for r in mods if r["embedding"]}
    signs = {k for k in tensors if k.endswith(".signs")}
    if (not meta.gdn_v_grouped or set(meta.weight_names) != forward or set(meta.inverse_weight_names) != inverse
            or signs != {f"{pre}{r['path']}.signs" for r in mods}
            or any(".mtp." in k or k.startswith("mtp.") for k in tensors)):
        raise PrismCheckpointError("transform manifest disagrees with tensors")
    for r in mods:
        n = pre + r["path"]
        w, s, b, sg = (tensors.get(n + x) for x in (".weight", ".scales", ".biases", ".signs"))
        if (w is None or s is None or b is None or sg is None or w.dim() != 2 or w.dtype not in (torch.int32,
                                                                                                   torch.uint32)
                or w.shape[1] == 0 or s.dim() != 2 or s.dtype != torch.float16 or b.dtype != torch.float16
                or s.shape != b.shape or s.shape[0] != w.shape[0] or s.shape[1] * 8 != w.shape[1]
                or tuple(sg.shape) != (w.shape[1] * 16,)
                or sg.dtype not in (torch.float16, torch.float32, torch.bfloat16) or r["block"] != meta.block):
            raise PrismCheckpointError("packed tensor shape/dtype mismatch")
        t = meta.transform(w.shape[1] * 16)
        if not torch.equal(sg.float(), t.signs):
            raise PrismCheckpointError("tensor signs disagree with metadata")


def text_config(hf: dict) -> dict:
    """The Qwen 3.5 text configuration the decoder is built from."""
    t = dict(hf["text_config"])
    t.setdefault("model_type", "qwen3_5_text")
    t["quantization"] = dict(hf["quantization"])
    return t


def inverse_embedding(table: torch.Tensor, transform, chunk: int = 4096) -> torch.Tensor:
    """Rows (e H) * signs of a dequantised embedding table, in chunks."""
    out = torch.empty_like(table)
    for i in range(0, table.shape[0], chunk):
        out[i:i + chunk] = transform.inverse(table[i:i + chunk])
    return out
