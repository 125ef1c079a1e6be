"""LoRA / DoRA adapters for :class:`DecoderLM`.

Parity: LoRALinear / DoRALinear (MLXLMCommon/Adapters/LoRA/LoRA+Layers.swift:26,
DoRA+Layers.swift:64), LoRAContainer load / fuse / unload
(LoRAContainer.swift:133-230) and the PEFT loader (PEFTAdapter.swift).

The model keeps its projections fused (q|k|v stacked, gate/up interleaved in
64-row blocks, tensor-parallel shards), so an adapter for ``q_proj`` or
``gate_proj`` is a low-rank update of a row range (or of interleaved rows) of a
fused weight. Serving applies an adapter by adding the update into a copy of
the fused weights: decode then runs at exactly the base model's speed, and the
untouched originals are kept so :meth:`LoRAContainer.unload` restores them.
:meth:`LoRAContainer.fuse` makes the update permanent and drops the originals.

Math (per adapted projection W [out, in], A [r, in], B [out, r], scale s):
    LoRA   W' = W + s * B @ A
    DoRA   V  = W + s * B @ A;  W' = (m / ||V||_row) * V    (m [out])
Tensor parallelism: row-sharded projections (q, k, v, gate, up) take the
rank's rows of B; column-sharded ones (o, down) take the rank's columns of A;
DoRA row norms of column-sharded projections are summed across ranks.

File formats:
    MLX   adapter_config.json {fine_tune_type, num_layers, lora_parameters:
          {rank, scale, dropout, keys}} + adapters.safetensors with
          ``model.layers.{i}.<key>.lora_a`` [in, r], ``.lora_b`` [r, out],
          DoRA ``.m`` [out]
    PEFT  adapter_config.json {r, lora_alpha, target_modules, use_dora} +
          adapter_model.safetensors with ``...layers.{i}.<key>.lora_A.weight``
          [r, in], ``.lora_B.weight`` [out, r], ``.lora_magnitude_vector``;
          scale = lora_alpha / r
"""
from __future__ import annotations

import json
import math
import os
import re
from dataclasses import dataclass, field

import torch

from ..loader.safetensors import load_safetensors, save_safetensors
from ..ops.reference import deinterleave_gate_up, interleave_gate_up

# adapter key -> (fused weight, part)
TARGETS = {
    "self_attn.q_proj": ("wqkv", "q"),
    "self_attn.k_proj": ("wqkv", "k"),
    "self_attn.v_proj": ("wqkv", "v"),
    "self_attn.o_proj": ("wo", None),
    "mlp.gate_proj": ("wgu", "gate"),
    "mlp.up_proj": ("wgu", "up"),
    "mlp.down_proj": ("wd", None),
}
DEFAULT_KEYS = ("self_attn.q_proj", "self_attn.v_proj")
_SHORT = {k.split(".")[-1]: k for k in TARGETS}


@dataclass
class LoRAParameters:
    rank: int = 8
    scale: float = 20.0
    dropout: float = 0.0
    keys: list[str] | None = None

    def __post_init__(self):
        if not (0.0 <= self.dropout < 1.0):
            raise ValueError("LoRA dropout must be in [0, 1)")
        if self.rank <= 0:
            raise ValueError("LoRA rank must be positive")


@dataclass
class LoRAConfiguration:
    num_layers: int = 16
    fine_tune_type: str = "lora"  # lora | dora
    lora_parameters: LoRAParameters = field(default_factory=LoRAParameters)

    def to_dict(self) -> dict:
        p = self.lora_parameters
        d = {"rank": p.rank, "scale": p.scale, "dropout": p.dropout}
        if p.keys is not None:
            d["keys"] = list(p.keys)
        return {"fine_tune_type": self.fine_tune_type, "num_layers": self.num_layers, "lora_parameters": d}

    @classmethod
    def from_dict(cls, d: dict) -> "LoRAConfiguration":
        lp = d.get("lora_parameters", {})
        ft = d.get("fine_tune_type", "lora")
        if ft not in ("lora", "dora"):
            raise ValueError(f"unsupported fine_tune_type {ft!r} (lora or dora)")
        return cls(num_layers=int(d.get("num_layers", 16)), fine_tune_type=ft,
                   lora_parameters=LoRAParameters(rank=int(lp.get("rank", 8)), scale=float(lp.get("scale", 20.0)),
                                                  dropout=float(lp.get("dropout", 0.0)), keys=lp.get("keys")))


def _norm_key(k: str) -> str:
    if k in TARGETS:
        return k
    if k in _SHORT:
        return _SHORT[k]
    raise ValueError(f"unsupported LoRA target {k!r}; supported: {sorted(TARGETS)}")


class LoRAContainer:
    """Adapter weights plus configuration. ``tensors`` maps
    ``(layer, key) -> {"a": [r, in], "b": [out, r], "m": [out] or None}``
    (fp32, full unsharded shapes)."""

    def __init__(self, configuration: LoRAConfiguration, tensors: dict):
        self.configuration = configuration
        self.tensors = tensors
        self._originals: dict | None = None
        self._model = None

    # ------------------------------------------------------------------ construction
    @classmethod
    def init_for(cls, model, configuration: LoRAConfiguration, seed: int = 0) -> "LoRAContainer":
        """Fresh adapter for `model`: A ~ U(-1/sqrt(in), 1/sqrt(in)), B = 0 (so
        the adapted model starts equal to the base), DoRA m = ||W||_row."""
        cfg = model.cfg
        g = torch.Generator().manual_seed(seed)
        p = configuration.lora_parameters
        keys = [_norm_key(k) for k in (p.keys or DEFAULT_KEYS)]
        nl = min(configuration.num_layers, cfg.num_layers)
        dims = _dims(cfg)
        tens = {}
        for li in range(cfg.num_layers - nl, cfg.num_layers):
            for k in keys:
                out, inp = dims[k]
                bound = 1.0 / math.sqrt(inp)
                a = (torch.rand(p.rank, inp, generator=g) * 2 - 1) * bound
                b = torch.zeros(out, p.rank)
                m = None
                if configuration.fine_tune_type == "dora":
                    m = _full_row_norm(model, li, k)
                tens[(li, k)] = {"a": a, "b": b, "m": m}
        return cls(configuration, tens)

    @classmethod
    def from_directory(cls, path: str) -> "LoRAContainer":
        """Load an MLX-format or PEFT-format adapter directory."""
        with open(os.path.join(path, "adapter_config.json")) as f:
            d = json.load(f)
        if "r" in d or "peft_type" in d or "lora_alpha" in d:
            return cls._from_peft(path, d)
        conf = LoRAConfiguration.from_dict(d)
        raw, _ = load_safetensors(os.path.join(path, "adapters.safetensors"))
        tens: dict = {}
        pat = re.compile(r"(?:.*\.)?layers\.(\d+)\.(.+)\.(lora_a|lora_b|m)$")
        for name, t in raw.items():
            mt = pat.match(name)
            if not mt:
                continue
            li, key, kind = int(mt.group(1)), _norm_key(mt.group(2)), mt.group(3)
            ent = tens.setdefault((li, key), {"a": None, "b": None, "m": None})
            t = t.float()
            if kind == "lora_a":
                ent["a"] = t.t().contiguous()  # [in, r] -> [r, in]
            elif kind == "lora_b":
                ent["b"] = t.t().contiguous()  # [r, out] -> [out, r]
            else:
                ent["m"] = t
        _check_complete(tens, conf)
        return cls(conf, tens)

    @classmethod
    def _from_peft(cls, path: str, d: dict) -> "LoRAContainer":
        r = int(d["r"])
        alpha = float(d["lora_alpha"])
        drop = float(d.get("lora_dropout", 0.0) or 0.0)
        targets = d.get("target_modules") or []
        if isinstance(targets, str):
            targets = [targets]
        raw, _ = load_safetensors(os.path.join(path, "adapter_model.safetensors"))
        tens: dict = {}
        pat = re.compile(r".*layers\.(\d+)\.(.+?)\.(lora_A\.weight|lora_B\.weight|lora_magnitude_vector)"
                         r"(?:\.weight)?$")
        for name, t in raw.items():
            mt = pat.match(name)
            if not mt:
                continue
            li, key, kind = int(mt.group(1)), _norm_key(mt.group(2)), mt.group(3)
            ent = tens.setdefault((li, key), {"a": None, "b": None, "m": None})
            t = t.float()
            if kind.startswith("lora_A"):
                ent["a"] = t
            elif kind.startswith("lora_B"):
                ent["b"] = t
            else:
                ent["m"] = t
        layers = sorted({li for li, _ in tens})
        keys = sorted({k for _, k in tens}) or [_norm_key(k) for k in targets]
        conf = LoRAConfiguration(num_layers=len(layers), fine_tune_type="dora" if d.get("use_dora") else "lora",
                                 lora_parameters=LoRAParameters(rank=r, scale=alpha / r, dropout=drop, keys=keys))
        _check_complete(tens, conf)
        return cls(conf, tens)

    def save(self, path: str):
        """Write MLX format (adapter_config.json + adapters.safetensors)."""
        os.makedirs(path, exist_ok=True)
        with open(os.path.join(path, "adapter_config.json"), "w") as f:
            json.dump(self.configuration.to_dict(), f, indent=2)
        out = {}
        for (li, k), ent in sorted(self.tensors.items()):
            base = f"model.layers.{li}.{k}"
            out[base + ".lora_a"] = ent["a"].t().contiguous().float()
            out[base + ".lora_b"] = ent["b"].t().contiguous().float()
            if ent.get("m") is not None:
                out[base + ".m"] = ent["m"].float()
        save_safetensors(os.path.join(path, "adapters.safetensors"), out)

    # ------------------------------------------------------------------ apply
    def load(self, model):
        """Apply to `model` (updates a copy of each touched fused weight; the
        originals are kept for :meth:`unload`)."""
        if self._originals is not None:
            raise RuntimeError("adapter already loaded")
        self._originals = {}
        self._apply(model, keep=True)
        self._model = model
        model.lora = self
        return model

    def fuse(self, model):
        """Apply permanently (no originals kept)."""
        if self._originals is not None and self._model is model:
            self._originals = None
            model.lora = None
            return model
        self._apply(model, keep=False)
        return model

    def unload(self, model=None):
        """Restore the weights saved by :meth:`load`."""
        model = model or self._model
        if self._originals is None or model is None:
            return model
        for (li, name), t in self._originals.items():
            setattr(model.layers[li], name, t)
        self._originals = None
        self._model = None
        model.lora = None
        return model

    def _apply(self, model, keep: bool):
        s = self.configuration.lora_parameters.scale
        dora = self.configuration.fine_tune_type == "dora"
        by_layer: dict[int, dict] = {}
        for (li, k), ent in self.tensors.items():
            by_layer.setdefault(li, {})[k] = ent
        for li, ents in sorted(by_layer.items()):
            if li >= len(model.layers):
                raise ValueError(f"adapter layer {li} beyond the model's {len(model.layers)} layers")
            L = model.layers[li]
            if L.moe and any(TARGETS[k][0] in ("wgu", "wd") for k in ents):
                raise ValueError("LoRA on MoE expert projections is not supported")
            touched = {TARGETS[k][0] for k in ents}
            new = {}
            for name in touched:
                w = getattr(L, name)
                if keep:
                    self._originals[(li, name)] = w
                new[name] = w.float().clone()
            if "wqkv" in new:
                _update_qkv(model, new["wqkv"], ents, s, dora)
            if "wgu" in new:
                _update_gu(model, new["wgu"], ents, s, dora)
            if "wo" in new:
                _update_cols(model, new["wo"], ents["self_attn.o_proj"], s, dora)
            if "wd" in new:
                _update_cols(model, new["wd"], ents["mlp.down_proj"], s, dora)
            for name, t in new.items():
                setattr(L, name, t.to(model.dtype).contiguous())


# ---------------------------------------------------------------------- helpers
def _dims(cfg):
    H, KVH, D, hid, F = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.hidden_size, cfg.intermediate_size
    return {"self_attn.q_proj": (H * D, hid), "self_attn.k_proj": (KVH * D, hid), "self_attn.v_proj": (KVH * D, hid),
            "self_attn.o_proj": (hid, H * D), "mlp.gate_proj": (F, hid), "mlp.up_proj": (F, hid),
            "mlp.down_proj": (hid, F)}


def _check_complete(tens, conf):
    for key, ent in tens.items():
        if ent["a"] is None or ent["b"] is None:
            raise ValueError(f"adapter entry {key} lacks lora_a or lora_b")
        if conf.fine_tune_type == "dora" and ent["m"] is None:
            raise ValueError(f"DoRA adapter entry {key} lacks its magnitude vector")


def _row_shard(model, t, kv=False):
    """Rows of a full [out, ...] tensor owned by this rank (heads split)."""
    tp, cfg = model.tp, model.cfg
    if tp.world == 1:
        return t
    if kv and cfg.num_kv_heads < tp.world:
        D = cfg.head_dim
        h = (tp.rank * cfg.num_kv_heads) // tp.world
        return t[h * D:(h + 1) * D]
    n = t.shape[0] // tp.world
    return t[tp.rank * n:(tp.rank + 1) * n]


def _col_shard(model, t):
    tp = model.tp
    if tp.world == 1:
        return t
    n = t.shape[-1] // tp.world
    return t[..., tp.rank * n:(tp.rank + 1) * n]


def _dora(v: torch.Tensor, m: torch.Tensor, sq_sum=None) -> torch.Tensor:
    sq = v.pow(2).sum(1)
    if sq_sum is not None:
        sq = sq_sum(sq)
    return v * (m / sq.sqrt().clamp_min(1e-12))[:, None]


def _update_rows(model, w, ent, s, dora, kv=False):
    b = _row_shard(model, ent["b"], kv).to(w.device)
    v = w + s * (b @ ent["a"].to(w.device))
    if dora:
        v = _dora(v, _row_shard(model, ent["m"], kv).to(w.device))
    return v


def _update_qkv(model, w, ents, s, dora):
    qn, kn = model.H * model.D, model.KVH * model.D
    parts = {"self_attn.q_proj": (0, qn, False), "self_attn.k_proj": (qn, qn + kn, True),
             "self_attn.v_proj": (qn + kn, qn + 2 * kn, True)}
    for k, (lo, hi, kv) in parts.items():
        if k in ents:
            w[lo:hi] = _update_rows(model, w[lo:hi], ents[k], s, dora, kv)


def _update_gu(model, w, ents, s, dora):
    g, u = deinterleave_gate_up(w)
    if "mlp.gate_proj" in ents:
        g = _update_rows(model, g, ents["mlp.gate_proj"], s, dora)
    if "mlp.up_proj" in ents:
        u = _update_rows(model, u, ents["mlp.up_proj"], s, dora)
    w.copy_(interleave_gate_up(g, u))


def _update_cols(model, w, ent, s, dora):
    a = _col_shard(model, ent["a"]).to(w.device)
    v = w + s * (ent["b"].to(w.device) @ a)
    if dora:
        red = None
        if model.tp.world > 1:
            import torch.distributed as dist

            def red(sq):
                sq = sq.contiguous()
                dist.all_reduce(sq, group=model.tp.group)
                return sq
        v = _dora(v, ent["m"].to(w.device), red)
    w.copy_(v)


def _full_row_norm(model, li, key):
    """||W||_row of the unsharded base projection (world 1) used to initialise DoRA."""
    if model.tp.world != 1:
        raise ValueError("initialising a DoRA adapter needs the unsharded model (TP world 1)")
    L = model.layers[li]
    qn, kn = model.H * model.D, model.KVH * model.D
    if key == "self_attn.q_proj":
        w = L.wqkv[:qn]
    elif key == "self_attn.k_proj":
        w = L.wqkv[qn:qn + kn]
    elif key == "self_attn.v_proj":
        w = L.wqkv[qn + kn:]
    elif key == "self_attn.o_proj":
        w = L.wo
    elif key in ("mlp.gate_proj", "mlp.up_proj"):
        g, u = deinterleave_gate_up(L.wgu)
        w = g if key == "mlp.gate_proj" else u
    else:
        w = L.wd
    return w.float().pow(2).sum(1).sqrt().cpu()
