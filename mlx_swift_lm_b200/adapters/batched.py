"""Several LoRA adapters served in one batch: each token row names an adapter
slot (or none) and every adapted projection adds its own low-rank delta.

The merged path (:meth:`.lora.LoRAContainer.load`) adds one adapter into the
weights, which serves one adapter at a time. :class:`BatchedLoRA` keeps the
base weights untouched and holds up to ``max_adapters`` adapters stacked per
projection in fixed device buffers (so captured CUDA graphs stay valid when
adapters are added or removed):

    qkv  A [S, 3R, hidden]   B^T [S, 3R, q|k|v rows]   (q, k, v parts in R-wide rank blocks)
    o    A [S, R, H*D]       B^T [S, R, hidden]
    gu   A [S, 2R, hidden]   B^T [S, 2R, 2F]           (gate / up B columns at their interleaved rows)
    d    A [S, R, F]         B^T [S, R, hidden]

Each adapter's scale (``scale``, PEFT ``alpha / r``) sits in ``scale [S]``.
The decoder adds ``scale * (x A^T) B`` after each adapted projection
(``ops.lora``): the math of the reference's LoRALinear
(Adapters/LoRA/LoRA+Layers.swift:26) with a per-row adapter choice.
DoRA adapters (a weight-norm rescale of the merged weight) and adapters on
MoE expert projections are served through the merged path only.
"""
from __future__ import annotations

import threading

import torch

from ..ops.reference import interleave_gate_up
from .lora import TARGETS, LoRAContainer

_TARGET_OF = {"self_attn.q_proj": ("qkv", 0), "self_attn.k_proj": ("qkv", 1), "self_attn.v_proj": ("qkv", 2),
              "self_attn.o_proj": ("o", 0), "mlp.gate_proj": ("gu", 0), "mlp.up_proj": ("gu", 1),
              "mlp.down_proj": ("d", 0)}
_PARTS = {"qkv": 3, "o": 1, "gu": 2, "d": 1}


class BatchedLoRA:
    def __init__(self, model, max_adapters: int = 4, max_rank: int = 16,
                 targets=("qkv", "o", "gu", "d"), layers=None):
        if model.tp.world != 1:
            raise ValueError("batched LoRA serves tensor-parallel world 1 (merge the adapter under TP)")
        self.model = model
        self.S = max_adapters
        self.R = max_rank
        self.targets = tuple(targets)
        cfg = model.cfg
        dev, dt = model.device, model.dtype
        H, KVH, D, hid, F = model.H, model.KVH, model.D, cfg.hidden_size, model.F
        dims = {"qkv": (hid, (H + 2 * KVH) * D), "o": (H * D, hid), "gu": (hid, 2 * F), "d": (F, hid)}
        self.layer_ids = range(len(model.layers)) if layers is None else layers
        self.buf: dict[tuple[int, str], tuple[torch.Tensor, torch.Tensor]] = {}
        for li in self.layer_ids:
            L = model.layers[li]
            for tg in self.targets:
                if tg in ("gu", "d") and (L.moe or L.wgu is None):
                    continue
                if tg in ("qkv", "o") and (L.linear or L.wqkv is None or L.mla_kv_a is not None):
                    continue
                K, N = dims[tg]
                r = _PARTS[tg] * max_rank
                self.buf[(li, tg)] = (torch.zeros(max_adapters, r, K, device=dev, dtype=dt),
                                      torch.zeros(max_adapters, r, N, device=dev, dtype=dt))
        self.scale = torch.zeros(max_adapters, device=dev, dtype=torch.float32)
        self.names: dict[str, int] = {}
        self._lock = threading.Lock()
        # per-forward scratch for the shrink output, keyed by (rows, rank)
        self._t: dict[tuple[int, int], torch.Tensor] = {}
        self._index = {id(L): li for li, L in enumerate(model.layers)}

    # ------------------------------------------------------------------ registry
    def add(self, name: str, adapter) -> int:
        """Write `adapter` (a LoRAContainer or a directory) into a free slot."""
        if isinstance(adapter, str):
            adapter = LoRAContainer.from_directory(adapter)
        conf = adapter.configuration
        if conf.fine_tune_type == "dora":
            raise ValueError("DoRA adapters are served merged (LoRAContainer.load), not batched")
        with self._lock:
            if name in self.names:
                raise ValueError(f"adapter {name!r} is already loaded")
            free = [s for s in range(self.S) if s not in self.names.values()]
            if not free:
                raise ValueError(f"all {self.S} adapter slots are in use")
            s = free[0]
            self._write(s, adapter)
            self.scale[s] = float(conf.lora_parameters.scale)
            self.names[name] = s
        return s

    def remove(self, name: str):
        with self._lock:
            s = self.names.pop(name)
            for A, Bt in self.buf.values():
                A[s].zero_()
                Bt[s].zero_()
            self.scale[s] = 0.0

    def slot(self, name: str | None) -> int:
        if name is None:
            return -1
        s = self.names.get(name)
        if s is None:
            raise ValueError(f"unknown adapter {name!r}; loaded: {sorted(self.names)}")
        return s

    def _write(self, s: int, adapter: LoRAContainer):
        m = self.model
        H, KVH, D = m.H, m.KVH, m.D
        qn, kn = H * D, KVH * D
        R = self.R
        for A, Bt in self.buf.values():
            A[s].zero_()
            Bt[s].zero_()
        gu_parts: dict[int, dict] = {}
        for (li, key), ent in adapter.tensors.items():
            if key not in TARGETS:
                raise ValueError(f"unsupported LoRA target {key!r}")
            tg, part = _TARGET_OF[key]
            if (li, tg) not in self.buf:
                raise ValueError(f"layer {li} has no batched-LoRA buffer for {key} (MoE, linear or MLA layer?)")
            a, b = ent["a"], ent["b"]  # [r, in], [out, r]
            r = a.shape[0]
            if r > R:
                raise ValueError(f"adapter rank {r} exceeds the batched max_rank {R}")
            A, Bt = self.buf[(li, tg)]
            A[s, part * R:part * R + r] = a.to(A.device, A.dtype)
            if tg == "qkv":
                lo = (0, qn, qn + kn)[part]
                Bt[s, part * R:part * R + r, lo:lo + b.shape[0]] = b.t().to(Bt.device, Bt.dtype)
            elif tg == "gu":
                gu_parts.setdefault(li, {})[part] = b
            else:
                Bt[s, :r] = b.t().to(Bt.device, Bt.dtype)
        for li, parts in gu_parts.items():
            A, Bt = self.buf[(li, "gu")]
            F = Bt.shape[-1] // 2
            g = torch.zeros(F, 2 * R)
            u = torch.zeros(F, 2 * R)
            if 0 in parts:
                g[:, :parts[0].shape[1]] = parts[0].float()
            if 1 in parts:
                u[:, R:R + parts[1].shape[1]] = parts[1].float()
            Bt[s] = interleave_gate_up(g, u).t().to(Bt.device, Bt.dtype)

    # ------------------------------------------------------------------ forward
    def tensors(self, L, target: str):
        li = self._index.get(id(L))
        return None if li is None else self.buf.get((li, target))

    def scratch(self, T: int, R: int, device) -> torch.Tensor:
        t = self._t.get((T, R))
        if t is None:
            t = self._t[(T, R)] = torch.empty(T, R, dtype=torch.float32, device=device)
        return t
