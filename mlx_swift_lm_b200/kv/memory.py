"""HBM budget policies and memory measurement.

Parity: MLXLMCommon/WiredMemoryPolicies.swift:31-180 (sum / max / fixed /
budget policies computing a limit from a baseline plus the active tickets'
sizes, with admission against a cap) and WiredMemoryUtils.swift (weights +
KV + workspace measurement). On Apple GPUs the limit is the "wired" working
set of unified memory; on a B200 it is a budget of the GPU's 180 GB of HBM
that the KV pool and per-request tickets are admitted against. The recommended
working set defaults to total HBM minus a headroom for CUDA graphs, cuBLAS /
NCCL workspaces and fragmentation.
"""
from __future__ import annotations

import contextlib
import threading
from dataclasses import dataclass

import torch

DEFAULT_HEADROOM = 4 << 30


def recommended_working_set(device=None, headroom: int = DEFAULT_HEADROOM) -> int | None:
    if not torch.cuda.is_available():
        return None
    free, total = torch.cuda.mem_get_info(device)
    return max(0, total - headroom)


def _clamp(value: int, cap: int | None, device=None) -> int:
    if cap is not None:
        return min(value, max(0, cap))
    ws = recommended_working_set(device)
    return min(value, ws) if ws is not None else value


@dataclass(frozen=True)
class SumPolicy:
    """baseline + sum(active), clamped to `cap` (or the working set)."""
    cap: int | None = None

    def limit(self, baseline: int, active: list[int]) -> int:
        return _clamp(baseline + sum(active), self.cap)

    def can_admit(self, baseline: int, active: list[int], new: int) -> bool:
        p = baseline + sum(active) + max(0, new)
        return _clamp(p, self.cap) == p


@dataclass(frozen=True)
class MaxPolicy:
    """max(baseline, largest active ticket)."""

    def limit(self, baseline: int, active: list[int]) -> int:
        return max(baseline, max(active, default=0))

    def can_admit(self, baseline: int, active: list[int], new: int) -> bool:
        return True


@dataclass(frozen=True)
class FixedPolicy:
    bytes: int

    def limit(self, baseline: int, active: list[int]) -> int:
        return self.bytes

    def can_admit(self, baseline: int, active: list[int], new: int) -> bool:
        return baseline + sum(active) + max(0, new) <= self.bytes


@dataclass(frozen=True)
class BudgetPolicy:
    """baseline + base_bytes + sum(active), clamped; admission against the cap."""
    base_bytes: int
    cap: int | None = None

    def limit(self, baseline: int, active: list[int]) -> int:
        return _clamp(baseline + max(0, self.base_bytes) + sum(active), self.cap)

    def can_admit(self, baseline: int, active: list[int], new: int) -> bool:
        p = baseline + max(0, self.base_bytes) + sum(active) + max(0, new)
        return _clamp(p, self.cap) == p


class MemoryBudget:
    """Tickets of bytes admitted against a policy over a fixed baseline
    (normally the model's weight bytes)."""

    def __init__(self, policy, baseline: int = 0):
        self.policy = policy
        self.baseline = baseline
        self._active: dict[int, int] = {}
        self._next = 0
        self._lock = threading.Lock()

    @property
    def limit(self) -> int:
        return self.policy.limit(self.baseline, list(self._active.values()))

    def try_acquire(self, size: int) -> int | None:
        with self._lock:
            if not self.policy.can_admit(self.baseline, list(self._active.values()), size):
                return None
            self._next += 1
            self._active[self._next] = size
            return self._next

    def release(self, ticket: int):
        with self._lock:
            self._active.pop(ticket, None)

    @contextlib.contextmanager
    def ticket(self, size: int):
        t = self.try_acquire(size)
        if t is None:
            raise MemoryError(f"a {size}-byte ticket exceeds the memory budget (limit {self.limit})")
        try:
            yield t
        finally:
            self.release(t)


@dataclass
class MemoryMeasurement:
    weight_bytes: int
    kv_bytes: int
    workspace_bytes: int
    peak_active_bytes: int
    token_count: int = 0

    @property
    def total_bytes(self) -> int:
        return max(0, self.weight_bytes) + max(0, self.kv_bytes) + max(0, self.workspace_bytes)


def model_bytes(model) -> int:
    """Bytes of a model's weights (packed quantised weights count their codes,
    scales and biases)."""
    from ..ops.qlinear import QuantizedWeight

    seen, n = set(), 0
    for _, t in model.named_tensors():
        if t is None or id(t) in seen:
            continue
        seen.add(id(t))
        n += t.nbytes() if isinstance(t, QuantizedWeight) else t.numel() * t.element_size()
    return n


def measure(model, kv=None, device=None) -> MemoryMeasurement:
    """Weights, KV pool and the rest of the allocator's peak as workspace."""
    w = model_bytes(model)
    k = 0
    if kv is not None:
        k = kv.slab_bytes
        if kv.rec is not None:
            k += kv.rec.conv.numel() * kv.rec.conv.element_size() + kv.rec.ssm.numel() * 4
    peak = torch.cuda.max_memory_allocated(device) if torch.cuda.is_available() else 0
    return MemoryMeasurement(w, k, max(0, peak - w - k), peak)


def kv_budget_bytes(device=None, fraction: float = 0.9, headroom: int = DEFAULT_HEADROOM) -> int:
    """KV pool size from the HBM still free after the weights are loaded:
    `fraction` of (free - headroom)."""
    free, _ = torch.cuda.mem_get_info(device)
    return max(0, int((free - headroom) * fraction))
