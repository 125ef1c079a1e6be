"""Adapter registry: adapter type name -> loader, plus a named-adapter store.

Parity: ModelAdapterFactory / ModelAdapterTypeRegistry
(MLXLMCommon/Adapters/ModelAdapterFactory.swift,
ModelAdapterTypeRegistry.swift): an adapter directory is resolved to a
container by the ``fine_tune_type`` (or PEFT ``peft_type``) of its
``adapter_config.json``.
"""
from __future__ import annotations

import json
import os
import threading
from typing import Callable

from .lora import LoRAContainer

_LOADERS: dict[str, Callable[[str], object]] = {
    "lora": LoRAContainer.from_directory,
    "dora": LoRAContainer.from_directory,
}


def register_adapter_type(name: str, loader: Callable[[str], object]):
    _LOADERS[name.lower()] = loader


def adapter_type(path: str) -> str:
    with open(os.path.join(path, "adapter_config.json")) as f:
        d = json.load(f)
    if "peft_type" in d or "r" in d:
        t = str(d.get("peft_type", "LORA")).lower()
        return "dora" if d.get("use_dora") else t
    return str(d.get("fine_tune_type", "lora")).lower()


def load_adapter(path: str):
    t = adapter_type(path)
    if t not in _LOADERS:
        raise ValueError(f"unknown adapter type {t!r}; registered: {sorted(_LOADERS)}")
    return _LOADERS[t](path)


class AdapterRegistry:
    """Named adapters for one model; at most one is applied at a time."""

    def __init__(self, model):
        self.model = model
        self._adapters: dict[str, object] = {}
        self.active: str | None = None
        self._lock = threading.Lock()

    def register(self, name: str, adapter_or_path):
        ad = load_adapter(adapter_or_path) if isinstance(adapter_or_path, str) else adapter_or_path
        with self._lock:
            self._adapters[name] = ad
        return ad

    def names(self):
        return sorted(self._adapters)

    def activate(self, name: str | None):
        with self._lock:
            if self.active == name:
                return
            if self.active is not None:
                self._adapters[self.active].unload(self.model)
                self.active = None
            if name is not None:
                self._adapters[name].load(self.model)
                self.active = name
