"""LoRA / DoRA adapter training: data loading, batching, masked next-token
loss, an Adam training loop with periodic validation and checkpointing.

Parity: LoRATrain (MLXLLM/LoraTrain.swift:134-433: Parameters :141, loss,
LoRABatchIterator, evaluate, train with progress callbacks, save) and
loadLoRAData (MLXLLM/Lora+Data.swift:21: ``.jsonl`` lines with a "text" field
or ``.txt`` lines). Resuming continues from ``completed_iterations`` with the
adapter weights the container already holds.

Loss: cross entropy of position j's logits against token j+1, counted only
where token j+1 is a real token of the sample (padding never scores).
"""
from __future__ import annotations

import json
import os
import random
import time
from dataclasses import dataclass
from typing import Callable, Iterator

import torch
import torch.nn.functional as Fn

from ..adapters.lora import LoRAContainer
from .forward import TrainableLoRA, train_forward


@dataclass
class TrainParameters:
    batch_size: int = 4
    iterations: int = 1000
    steps_per_report: int = 10
    steps_per_eval: int = 100
    validation_batches: int = 10  # 0 = the whole validation set
    save_every: int = 100
    adapter_path: str | None = None
    completed_iterations: int = 0
    learning_rate: float = 1e-5
    seed: int = 0

    def __post_init__(self):
        if self.completed_iterations < 0:
            raise ValueError("completed_iterations must be >= 0")


@dataclass
class Progress:
    kind: str  # "train" | "validation" | "save"
    iteration: int
    loss: float | None = None
    iterations_per_second: float | None = None
    tokens_per_second: float | None = None
    path: str | None = None


def load_lora_data(directory: str, name: str) -> list[str]:
    """``<directory>/<name>.jsonl`` (lines of {"text": ...}) or ``<name>.txt``."""
    for ext in ("jsonl", "txt"):
        p = os.path.join(directory, f"{name}.{ext}")
        if os.path.exists(p):
            return load_lora_file(p)
    raise FileNotFoundError(f"no {name}.jsonl or {name}.txt under {directory}")


def load_lora_file(path: str) -> list[str]:
    with open(path, encoding="utf-8") as f:
        lines = f.read().split("\n")
    if path.endswith(".jsonl"):
        out = []
        for ln in lines:
            if ln.startswith("{"):
                t = json.loads(ln).get("text")
                if t is not None:
                    out.append(t)
        return out
    return [ln for ln in lines if ln]


def iterate_batches(dataset: list[str], tokenizer, batch_size: int, train: bool,
                    seed: int = 0) -> Iterator[tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
    """(inputs [B, S-1], targets [B, S-1], lengths [B]) batches; endless and
    reshuffled each epoch when `train`, one pass otherwise."""
    rng = random.Random(seed)
    idx = list(range(len(dataset)))
    if train:
        rng.shuffle(idx)
    i = 0
    while True:
        if i >= len(idx):
            if not train:
                return
            rng.shuffle(idx)
            i = 0
        chunk = idx[i:i + batch_size]
        i += batch_size
        toks = [tokenizer.encode(dataset[j]) for j in chunk]
        lengths = [len(t) for t in toks]
        S = max(lengths)
        if S < 2:
            raise ValueError("LoRA batch has no sample of 2 or more tokens: each token is predicted from the "
                             "ones before it")
        arr = torch.zeros(len(toks), S, dtype=torch.long)
        for r, t in enumerate(toks):
            arr[r, :len(t)] = torch.tensor(t, dtype=torch.long)
        yield arr[:, :-1], arr[:, 1:], torch.tensor(lengths)


def loss_fn(model, lora: TrainableLoRA | None, inputs, targets, lengths, training=True):
    """(mean loss over scored tokens, number of scored tokens)."""
    logits = train_forward(model, inputs, lora, training)
    S = inputs.shape[1]
    mask = torch.arange(S)[None, :] < (lengths[:, None] - 1)
    mask = mask.to(logits.device)
    ce = Fn.cross_entropy(logits.reshape(-1, logits.shape[-1]), targets.to(logits.device).reshape(-1),
                          reduction="none").reshape(mask.shape)
    n = mask.sum()
    return (ce * mask).sum() / n.clamp_min(1), int(n)


@torch.no_grad()
def evaluate(model, lora, dataset, tokenizer, batch_size, batches=0):
    tot, ntok = 0.0, 0
    for k, (x, y, ln) in enumerate(iterate_batches(dataset, tokenizer, batch_size, train=False)):
        if batches and k >= batches:
            break
        l, n = loss_fn(model, lora, x, y, ln, training=False)
        tot += float(l) * n
        ntok += n
    return tot / max(ntok, 1)


def train(model, adapter: LoRAContainer, tokenizer, train_set: list[str], valid_set: list[str],
          params: TrainParameters, progress: Callable[[Progress], bool] | None = None,
          optimizer_factory=None) -> LoRAContainer:
    """Train `adapter` on `train_set`; returns it with the trained weights.
    `progress` receives Progress events and may return False to stop."""
    lora = TrainableLoRA(adapter, model.embed.device)
    opt = (optimizer_factory or (lambda ps: torch.optim.Adam(ps, lr=params.learning_rate)))(list(lora.parameters()))
    it = iterate_batches(train_set, tokenizer, params.batch_size, train=True, seed=params.seed)
    losses, ntoks = [], 0
    t0 = time.perf_counter()
    start = params.completed_iterations
    for step in range(start, params.iterations):
        x, y, ln = next(it)
        loss, n = loss_fn(model, lora, x, y, ln, training=True)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
        ntoks += n
        i = step + 1
        if i % params.steps_per_report == 0:
            dt = time.perf_counter() - t0
            ev = Progress("train", i, sum(losses) / len(losses), params.steps_per_report / dt, ntoks / dt)
            losses, ntoks = [], 0
            t0 = time.perf_counter()
            if progress and progress(ev) is False:
                break
        if valid_set and (i == 1 or i % params.steps_per_eval == 0):
            vl = evaluate(model, lora, valid_set, tokenizer, params.batch_size, params.validation_batches)
            if progress and progress(Progress("validation", i, vl)) is False:
                break
        if params.adapter_path and i % params.save_every == 0:
            lora.write_back()
            adapter.save(params.adapter_path)
            if progress and progress(Progress("save", i, path=params.adapter_path)) is False:
                break
    lora.write_back()
    if params.adapter_path:
        adapter.save(params.adapter_path)
    return adapter
