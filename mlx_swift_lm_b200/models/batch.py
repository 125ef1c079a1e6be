"""Flattened forward batch consumed by the decoder.

Tokens of a step are laid out ``[decode rows (1 token each) | prefill chunks]``
- the rectangular ``[B, 1]`` decode of the reference engine
(EngineLoopV2.swift:4633-4708) followed by the packed prefill rows
(:4721-4884). Every token carries its absolute position and the cache slot
(``page * 16 + offset``) its K/V is written to.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class ForwardBatch:
    input_ids: torch.Tensor  # [T] int32
    positions: torch.Tensor  # [T] int32
    slots: torch.Tensor  # [T] int64
    num_decode: int = 0
    # decode rows
    dec_page_table: torch.Tensor | None = None  # [Bd, maxp] int32
    dec_seq_lens: torch.Tensor | None = None  # [Bd] int32 (context length incl. the new token)
    dec_max_parts: int = 1
    # prefill rows
    pf_cu_q: torch.Tensor | None = None  # [R+1] int32 (offsets relative to the prefill part)
    pf_cu_q_host: list | None = None
    pf_pos0: torch.Tensor | None = None  # [R] int32
    pf_page_table: torch.Tensor | None = None  # [R, maxp] int32
    # rows whose logits are needed (indices into the T tokens); None = all tokens
    logit_idx: torch.Tensor | None = None
    logit_idx_host: list | None = None  # the same indices on the host (microbatch splitting)
    # per-token LoRA adapter slot (-1 = none), used when adapters are active
    lora_slots: torch.Tensor | None = None
    # data-parallel rank that owns each row's KV (expert-parallel models); host list
    row_ranks: list | None = None
    # recurrent-state slot of each row (hybrid models with linear-attention layers)
    state_slots: torch.Tensor | None = None  # [rows] int32
    # engine request state of each row (host; multimodal models read Request.mm)
    row_states: list | None = None
    pf_pos0_host: list | None = None
    # per-token rotary cos|sin table [T, rot_dim] replacing the position lookup (M-RoPE prompts)
    rope_table: torch.Tensor | None = None
    # prefill rows attend to their whole chunk (mask-diffusion blocks) instead of causally
    bidirectional: bool = False
    # sliding-window ring layers (kv.paged ring storage): their own slots and page tables
    ring_slots: torch.Tensor | None = None  # [T] int64
    ring_dec_page_table: torch.Tensor | None = None  # [Bd, maxp] int32
    ring_pf_page_table: torch.Tensor | None = None  # [R, maxp] int32

    def tables(self, kv, ki: int):
        """(slots, decode page table, prefill page table) of KV layer ki."""
        if self.ring_slots is not None and kv.is_ring(ki):
            return self.ring_slots, self.ring_dec_page_table, self.ring_pf_page_table
        return self.slots, self.dec_page_table, self.pf_page_table

    @property
    def num_tokens(self) -> int:
        return int(self.input_ids.shape[0])

    @property
    def num_prefill_tokens(self) -> int:
        return self.num_tokens - self.num_decode
