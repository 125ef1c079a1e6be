"""Request, sampling and event types of the continuous-batching engine.

Field-for-field parity with the reference contracts
(ContinuousBatchingV2/CBv2Contracts.swift): ``SamplingParams`` <-
``CBv2SamplingParams`` (:37), ``Request`` <- ``CBv2Request`` (:75), ``Event`` <-
``CBv2Event`` (:999), ``RequestTiming`` <- ``CBv2RequestTiming`` (:1027),
``Usage`` <- ``CBv2Usage`` (:1107), ``CapacitySnapshot`` <-
``CBv2CapacitySnapshot`` (:1188).
"""
from __future__ import annotations

import enum
import itertools
import time
from dataclasses import dataclass, field
from typing import Any, Callable

_ids = itertools.count(1)


def next_request_id() -> int:
    return next(_ids)


@dataclass
class SamplingParams:
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0
    min_p: float = 0.0
    repetition_penalty: float = 1.0
    repetition_context_size: int = 64
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    seed: int | None = None
    logit_bias: dict[int, float] = field(default_factory=dict)
    top_logprobs: int = 0  # logprobs from RAW logits (before any transform); 0 = none
    logprobs: bool = False

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0

    @property
    def needs_processing(self) -> bool:
        return bool(self.logit_bias) or self.repetition_penalty != 1.0 or self.frequency_penalty != 0.0 or \
            self.presence_penalty != 0.0


class FinishReason(str, enum.Enum):
    STOP = "stop"  # stop token or stop string
    LENGTH = "length"
    CANCELLED = "cancelled"
    ERROR = "error"
    WATCHDOG = "watchdog"
    DEADLINE = "deadline"


@dataclass
class Request:
    prompt_tokens: list[int]
    max_tokens: int = 256
    sampling: SamplingParams = field(default_factory=SamplingParams)
    stop_tokens: set[int] = field(default_factory=set)
    stop_strings: list[str] = field(default_factory=list)
    priority: int = 0
    id: int = field(default_factory=next_request_id)
    cache_salt: str | None = None
    prefix_cache_enabled: bool = True
    token_constraint: Any = None  # grammar / tool constraint (api.guided)
    reasoning_budget: int | None = None
    lora: str | None = None  # adapter name
    ignore_eos: bool = False
    on_prefill_completed: Callable | None = None
    first_token_deadline: Any = None  # engine.leases.FirstTokenDeadline (admission control)
    mm: Any = None  # multimodal payload of a vision-language prompt (models.vlm.Qwen2VLModel.prepare)


@dataclass
class RequestTiming:
    submitted: float = 0.0
    admitted: float = 0.0
    first_token: float = 0.0
    last_token: float = 0.0
    finished: float = 0.0
    prefill_chunks: int = 0
    decode_steps: int = 0
    preemptions: int = 0
    mtp_proposed: int = 0
    mtp_accepted: int = 0
    token_times: list[float] = field(default_factory=list)

    @property
    def ttft(self) -> float:
        return self.first_token - self.submitted if self.first_token else float("nan")

    def itls(self) -> list[float]:
        t = self.token_times
        return [t[i] - t[i - 1] for i in range(1, len(t))]


@dataclass
class Usage:
    prompt_tokens: int = 0
    completion_tokens: int = 0
    cached_prompt_tokens: int = 0

    @property
    def total_tokens(self) -> int:
        return self.prompt_tokens + self.completion_tokens


@dataclass
class TokenLogprob:
    token: int
    logprob: float
    top: list[tuple[int, float]] = field(default_factory=list)


@dataclass
class Event:
    """Output event of a request stream: new tokens/text, or the terminal event."""
    request_id: int
    tokens: list[int] = field(default_factory=list)
    text: str = ""
    finished: bool = False
    finish_reason: FinishReason | None = None
    usage: Usage | None = None
    timing: RequestTiming | None = None
    logprobs: list[TokenLogprob] | None = None
    error: str | None = None
    cause: str | None = None  # typed terminal cause (engine.leases.TerminalCause) of engine-ended requests


@dataclass
class CapacitySnapshot:
    active_requests: int
    waiting_requests: int
    kv_pages_total: int
    kv_pages_used: int
    kv_pages_free: int
    kv_bytes_per_page: int
    active_tokens: int
    steps: int
    last_step_ms: float
    decode_rows: int
    healthy: bool
    ledger_bytes_capacity: int = 0  # admission ledger: bytes the requests may hold
    ledger_bytes_reserved: int = 0  # ledger charge of the live requests (soft truth)
    admission_watermark_bytes: int = 0

    @property
    def kv_bytes_in_use(self) -> int:
        return self.kv_pages_used * self.kv_bytes_per_page

    @property
    def kv_bytes_capacity(self) -> int:
        return self.kv_pages_total * self.kv_bytes_per_page


def now() -> float:
    return time.perf_counter()
