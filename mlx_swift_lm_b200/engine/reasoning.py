"""Reasoning (thinking) budget: a per-request cap on the tokens generated
inside a model's thought markers.

Behaviour (ContinuousBatchingV2/ReasoningBudgetV2.swift:6-150):
* the row is inside a thought after the opener (or from the start when the
  prompt template already opened it); the markers themselves spend nothing;
* once ``max_tokens`` thought tokens are generated, the next token is forced
  to the closer, whatever its logit;
* inside a thought, and after it closed, the opener is banned (one thought
  per reply);
* the state advances only on confirmed tokens, so a request's budget is the
  same whatever its batch-mates do; a token stream that breaks the rules
  (a second opener, a thought token past the limit) records a failure that
  ends the request with an error.
The output-token limit (``max_tokens`` of the request) still applies.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class ReasoningBudget:
    max_tokens: int
    open_id: int
    close_id: int
    starts_inside: bool = False

    def __post_init__(self):
        if not (0 < self.max_tokens <= 2 ** 31 - 1) or self.open_id < 0 or self.close_id < 0 \
                or self.open_id == self.close_id:
            raise ValueError("reasoning budget: need 1 <= max_tokens < 2^31 and distinct, non-negative marker ids")


class ReasoningBudgetState:
    def __init__(self, budget: ReasoningBudget, history=()):
        self.budget = budget
        self.inside = budget.starts_inside
        self.closed = False
        self.consumed = 0
        self.failure: str | None = None
        for t in history:
            self.confirm(t)

    def confirm(self, tok: int):
        if self.failure is not None:
            return
        b = self.budget
        if tok == b.open_id:
            if self.inside or self.closed:
                self.failure = "reasoning budget: repeated thought opener"
            else:
                self.inside = True
        elif tok == b.close_id:
            self.inside = False
            self.closed = True
        elif self.inside:
            if self.consumed >= b.max_tokens:
                self.failure = "reasoning budget: token beyond thought limit"
                return
            self.consumed += 1

    def forced(self) -> int | None:
        """The token the next step must produce, if any."""
        if self.inside and self.consumed >= self.budget.max_tokens:
            return self.budget.close_id
        return None

    def banned(self) -> int | None:
        return self.budget.open_id if (self.inside or self.closed) else None

    def allowed_mask(self, vocab: int):
        """numpy bool [vocab] of allowed tokens, or None when every token is."""
        b = self.budget
        if b.open_id >= vocab or b.close_id >= vocab:
            self.failure = "reasoning budget: marker outside model vocabulary"
            return None
        f = self.forced()
        if f is not None:
            m = np.zeros(vocab, dtype=bool)
            m[f] = True
            return m
        ban = self.banned()
        if ban is None:
            return None
        m = np.ones(vocab, dtype=bool)
        m[ban] = False
        return m


def resolve_budget(value, markers) -> ReasoningBudget | None:
    """A request's ``reasoning_budget``: a :class:`ReasoningBudget`, or an int
    with the engine's ``reasoning_markers`` (open_id, close_id, starts_inside)."""
    if value is None:
        return None
    if isinstance(value, ReasoningBudget):
        return value
    if markers is None:
        raise ValueError("reasoning_budget needs the model's thought-marker token ids (EngineConfig.reasoning_markers)")
    o, c, inside = (tuple(markers) + (False,))[:3]
    return ReasoningBudget(int(value), int(o), int(c), bool(inside))
