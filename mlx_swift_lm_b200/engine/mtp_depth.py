"""Adaptive MTP draft depth.

The behaviour follows the reference's depth controller
(ContinuousBatchingV2/MTP/CBv2MTPDepthController.swift:12): per draft
position, an exponentially weighted *conditional* acceptance rate (the rate
that draft i is accepted given drafts 1..i-1 were); per depth, an
exponentially weighted round cost with clamped innovations; the depth chosen
maximises expected emitted tokens per unit of round time, switches only on a
clear gain (hysteresis), and neighbouring depths are probed now and then with
an interval that doubles while the choice is stable.

Expected tokens of a round at depth k (one target token always, plus the
accepted prefix of the drafts):

    E(k) = 1 + sum_{i=1..k} prod_{j=1..i} a_j

Unmeasured depths borrow the nearest measured acceptance (positions past the
last measured one reuse it) and a cost extrapolated linearly from the
measured depths.
"""
from __future__ import annotations

from dataclasses import dataclass, field

ACCEPT_ALPHA = 0.1
ACCEPT_MIN_SAMPLES = 10
COST_ALPHA = 0.3
COST_CLAMP = 0.25
HYSTERESIS = 0.05
PROBE_BASE = 8
PROBE_MAX = 256


@dataclass
class _Ewma:
    value: float = 0.0
    n: int = 0

    def add(self, x: float, alpha: float, clamp: float | None = None):
        if self.n == 0:
            self.value = x
        else:
            d = x - self.value
            if clamp is not None:
                lim = clamp * self.value
                d = max(-lim, min(lim, d))
            self.value += alpha * d
        self.n += 1


@dataclass
class DepthController:
    k_max: int
    k_min: int = 1
    depth: int = 0
    accept: list = field(default_factory=list)  # [k_max + 1] conditional acceptance per position (1-based)
    cost: list = field(default_factory=list)  # [k_max + 1] round cost per depth
    rounds: int = 0
    probe_interval: int = PROBE_BASE
    next_probe: int = PROBE_BASE
    probing: bool = False

    def __post_init__(self):
        self.accept = [_Ewma() for _ in range(self.k_max + 1)]
        self.cost = [_Ewma() for _ in range(self.k_max + 1)]
        self.depth = self.depth or self.k_max

    # ------------------------------------------------------------------ model
    def rate(self, i: int) -> float:
        """Conditional acceptance of draft position i (1-based)."""
        for j in range(i, 0, -1):
            if self.accept[j].n >= ACCEPT_MIN_SAMPLES:
                return self.accept[j].value
        return 1.0

    def expected_tokens(self, k: int) -> float:
        e, p = 1.0, 1.0
        for i in range(1, k + 1):
            p *= self.rate(i)
            e += p
        return e

    def round_cost(self, k: int) -> float | None:
        if self.cost[k].n:
            return self.cost[k].value
        known = [(d, c.value) for d, c in enumerate(self.cost) if c.n and d >= self.k_min]
        if not known:
            return None
        if len(known) == 1:
            d0, c0 = known[0]
            return c0 * (1 + k) / (1 + d0)  # one target pass + k draft passes
        (d0, c0), (d1, c1) = known[0], known[-1]
        slope = (c1 - c0) / (d1 - d0)
        return max(c0 + slope * (k - d0), 1e-9)

    def score(self, k: int) -> float | None:
        c = self.round_cost(k)
        return None if c is None else self.expected_tokens(k) / c

    # ------------------------------------------------------------------ control
    def choose(self) -> int:
        """Depth of the next round."""
        self.rounds += 1
        self.probing = False
        if self.rounds >= self.next_probe:
            # probe a neighbour of the current depth
            cands = [d for d in (self.depth - 1, self.depth + 1) if self.k_min <= d <= self.k_max]
            if cands:
                self.probing = True
                self.next_probe = self.rounds + self.probe_interval
                self.probe_interval = min(PROBE_MAX, self.probe_interval * 2)
                return min(cands, key=lambda d: self.cost[d].n)
        return self.depth

    def observe(self, k: int, accepted: list[int], seconds: float):
        """A round of depth `k` finished in `seconds`; `accepted[r]` is how many
        drafts row r kept."""
        for a in accepted:
            for i in range(1, k + 1):
                if a < i - 1:
                    break
                self.accept[i].add(1.0 if a >= i else 0.0, ACCEPT_ALPHA)
        if seconds > 0:
            self.cost[k].add(seconds, COST_ALPHA, COST_CLAMP)
        self._update()

    def _update(self):
        scores = {d: self.score(d) for d in range(self.k_min, self.k_max + 1)}
        scores = {d: s for d, s in scores.items() if s is not None}
        if not scores:
            return
        best = max(scores, key=lambda d: scores[d])
        cur = scores.get(self.depth)
        if best != self.depth and (cur is None or scores[best] > cur * (1 + HYSTERESIS)):
            self.depth = best
            self.probe_interval = PROBE_BASE  # the choice moved: probe again soon
            self.next_probe = self.rounds + PROBE_BASE
