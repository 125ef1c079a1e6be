"""Incremental UTF-8-safe detokenisation and stop-string holdback.

* :class:`IncrementalDetokenizer` - emits text as tokens arrive without ever
  emitting a partial multi-byte character (the reference's DetokenizerV2,
  ContinuousBatchingV2/DetokenizerV2.swift:39): text whose decode ends in the
  replacement character is held until the character completes. A sliding
  (prefix, read) offset pair keeps each decode call O(window).
* :class:`StopHoldback` - matches stop strings across token boundaries,
  holding back the longest suffix that could still start a stop string
  (StopHoldback.swift:25).
"""
from __future__ import annotations


class IncrementalDetokenizer:
    def __init__(self, tokenizer, skip_special_tokens: bool = True):
        self.tok = tokenizer
        self.ids: list[int] = []
        self.prefix_offset = 0
        self.read_offset = 0
        self.skip = skip_special_tokens

    def _decode(self, ids):
        try:
            return self.tok.decode(ids, skip_special_tokens=self.skip)
        except TypeError:
            return self.tok.decode(ids)

    def push(self, token_ids) -> str:
        out = []
        for t in token_ids:
            self.ids.append(int(t))
            prefix = self._decode(self.ids[self.prefix_offset:self.read_offset])
            full = self._decode(self.ids[self.prefix_offset:])
            if len(full) > len(prefix) and not full.endswith("�"):
                out.append(full[len(prefix):])
                self.prefix_offset = self.read_offset
                self.read_offset = len(self.ids)
        return "".join(out)

    def flush(self) -> str:
        prefix = self._decode(self.ids[self.prefix_offset:self.read_offset])
        full = self._decode(self.ids[self.prefix_offset:])
        self.prefix_offset = self.read_offset = len(self.ids)
        return full[len(prefix):] if len(full) > len(prefix) else ""


class StopHoldback:
    def __init__(self, stop_strings):
        self.stops = [s for s in (stop_strings or []) if s]
        self.pending = ""
        self.stopped = False

    def push(self, text: str) -> tuple[str, bool]:
        """Returns (text safe to emit, stopped)."""
        if self.stopped:
            return "", True
        if not self.stops:
            return text, False
        self.pending += text
        cut = -1
        for s in self.stops:
            i = self.pending.find(s)
            if i >= 0 and (cut < 0 or i < cut):
                cut = i
        if cut >= 0:
            out = self.pending[:cut]
            self.pending = ""
            self.stopped = True
            return out, True
        hold = 0
        for s in self.stops:
            for k in range(min(len(s) - 1, len(self.pending)), 0, -1):
                if self.pending.endswith(s[:k]):
                    hold = max(hold, k)
                    break
        out = self.pending[: len(self.pending) - hold]
        self.pending = self.pending[len(self.pending) - hold:]
        return out, False

    def flush(self) -> str:
        out, self.pending = self.pending, ""
        return out
