"""Communicator guard: turn a stuck or failed collective into an engine error
instead of a hang.

The fused collective kernels never spin without a limit: a peer flag that does
not arrive within the wait limit records ``kErrPeerWait`` in the unit's device
status word and the kernel returns. NCCL collectives fail with an exception
once the process group's timeout passes (a rank that died, a peer that left).
:class:`CommGuard` joins those signals to the engine (the reference's
watchdog wedge handling, ContinuousBatchingV2/EngineLoopV2.swift:7122-7188,
and the B200 plan of aborting the communicator):

* ``check()`` reads the device status words (it synchronises the device, so
  the engine calls it every ``check_every`` steps, 0 = only on errors);
* ``on_step_error(exc)`` classifies a step exception: collective failures
  (``DistBackendError``, timeouts, NCCL errors) abort the communicator;
* ``abort(reason)`` marks the engine unhealthy, ends every live stream with
  finish reason ERROR and cause ``comm_abort``, and aborts the process group
  (``ncclCommAbort`` through torch for NCCL groups; an injected ``abort_fn``
  for tests and other backends), so every other rank's next collective errors
  too. After an abort the engine takes no more work; a supervisor restarts
  the ranks.
"""
from __future__ import annotations

import threading

from ..engine.scheduler import Status
from ..engine.types import Event, FinishReason

K_ERR_PEER_WAIT = 4
K_ERR_GEMM_WAIT = 1
COLLECTIVE_ERRORS = ("DistBackendError", "DistNetworkError", "DistError", "TimeoutError")
# message fragments of a failed collective: NCCL errors, a gloo transport
# whose peer left (reset / closed pipe) and process-group timeouts
_COLLECTIVE_TEXT = ("nccl", "gloo/transport", "timed out", "connection closed", "connection reset", "broken pipe")


def _default_abort(group):
    import torch.distributed as dist

    if not dist.is_initialized():
        return
    backend = dist.get_backend(group)
    if backend == "nccl":
        from torch.distributed.distributed_c10d import _abort_process_group

        _abort_process_group(group)


class CommGuard:
    def __init__(self, engine, group=None, abort_fn=None, check_every: int = 0, read_status=None):
        self.engine = engine
        self.group = group
        self.abort_fn = abort_fn or _default_abort
        self.check_every = check_every
        if read_status is None:
            from ..ops import _lib

            read_status = _lib.read_status
        self.read_status = read_status
        self.aborted: str | None = None
        self._lock = threading.Lock()
        engine.comm_guard = self
        prev = engine.on_step_wedge

        def wedge():
            if prev is not None:
                prev()
            self.abort("engine step exceeded its timeout")

        engine.on_step_wedge = wedge

    def check(self) -> bool:
        """False (and the communicator aborted) when a collective kernel gave up
        waiting for a peer."""
        st = self.read_status(clear=False)
        bad = {k: v for k, v in st.items() if v & (K_ERR_PEER_WAIT | K_ERR_GEMM_WAIT)}
        if bad:
            self.abort(f"collective wait expired: {bad}")
            return False
        return True

    def after_step(self, steps: int):
        if self.check_every and steps % self.check_every == 0:
            self.check()

    def on_step_error(self, exc: BaseException) -> bool:
        """True if `exc` is a collective failure (the communicator is then aborted)."""
        name = type(exc).__name__
        text = str(exc).lower()
        if name in COLLECTIVE_ERRORS or any(k in text for k in _COLLECTIVE_TEXT):
            self.abort(f"collective failed: {name}: {str(exc)[:200]}")
            return True
        return False

    def abort(self, reason: str):
        with self._lock:
            if self.aborted is not None:
                return
            self.aborted = reason
        eng = self.engine
        eng.healthy = False
        for st in list(eng.states.values()):
            if st.status == Status.FINISHED:
                continue
            try:
                st.status = Status.FINISHED
                st.stream.put(Event(st.req.id, finished=True, finish_reason=FinishReason.ERROR, usage=st.usage,
                                    timing=st.timing, error=reason, cause="comm_abort"))
            except Exception:
                pass
        try:
            self.abort_fn(self.group)
        except Exception:
            pass
