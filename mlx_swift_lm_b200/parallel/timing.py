"""Device timing across ranks: every multi-GPU number is the device time of
the slowest rank (CUDA events on the launching stream, then a MAX all-reduce),
never a host wall clock of one rank."""
from __future__ import annotations

import torch


class DeviceTimer:
    """CUDA-event timer on the current stream: ``start()`` / ``stop()`` around
    the work, ``ms()`` after a synchronize."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.e0 = torch.cuda.Event(enable_timing=True)
        self.e1 = torch.cuda.Event(enable_timing=True)

    def start(self):
        self.e0.record(torch.cuda.current_stream(self.device))
        return self

    def stop(self):
        self.e1.record(torch.cuda.current_stream(self.device))
        return self

    def ms(self) -> float:
        self.e1.synchronize()
        return self.e0.elapsed_time(self.e1)


def max_over_ranks(values, device, group=None) -> list[float]:
    """Elementwise maximum of per-rank float values (all ranks call it, in
    the same order); the identity without an initialised process group."""
    import torch.distributed as dist

    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t.tolist()
