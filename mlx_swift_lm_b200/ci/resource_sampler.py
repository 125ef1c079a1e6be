"""Resource sampler for CI test and bench runs.

Parity: .github/scripts/ci-resource-sampler.py of the reference (sample the
runner's memory and load at a fixed interval while a job runs, write the
samples and a summary so a job's peak usage and slow steps can be read
afterwards).

Samples host CPU load and memory (psutil) and, per visible GPU, memory in
use, SM clock, power and the active clock-event reasons through NVML. NVML
is only read here; no GPU setting is changed.

    python -m mlx_swift_lm_b200.ci.resource_sampler --out res.csv [--interval 0.5] -- python -m pytest tests -m gpu
"""
from __future__ import annotations

import argparse
import csv
import subprocess
import sys
import threading
import time

REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
           0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake"}


class _Nvml:
    """The few NVML reads the sampler makes (pynvml); `None` without NVML."""

    def __init__(self):
        import pynvml

        self.n = pynvml
        pynvml.nvmlInit()
        self.handles = [pynvml.nvmlDeviceGetHandleByIndex(i) for i in range(pynvml.nvmlDeviceGetCount())]

    def sample(self) -> list[dict]:
        n = self.n
        out = []
        for i, h in enumerate(self.handles):
            mem = n.nvmlDeviceGetMemoryInfo(h)
            out.append({"gpu": i, "mem_used_mb": mem.used / 2 ** 20,
                        "sm_mhz": n.nvmlDeviceGetClockInfo(h, n.NVML_CLOCK_SM),
                        "power_w": n.nvmlDeviceGetPowerUsage(h) / 1000.0,
                        "reasons": n.nvmlDeviceGetCurrentClocksEventReasons(h)})
        return out

    def close(self):
        self.n.nvmlShutdown()


def _open_nvml():
    try:
        return _Nvml()
    except Exception:
        return None


class ResourceSampler:
    def __init__(self, interval: float = 0.5, nvml=None, host=True):
        self.interval = interval
        self.nvml = nvml if nvml is not None else _open_nvml()
        self.host = host
        self.rows: list[dict] = []
        self._stop = threading.Event()
        self._t = None
        self.t0 = 0.0

    def _host(self) -> dict:
        try:
            import psutil

            vm = psutil.virtual_memory()
            return {"cpu_pct": psutil.cpu_percent(None), "host_mem_used_mb": (vm.total - vm.available) / 2 ** 20}
        except Exception:
            return {}

    def sample_once(self):
        t = time.monotonic() - self.t0
        base = {"t": round(t, 3), **(self._host() if self.host else {})}
        gpus = self.nvml.sample() if self.nvml else [{}]
        for g in gpus:
            row = dict(base, **g)
            if "reasons" in row:
                row["reasons"] = "|".join(v for k, v in REASONS.items() if row["reasons"] & k)
            self.rows.append(row)

    def _loop(self):
        while not self._stop.wait(self.interval):
            self.sample_once()

    def __enter__(self):
        self.t0 = time.monotonic()
        self.sample_once()
        self._t = threading.Thread(target=self._loop, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._t.join()
        self.sample_once()
        if self.nvml:
            self.nvml.close()

    def summary(self) -> dict:
        s = {"samples": len(self.rows), "seconds": max((r["t"] for r in self.rows), default=0.0)}
        for k in ("host_mem_used_mb", "mem_used_mb", "power_w", "cpu_pct"):
            v = [r[k] for r in self.rows if k in r]
            if v:
                s["peak_" + k] = max(v)
        clk = sorted(r["sm_mhz"] for r in self.rows if "sm_mhz" in r)
        if clk:
            s["median_sm_mhz"] = clk[len(clk) // 2]
        s["reasons"] = sorted({x for r in self.rows for x in str(r.get("reasons", "")).split("|") if x})
        return s

    def write(self, path: str):
        keys = sorted({k for r in self.rows for k in r}, key=lambda k: (k != "t", k))
        with open(path, "w", newline="") as f:
            w = csv.DictWriter(f, fieldnames=keys)
            w.writeheader()
            w.writerows(self.rows)


def main(argv=None):
    ap = argparse.ArgumentParser(prog="resource_sampler")
    ap.add_argument("--out", required=True)
    ap.add_argument("--interval", type=float, default=0.5)
    ap.add_argument("cmd", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    cmd = a.cmd[1:] if a.cmd and a.cmd[0] == "--" else a.cmd
    with ResourceSampler(a.interval) as s:
        rc = subprocess.call(cmd) if cmd else 0
    s.write(a.out)
    print("resource summary:", s.summary(), file=sys.stderr)
    return rc


if __name__ == "__main__":
    sys.exit(main())
