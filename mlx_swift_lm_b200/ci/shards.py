"""Test shards for parallel CI jobs.

Parity: .github/scripts/test_shards.py of the reference (a checked-in map
assigns test units to shards; ``check`` fails when a collected test is in no
shard or in two, ``run`` runs one shard, ``verify`` fails unless every listed
test executed exactly once across the shard reports, ``plan`` rebalances the
map from measured durations, ``matrix`` prints the shard numbers; a shard
marked ``rest`` takes every test no other shard names, so a new test always
runs).

Here a unit is a test file (``tests/test_x_cpu.py``) or a test id
(``file::name``). The map is JSON: ``{"shards": [{"units": [...]}, ...,
{"rest": true}], "marker": "not gpu"}``.

    python -m mlx_swift_lm_b200.ci.shards plan --shards 4 [--durations d.json] > .github/test-shards.json
    python -m mlx_swift_lm_b200.ci.shards check
    python -m mlx_swift_lm_b200.ci.shards run 2 --report out/shard2.xml
    python -m mlx_swift_lm_b200.ci.shards verify out/*.xml
    python -m mlx_swift_lm_b200.ci.shards matrix
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import xml.etree.ElementTree as ET

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
DEFAULT_MAP = os.path.join(ROOT, ".github", "test-shards.json")


def collect(marker: str = "not gpu", tests_dir: str = "tests") -> list[str]:
    """Test ids pytest collects under `marker` (file::name[param])."""
    r = subprocess.run([sys.executable, "-m", "pytest", tests_dir, "--collect-only", "-q", "-m", marker,
                        "-p", "no:cacheprovider"], capture_output=True, text=True, cwd=ROOT)
    ids = [ln.strip() for ln in r.stdout.splitlines() if "::" in ln and not ln.startswith(" ")]
    if r.returncode not in (0, 5):
        raise RuntimeError("collection failed:\n" + r.stdout[-2000:] + r.stderr[-2000:])
    return ids


def _unit_of(test_id: str, units: list[str]) -> bool:
    return any(test_id == u or test_id.startswith(u + "::") or test_id.split("::")[0] == u for u in units)


def assign(ids: list[str], m: dict) -> dict[int, list[str]]:
    """shard index -> test ids (the rest shard takes what no other names)."""
    out = {i: [] for i in range(len(m["shards"]))}
    rest = [i for i, s in enumerate(m["shards"]) if s.get("rest")]
    for t in ids:
        hit = [i for i, s in enumerate(m["shards"]) if not s.get("rest") and _unit_of(t, s.get("units", []))]
        if not hit and rest:
            hit = rest[:1]
        for i in hit:
            out[i].append(t)
    return out


def check(ids: list[str], m: dict) -> list[str]:
    """Problems: tests in no shard or in several, units that select nothing."""
    probs = []
    seen: dict[str, int] = {}
    for i, ts in assign(ids, m).items():
        for t in ts:
            seen[t] = seen.get(t, 0) + 1
    for t in ids:
        n = seen.get(t, 0)
        if n != 1:
            probs.append(f"{t}: in {n} shards")
    for i, s in enumerate(m["shards"]):
        for u in s.get("units", []):
            if not any(_unit_of(t, [u]) for t in ids):
                probs.append(f"shard {i}: unit {u} selects no test")
    return probs


def plan(ids: list[str], shards: int, durations: dict[str, float] | None = None, marker: str = "not gpu") -> dict:
    """Balance test files over `shards` - 1 shards by duration (longest
    first onto the lightest shard); the last shard is the rest shard."""
    files: dict[str, float] = {}
    for t in ids:
        f = t.split("::")[0]
        files[f] = files.get(f, 0.0) + ((durations or {}).get(t, 1.0))
    n = max(1, shards - 1)
    load = [0.0] * n
    units: list[list[str]] = [[] for _ in range(n)]
    for f, d in sorted(files.items(), key=lambda kv: (-kv[1], kv[0])):
        i = min(range(n), key=lambda j: (load[j], j))
        units[i].append(f)
        load[i] += d
    m = {"marker": marker, "shards": [{"units": sorted(u)} for u in units]}
    if shards > 1:
        m["shards"].append({"rest": True, "units": []})
    return m


def executed(reports: list[str]) -> dict[str, int]:
    """Test id -> executions (passed, failed or errored; skips excluded) from junit reports."""
    cnt: dict[str, int] = {}
    for p in reports:
        for tc in ET.parse(p).getroot().iter("testcase"):
            if tc.find("skipped") is not None:
                continue
            cls, name = tc.get("classname", ""), tc.get("name", "")
            f = cls.replace(".", "/") + ".py"
            tid = f"{f}::{name}"
            cnt[tid] = cnt.get(tid, 0) + 1
    return cnt


def verify(ids: list[str], reports: list[str]) -> list[str]:
    cnt = executed(reports)
    return [f"{t}: executed {cnt.get(t, 0)} times" for t in ids if cnt.get(t, 0) != 1]


def _load(path):
    with open(path) as f:
        return json.load(f)


def main(argv=None):
    ap = argparse.ArgumentParser(prog="shards")
    ap.add_argument("--map", default=DEFAULT_MAP)
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("plan")
    p.add_argument("--shards", type=int, default=4)
    p.add_argument("--durations")
    p.add_argument("--marker", default="not gpu")
    sub.add_parser("check")
    p = sub.add_parser("run")
    p.add_argument("index", type=int)
    p.add_argument("--report")
    p = sub.add_parser("verify")
    p.add_argument("reports", nargs="+")
    sub.add_parser("matrix")
    a = ap.parse_args(argv)
    if a.cmd == "plan":
        print(json.dumps(plan(collect(a.marker), a.shards, _load(a.durations) if a.durations else None, a.marker),
                         indent=1))
        return 0
    m = _load(a.map)
    if a.cmd == "matrix":
        print(json.dumps(list(range(len(m["shards"])))))
        return 0
    ids = collect(m.get("marker", "not gpu"))
    if a.cmd == "check":
        probs = check(ids, m)
        print("\n".join(probs) or f"{len(ids)} tests, each in exactly one of {len(m['shards'])} shards")
        return 1 if probs else 0
    if a.cmd == "run":
        mine = assign(ids, m)[a.index]
        if not mine:
            print("empty shard")
            return 0
        cmd = [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-m", m.get("marker", "not gpu")]
        if a.report:
            cmd += ["--junitxml", a.report]
        return subprocess.call(cmd + mine, cwd=ROOT)
    probs = verify(ids, a.reports)
    print("\n".join(probs) or f"all {len(ids)} tests executed exactly once")
    return 1 if probs else 0


if __name__ == "__main__":
    sys.exit(main())
