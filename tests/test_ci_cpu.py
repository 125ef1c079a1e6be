"""CI tooling: shard planning / checking / verification on synthetic test
lists and junit reports, the resource sampler against a fake NVML, and the
repository policy checks on this repository."""
import json
import os

from mlx_swift_lm_b200.ci import policy, shards
from mlx_swift_lm_b200.ci.resource_sampler import ResourceSampler

IDS = [f"tests/test_{f}_cpu.py::test_{i}" for f in "abcde" for i in range(3)] + ["tests/test_new_cpu.py::test_x"]


def test_plan_check_and_rest_shard():
    dur = {t: (10.0 if "test_a" in t else 1.0) for t in IDS}
    m = shards.plan(IDS[:-1], 3, dur)
    assert len(m["shards"]) == 3 and m["shards"][-1]["rest"]
    a = shards.assign(IDS, m)
    # the slow file sits alone; the new test (in no map) lands in the rest shard
    assert any(all("test_a" in t for t in ts) and ts for ts in a.values())
    assert "tests/test_new_cpu.py::test_x" in a[2]
    assert shards.check(IDS, m) == []
    m["shards"][1]["units"].append(m["shards"][0]["units"][0])  # a file in two shards
    assert any("in 2 shards" in p for p in shards.check(IDS, m))
    m["shards"][0]["units"].append("tests/test_gone_cpu.py")
    assert any("selects no test" in p for p in shards.check(IDS, m))


def _junit(path, ids, skip=()):
    cases = []
    for t in ids:
        f, name = t.split("::")
        cls = f[:-3].replace("/", ".")
        inner = '<skipped message="x"/>' if t in skip else ""
        cases.append(f'<testcase classname="{cls}" name="{name}" time="0.1">{inner}</testcase>')
    with open(path, "w") as fh:
        fh.write('<testsuites><testsuite name="pytest">' + "".join(cases) + "</testsuite></testsuites>")


def test_verify_counts_each_test_once(tmp_path):
    a, b = str(tmp_path / "a.xml"), str(tmp_path / "b.xml")
    _junit(a, IDS[:8])
    _junit(b, IDS[8:])
    assert shards.verify(IDS, [a, b]) == []
    _junit(b, IDS[7:], skip={IDS[9]})  # IDS[7] twice, IDS[9] skipped
    probs = shards.verify(IDS, [a, b])
    assert any(IDS[7] in p and "2 times" in p for p in probs) and any(IDS[9] in p and "0 times" in p for p in probs)


def test_checked_in_map_covers_the_cpu_tests():
    with open(shards.DEFAULT_MAP) as f:
        m = json.load(f)
    ids = [f"tests/{n}::t" for n in os.listdir(os.path.join(shards.ROOT, "tests"))
           if n.startswith("test_") and n.endswith("_cpu.py")]
    a = shards.assign(ids, m)
    assert sum(len(v) for v in a.values()) == len(ids)


class FakeNvml:
    def __init__(self):
        self.n = 0
        self.closed = False

    def sample(self):
        self.n += 1
        return [{"gpu": 0, "mem_used_mb": 100.0 * self.n, "sm_mhz": 1965, "power_w": 500.0, "reasons": 0x4},
                {"gpu": 1, "mem_used_mb": 5.0, "sm_mhz": 1800, "power_w": 100.0, "reasons": 0x1 | 0x40}]

    def close(self):
        self.closed = True


def test_resource_sampler_with_fake_nvml(tmp_path):
    import time

    fake = FakeNvml()
    with ResourceSampler(0.01, nvml=fake) as s:
        time.sleep(0.1)
    assert fake.closed and fake.n >= 3
    sm = s.summary()
    assert sm["peak_mem_used_mb"] == 100.0 * fake.n
    assert sm["reasons"] == ["gpu_idle", "hw_thermal_slowdown", "sw_power_cap"]
    out = str(tmp_path / "r.csv")
    s.write(out)
    with open(out) as f:
        head = f.readline().strip().split(",")
    assert head[0] == "t" and "sm_mhz" in head


def test_repository_policy_holds():
    assert policy.run() == []
    assert len(policy.declared_symbols()) > 30
    assert "b200_argmax_conf" in policy.defined_symbols()
