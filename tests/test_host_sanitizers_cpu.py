"""The native host runtime (page pool, block hasher, grammar matcher,
safetensors reader / writer) built with AddressSanitizer + UBSan, and with
ThreadSanitizer for the multi-threaded span reader, exercised in a child
process that preloads the sanitizer runtime. Any report aborts the child
(-fno-sanitize-recover), so the test fails on the first finding."""
import os
import subprocess
import sys
import textwrap

import pytest

from mlx_swift_lm_b200 import _build

EXERCISE = textwrap.dedent(r'''
    import os, sys, json, struct, random
    sys.path.insert(0, sys.argv[1])
    import _b200host as h
    assert h.__file__.startswith(sys.argv[1]), h.__file__
    # page pool: alloc / share / free / poison / generations
    p = h.PagePool(64)
    a = p.alloc(10); b = p.alloc(20)
    p.incref(a[:5]); p.decref(a); p.decref(a[:5])
    assert p.can_alloc(44) and not p.can_alloc(45)
    gen = p.generation(b[0]); p.decref(b); c = p.alloc(30)
    assert p.valid(b[0], gen) in (True, False)
    p.poison(c[0]); p.decref(c)
    # block hashing
    toks = [random.randrange(1 << 20) for _ in range(1000)]
    hs = h.block_hashes(toks, 16, "salt")
    assert len(hs) == 1000 // 16 and hs == h.block_hashes(toks, 16, "salt")
    assert len(h.sha256(b"abc")) in (32, 64)
    # grammar: a small regex over a toy vocabulary
    vocab = h.GrammarVocab([b"a", b"b", b"ab", b"{", b"}", b"\"", b"x", b"1", b"2", b","], [9])
    m = h.GrammarMatcher(vocab, '\\{"x":[12]+\\}')
    for tok in [3, 5, 6, 5]:
        m.mask()
        assert m.accept_token(tok), tok
    m.rollback(2)
    for tok in [6, 5]:
        assert m.accept_token(tok)
    m.forced_prefix(16)
    # safetensors: write then read spans on several threads
    import ctypes
    d = sys.argv[2]
    path = os.path.join(d, "t.safetensors")
    payload = (ctypes.c_uint8 * (1 << 17))(*([i % 251 for i in range(1 << 17)]))
    header = json.dumps({"w": {"dtype": "U8", "shape": [1 << 17], "data_offsets": [0, 1 << 17]}})
    h.st_write(path, header, [(ctypes.addressof(payload), 1 << 17)])
    hdr, base = h.st_read_header(path)
    dst = (ctypes.c_uint8 * (1 << 17))()
    spans = [(base + i * 4096, 4096, ctypes.addressof(dst) + i * 4096) for i in range(32)]
    h.st_read_spans(path, spans, 8)
    assert bytes(dst) == bytes(payload)
    print("ok")
''')


def _runtime(name):
    r = subprocess.run(["gcc", "-print-file-name=" + name], capture_output=True, text=True)
    path = r.stdout.strip()
    return path if os.path.isabs(path) and os.path.exists(path) else None


def _signatures_ok():
    import _b200host as h  # noqa: F401  (the release module imports)
    return True


@pytest.mark.parametrize("sanitizer,runtime", [("address,undefined", "libasan.so"), ("thread", "libtsan.so")])
def test_host_runtime_under_sanitizers(tmp_path, sanitizer, runtime):
    rt = _runtime(runtime)
    if rt is None:
        pytest.skip(f"{runtime} not installed")
    out = tmp_path / "san"
    try:
        _build.build_host_sanitized(str(out), sanitizer)
    except RuntimeError as e:
        pytest.skip(f"sanitized build unavailable: {str(e)[:200]}")
    env = dict(os.environ, LD_PRELOAD=rt, ASAN_OPTIONS="detect_leaks=0:abort_on_error=1",
               UBSAN_OPTIONS="halt_on_error=1:print_stacktrace=1",
               TSAN_OPTIONS="halt_on_error=1:report_signal_unsafe=0:ignore_noninstrumented_modules=1")
    r = subprocess.run([sys.executable, "-c", EXERCISE, str(out), str(tmp_path)], capture_output=True, text=True,
                       env=env, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, (r.stdout[-2000:], r.stderr[-4000:])
