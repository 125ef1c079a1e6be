"""The bounds-checked kernel build (libb200kernels_checked.so, loaded with
B200LM_CHECKED=1): a decode row whose length runs past its page-table row is
reported in the attention unit's status word (kErrBounds) and the kernel
finishes. The table is a view into a larger buffer, so the entries the
release build would read past the row are still valid page ids of the next
row: neither build touches memory outside its allocations."""
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

CHILD = textwrap.dedent(r'''
    import torch
    from mlx_swift_lm_b200 import ops
    from mlx_swift_lm_b200.ops import _lib
    assert _lib.LIB_PATH.endswith("libb200kernels_checked.so"), _lib.LIB_PATH
    dev = torch.device("cuda", 0)
    P, KVH, D, H = 64, 2, 128, 8
    kc = torch.randn(P, KVH, 16, D, device=dev).to(torch.bfloat16)
    vc = torch.randn(P, KVH, 16, D, device=dev).to(torch.bfloat16)
    buf = torch.arange(0, 3 * 4, dtype=torch.int32, device=dev).remainder(P).view(3, 4)
    pt = buf[:2]  # rows of 4 entries; the third row keeps an overrun of row 1 inside the buffer
    sl = torch.tensor([64, 100], dtype=torch.int32, device=dev)  # row 1 needs 7 pages > 4
    q = torch.randn(2, H, D, device=dev, dtype=torch.bfloat16)
    _lib.read_status(clear=True)
    ops.paged_decode(q, kc, vc, pt, sl, D ** -0.5, max_parts=1)
    torch.cuda.synchronize()
    st = _lib.read_status()
    bad = {k: v for k, v in st.items() if v}
    assert any(k.startswith("attn_decode") and v & 8 for k, v in bad.items()), st
    print("ok", bad)
''')


def test_checked_build_reports_table_overrun():
    env = dict(os.environ, B200LM_CHECKED="1")
    r = subprocess.run([sys.executable, "-c", CHILD], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, (r.stdout[-2000:], r.stderr[-3000:])
