"""The allocation-free paged decode entry point (b200_paged_decode_noalloc),
called through its exported C symbol, against the scratch-taking entry point
b200_paged_decode on the same inputs.

Both entry points run the same two kernels with the same arguments; only
where the split-KV partials live differs (a caller buffer versus the
library's built-in array), so the outputs must be bit-identical."""
import ctypes as C

import pytest
import torch

from mlx_swift_lm_b200.ops import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
TOO_LARGE = -2
SCRATCH_FLOATS = 2 * 1024 * 1024


def _noalloc_fn():
    so = C.CDLL(_lib.LIB_PATH)
    fn = so.b200_paged_decode_noalloc
    vp, i32 = C.c_void_p, C.c_int
    fn.restype = i32
    fn.argtypes = [vp, vp, vp, i32, vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32, i32, i32, C.c_float, C.c_float,
                   C.c_int64, vp]
    return fn


def _case(seed, B, H, KVH, D, lens, num_pages=160, fp8=False, sinks=False, dev=DEV):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, H, D, generator=g).to(dev, torch.bfloat16)
    kc = torch.randn(num_pages, KVH, 16, D, generator=g)
    vc = torch.randn(num_pages, KVH, 16, D, generator=g)
    ks = vs = None
    if fp8:  # stored = x / scale, one scale per KV head
        ks = (torch.rand(KVH, generator=g) * 0.5 + 0.25).to(dev)
        vs = (torch.rand(KVH, generator=g) * 0.5 + 0.25).to(dev)
        kc = (kc / ks.cpu()[None, :, None, None]).to(torch.float8_e4m3fn)
        vc = (vc / vs.cpu()[None, :, None, None]).to(torch.float8_e4m3fn)
    else:
        kc, vc = kc.to(torch.bfloat16), vc.to(torch.bfloat16)
    kc, vc = kc.to(dev), vc.to(dev)
    ld = max((n + 15) // 16 for n in lens)
    pt = torch.zeros(B, ld, dtype=torch.int32)
    perm = torch.randperm(num_pages, generator=g)
    assert sum((n + 15) // 16 for n in lens) <= num_pages
    used = 0
    for b, n in enumerate(lens):
        k = (n + 15) // 16
        pt[b, :k] = perm[used:used + k]
        used += k
    sl = torch.tensor(lens, dtype=torch.int32)
    sk = torch.randn(H, generator=g).to(dev) if sinks else None
    return dict(q=q, kc=kc, vc=vc, pt=pt.to(dev), sl=sl.to(dev), ks=ks, vs=vs, sinks=sk)


def _ptr(t):
    return None if t is None else t.data_ptr()


def _run(fn_noalloc, c, max_parts, window=0, softcap=0.0, dev=DEV):
    q, kc, vc, pt, sl = c["q"], c["kc"], c["vc"], c["pt"], c["sl"]
    B, H, D = q.shape
    KVH = kc.shape[1]
    fp8 = 1 if kc.dtype == torch.float8_e4m3fn else 0
    st = _lib.stream_ptr(dev)
    scale = D ** -0.5
    args_in = (q.data_ptr(), kc.data_ptr(), vc.data_ptr(), fp8, _ptr(c["ks"]), _ptr(c["vs"]), pt.data_ptr(),
               pt.shape[1], sl.data_ptr(), _ptr(c["sinks"]))
    out_ref = torch.empty_like(q)
    acc = torch.empty(B * H * max_parts * D, dtype=torch.float32, device=dev)
    ml = torch.empty(B * H * max_parts * 2, dtype=torch.float32, device=dev)
    rc = _lib.lib().b200_paged_decode(*args_in, out_ref.data_ptr(), acc.data_ptr(), ml.data_ptr(), B, H, KVH, D,
                                      max_parts, window, scale, softcap, kc.shape[0], st)
    assert rc == 0
    out = torch.full_like(q, float("nan"))
    rc = fn_noalloc(*args_in, out.data_ptr(), B, H, KVH, D, max_parts, window, scale, softcap, kc.shape[0], st)
    assert rc == 0
    torch.cuda.synchronize(dev)
    return out, out_ref


def test_noalloc_decode_matches_scratch_entry_two_calls():
    fn = _noalloc_fn()
    torch.cuda.set_device(DEV)
    # first call: GQA group 4, contexts spanning 1..3 partitions
    c = _case(11, B=5, H=8, KVH=2, D=128, lens=[1, 255, 256, 600, 700])
    out, ref = _run(fn, c, max_parts=3)
    assert torch.equal(out, ref)
    # second call in a row, new shapes and a sliding window: stale scratch must not leak in
    c = _case(12, B=3, H=4, KVH=4, D=64, lens=[513, 30, 1000], num_pages=128)
    out, ref = _run(fn, c, max_parts=4, window=300)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("D,fp8,sinks,softcap", [(256, False, False, 0.0), (128, True, False, 0.0),
                                                 (64, False, True, 0.0), (128, True, True, 30.0)])
def test_noalloc_decode_variants(D, fp8, sinks, softcap):
    """fp8-e4m3 pages with per-head scales, head dim 256, attention sinks and
    a logit softcap take their own kernel instantiations in both entries."""
    fn = _noalloc_fn()
    torch.cuda.set_device(DEV)
    c = _case(20 + D, B=4, H=16, KVH=4, D=D, lens=[17, 300, 513, 64], fp8=fp8, sinks=sinks)
    out, ref = _run(fn, c, max_parts=3, softcap=softcap)
    assert torch.isfinite(out).all()
    assert torch.equal(out, ref)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
def test_noalloc_decode_second_device():
    """The first call on another device looks up that device's own array and
    sets that device's kernel attributes."""
    fn = _noalloc_fn()
    dev = torch.device("cuda", 1)
    with torch.cuda.device(dev):
        c = _case(31, B=4, H=32, KVH=8, D=128, lens=[100, 900, 1500, 2], dev=dev)
        out, ref = _run(fn, c, max_parts=6, dev=dev)
        assert torch.equal(out, ref)


def test_noalloc_decode_rejects_oversized_scratch():
    fn = _noalloc_fn()
    B, H, D, KVH = 64, 32, 128, 8
    max_parts = 8  # 64*32*8*128 floats alone fill the array; the (max, sum) pairs do not fit
    assert B * H * max_parts * D + B * H * max_parts * 2 > SCRATCH_FLOATS
    q = torch.zeros(B, H, D, dtype=torch.bfloat16, device=DEV)
    out = torch.zeros_like(q)
    rc = fn(q.data_ptr(), None, None, 0, None, None, None, 1, None, None, out.data_ptr(), B, H, KVH, D, max_parts, 0,
            1.0, 0.0, 1, _lib.stream_ptr(DEV))
    assert rc == TOO_LARGE
