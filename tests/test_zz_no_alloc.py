"""The allocation-free paged decode entry point (b200_paged_decode_noalloc),
called through its exported C symbol, against the scratch-taking entry point
b200_paged_decode on the same inputs."""
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


def _case(seed, B, H, KVH, D, lens, num_pages=160):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, H, D, generator=g).to(DEV, torch.bfloat16)
    kc = torch.randn(num_pages, KVH, 16, D, generator=g).to(DEV, torch.bfloat16)
    vc = torch.randn(num_pages, KVH, 16, D, generator=g).to(DEV, torch.bfloat16)
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
    return q, kc, vc, pt.to(DEV), sl.to(DEV)


def _run(fn_noalloc, q, kc, vc, pt, sl, max_parts, window=0):
    B, H, D = q.shape
    KVH = kc.shape[1]
    st = _lib.stream_ptr(DEV)
    scale = D ** -0.5
    out_ref = torch.empty_like(q)
    acc = torch.empty(B * H * max_parts * D, dtype=torch.float32, device=DEV)
    ml = torch.empty(B * H * max_parts * 2, dtype=torch.float32, device=DEV)
    rc = _lib.lib().b200_paged_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), 0, None, None, pt.data_ptr(),
                                      pt.shape[1], sl.data_ptr(), None, out_ref.data_ptr(), acc.data_ptr(),
                                      ml.data_ptr(), B, H, KVH, D, max_parts, window, scale, 0.0, kc.shape[0], st)
    assert rc == 0
    out = torch.full_like(q, float("nan"))
    rc = fn_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), 0, None, None, pt.data_ptr(), pt.shape[1],
                    sl.data_ptr(), None, out.data_ptr(), B, H, KVH, D, max_parts, window, scale, 0.0, kc.shape[0], st)
    assert rc == 0
    torch.cuda.synchronize(DEV)
    return out, out_ref


def test_noalloc_decode_matches_scratch_entry_two_calls():
    fn = _noalloc_fn()
    torch.cuda.set_device(DEV)
    # first call: GQA group 4, contexts spanning 1..3 partitions
    q, kc, vc, pt, sl = _case(11, B=5, H=8, KVH=2, D=128, lens=[1, 255, 256, 600, 700])
    out, ref = _run(fn, q, kc, vc, pt, sl, max_parts=3)
    torch.testing.assert_close(out, ref, atol=1e-2, rtol=1e-2)
    # second call in a row, new shapes and a sliding window: stale scratch must not leak in
    q, kc, vc, pt, sl = _case(12, B=3, H=4, KVH=4, D=64, lens=[513, 30, 1000], num_pages=128)
    out, ref = _run(fn, q, kc, vc, pt, sl, max_parts=4, window=300)
    torch.testing.assert_close(out, ref, atol=1e-2, rtol=1e-2)


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
