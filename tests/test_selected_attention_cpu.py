"""Selected-KV decode attention (sparse / indexer-selected attention over
the paged cache) on CPU: the re-statement equals dense attention when every
position is selected, ignores unused and out-of-range slots, and equals
dense attention over the gathered subset."""
import torch

from mlx_swift_lm_b200 import ops
from mlx_swift_lm_b200.ops import reference as ref


def _setup(B=3, H=8, KVH=2, D=64, lens=(37, 5, 70), seed=0):
    g = torch.Generator().manual_seed(seed)
    maxp = max((n + 15) // 16 for n in lens)
    P = B * maxp + 2
    kc = torch.randn(P, KVH, 16, D, generator=g)
    vc = torch.randn(P, KVH, 16, D, generator=g)
    perm = torch.randperm(P, generator=g)
    pt = torch.zeros(B, maxp, dtype=torch.int32)
    for b in range(B):
        pt[b] = perm[b * maxp:(b + 1) * maxp]
    q = torch.randn(B, H, D, generator=g)
    return q, kc, vc, pt, torch.tensor(lens, dtype=torch.int32)


def test_all_selected_equals_dense():
    q, kc, vc, pt, sl = _setup()
    S = int(sl.max())
    sel = torch.full((3, S), -1, dtype=torch.int32)
    for b, n in enumerate(sl.tolist()):
        sel[b, :n] = torch.randperm(n)  # any order
    got = ops.paged_selected_decode(q, kc, vc, pt, sl, sel, 0.125)
    want = ref.paged_decode_ref(q, kc, vc, pt, sl, 0.125)
    assert torch.allclose(got, want, atol=1e-5)


def test_subset_and_ignored_slots():
    q, kc, vc, pt, sl = _setup(seed=1)
    sel = torch.tensor([[3, -1, 30, 200, 7], [0, 4, -1, -1, -1], [69, 1, 2, 50, -5]], dtype=torch.int32)
    got = ops.paged_selected_decode(q, kc, vc, pt, sl, sel, 0.125)
    for b in range(3):
        pos = [t for t in sel[b].tolist() if 0 <= t < int(sl[b])]
        k = ref.gather_pages(kc, pt[b].tolist(), int(sl[b]))[pos].repeat_interleave(4, 1)
        v = ref.gather_pages(vc, pt[b].tolist(), int(sl[b]))[pos].repeat_interleave(4, 1)
        p = torch.softmax(torch.einsum("hd,nhd->hn", q[b], k) * 0.125, -1)
        assert torch.allclose(got[b], torch.einsum("hn,nhd->hd", p, v), atol=1e-5)
