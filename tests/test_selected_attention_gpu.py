"""Selected-KV decode attention kernel against the fp32 re-statement
(subset selections with unused / out-of-range slots, GQA groups of 4 and 8,
head dims 64 and 128) and against the paged decode kernel when every
position is selected."""
import pytest
import torch

from mlx_swift_lm_b200 import ops
from mlx_swift_lm_b200.ops import _lib
from mlx_swift_lm_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("H,KVH,D,S", [(32, 8, 128, 64), (16, 2, 128, 300), (8, 2, 64, 17)])
def test_selected_decode_matches_reference(H, KVH, D, S):
    torch.manual_seed(H + D + S)
    B, lens = 5, [700, 33, 1, 260, 2048]
    maxp = (max(lens) + 15) // 16
    P = B * maxp + 3
    kc = torch.randn(P, KVH, 16, D).to(torch.bfloat16)
    vc = torch.randn(P, KVH, 16, D).to(torch.bfloat16)
    pt = torch.randperm(P)[:B * maxp].reshape(B, maxp).to(torch.int32)
    sl = torch.tensor(lens, dtype=torch.int32)
    sel = torch.stack([torch.randint(-50, n + 20, (S,)) for n in lens]).to(torch.int32)
    q = torch.randn(B, H, D).to(torch.bfloat16)
    want = ref.paged_selected_decode_ref(q.float(), kc.float(), vc.float(), pt, sl, sel, D ** -0.5)
    got = ops.paged_selected_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), pt.to(DEV), sl.to(DEV), sel.to(DEV),
                                    D ** -0.5)
    torch.cuda.synchronize()
    assert _rel(got.cpu(), want) < 1e-2


def test_full_selection_equals_paged_decode():
    torch.manual_seed(0)
    B, H, KVH, D, L = 4, 32, 8, 128, 300
    maxp = (L + 15) // 16
    kc = torch.randn(B * maxp, KVH, 16, D, device=DEV).to(torch.bfloat16)
    vc = torch.randn(B * maxp, KVH, 16, D, device=DEV).to(torch.bfloat16)
    pt = torch.arange(B * maxp, dtype=torch.int32, device=DEV).reshape(B, maxp)
    sl = torch.full((B,), L, dtype=torch.int32, device=DEV)
    q = torch.randn(B, H, D, device=DEV).to(torch.bfloat16)
    sel = torch.arange(L, dtype=torch.int32, device=DEV)[None].expand(B, L).contiguous()
    a = ops.paged_selected_decode(q, kc, vc, pt, sl, sel, D ** -0.5)
    b = ops.paged_decode(q, kc, vc, pt, sl, D ** -0.5)
    torch.cuda.synchronize()
    assert _rel(a, b) < 1e-2
