"""Dequantising tcgen05 GEMM (affine 4/8-bit weights, MLX groups) vs the fp32
oracle over the same dequantised weights."""
import pytest
import torch

from mlx_swift_lm_b200 import ops
from mlx_swift_lm_b200.ops import reference as ref
from mlx_swift_lm_b200.ops.qlinear import QuantizedWeight

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("M", [1, 16, 33, 64, 130, 300])
def test_gemm_q(bits, gs, M):
    torch.manual_seed(M + bits + gs)
    N, K = 384, 1024
    w = torch.randn(N, K) * 0.05
    q = QuantizedWeight.quantize(w, bits, gs).to(DEV)
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    y = ops.gemm(x, q)
    r = ref.gemm_ref(x.cpu(), q.dequantize().to(torch.bfloat16).cpu())
    assert _rel(y.cpu(), r) < 1e-2
    yf = ops.gemm(x, q, epi="f32")
    assert _rel(yf.cpu(), ref.gemm_ref(x.cpu(), q.dequantize().to(torch.bfloat16).cpu(), "f32")) < 1e-3


@pytest.mark.parametrize("epi", ["swiglu", "geglu", "swiglu_oai"])
def test_gemm_q_glu_bias_and_add(epi):
    torch.manual_seed(7)
    K, F, M = 512, 256, 48
    g = QuantizedWeight.quantize(torch.randn(F, K) * 0.05, 4, 64)
    u = QuantizedWeight.quantize(torch.randn(F, K) * 0.05, 4, 64)
    gu = QuantizedWeight.interleave_gate_up(g, u).to(DEV)
    b = torch.randn(2 * F, device=DEV, dtype=torch.bfloat16) * 0.1
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    y = ops.gemm(x, gu, epi=epi, bias=b)
    r = ref.gemm_ref(x.cpu(), gu.dequantize().to(torch.bfloat16).cpu(), epi, bias=b.cpu())
    assert _rel(y.cpu(), r) < 1.5e-2
    res = torch.randn(M, 2 * F, device=DEV, dtype=torch.bfloat16)
    ya = ops.gemm(x, gu, epi="add", residual=res)
    ra = ref.gemm_ref(x.cpu(), gu.dequantize().to(torch.bfloat16).cpu(), "add", res.cpu())
    assert _rel(ya.cpu(), ra) < 1e-2


def test_gemm_q_large_shape_and_batch_invariance():
    torch.manual_seed(9)
    N, K = 4096, 4096
    q = QuantizedWeight.quantize(torch.randn(N, K) * 0.02, 4, 64).to(DEV)
    x = torch.randn(64, K, device=DEV, dtype=torch.bfloat16)
    full = ops.gemm(x, q)
    one = ops.gemm(x[5:6].contiguous(), q)
    assert torch.equal(full[5:6], one)
    r = ref.gemm_ref(x[:8].cpu(), q.dequantize().to(torch.bfloat16).cpu())
    assert _rel(full[:8].cpu(), r) < 1e-2


@pytest.mark.parametrize("M", [1, 16, 64, 300])
def test_gemm_mxfp4(M):
    torch.manual_seed(M)
    N, K = 384, 1024
    q = QuantizedWeight.quantize_mxfp4(torch.randn(N, K) * 0.05).to(DEV)
    assert q.kernel_bits == -4
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    y = ops.gemm(x, q)
    r = ref.gemm_ref(x.cpu(), q.dequantize().to(torch.bfloat16).cpu())
    assert _rel(y.cpu(), r) < 1e-2


def test_mxfp4_dequant_exact():
    """One-hot activations read every weight back: the e2m1 table and the
    power-of-two scales are exact."""
    torch.manual_seed(3)
    N, K = 256, 128
    w = torch.randn(N, K) * torch.logspace(-3, 1, K)  # spread the block exponents
    q = QuantizedWeight.quantize_mxfp4(w).to(DEV)
    codes = q.codes_int()
    assert set(codes.unique().tolist()) == set(range(16)) - {8}  # -0 is never produced
    eye = torch.eye(K, device=DEV, dtype=torch.bfloat16)
    y = ops.gemm(eye, q, epi="f32")  # [K, N] = W^T
    assert torch.equal(y.t().cpu(), q.dequantize().cpu())


@pytest.mark.parametrize("M", [1, 64, 300])
def test_gemm_nvfp4(M):
    torch.manual_seed(M + 5)
    N, K = 384, 1024
    q = QuantizedWeight.quantize_nvfp4(torch.randn(N, K) * 0.05).to(DEV)
    assert q.kernel_bits == -4 and q.gs == 16
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    y = ops.gemm(x, q)
    r = ref.gemm_ref(x.cpu(), q.dequantize().to(torch.bfloat16).cpu())
    assert _rel(y.cpu(), r) < 1e-2
    eye = torch.eye(K, device=DEV, dtype=torch.bfloat16)[:128]
    yi = ops.gemm(eye, q, epi="f32")  # rows 0..127 of W^T exactly
    assert torch.equal(yi.t().cpu(), q.dequantize()[:, :128].cpu())
