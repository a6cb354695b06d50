"""The tcgen05/TMA GEMM of liborda_b200.so against a float64 torch reference
of the same bf16 operands, for every operand layout the loss uses:
  kind (0,0)  C = A @ B^T   logits   (A [M,K], B [N,K])
  kind (0,1)  C = A @ B     dgrad    (A [M,K], B [K,N])
  kind (1,1)  C = A^T @ B   wgrad    (A [K,M], B [K,N])
  kind (1,0)  C = A^T @ B^T          (A [K,M], B [N,K])
Shapes cover single tiles, K/M/N tails that rely on TMA zero fill, and a
multi-wave persistent schedule; each runs with the CTA-pair tiles (256 x 256,
tcgen05 cta_group::2, the default) and with single-CTA tiles (128 x 256,
ORDA_GEMM_CTA_PAIR=0). Tolerance: fp32 accumulation of exact bf16
products, so the relative L2 error to the float64 product is <= 1e-5 for
K <= 4096 and <= 1e-4 for the long-K (32000) case.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from orda_b200.device import DeviceContext

    c = DeviceContext(0)
    yield c
    c.close()


def _operand(rows, cols, gen, pad=0):
    """bf16 [rows, cols] view with leading dimension rounded up to 8 (+pad)."""
    ld = (cols + 7) // 8 * 8 + pad
    base = torch.randn(rows, ld, generator=gen, device="cuda").to(torch.bfloat16)
    return base[:, :cols]


SHAPES = [
    (128, 256, 64),
    (256, 512, 256),
    (200, 300, 72),
    (1, 8, 8),
    (513, 1000, 1000),
    (64, 4096, 512),
    (1000, 2304, 136),
    (2048, 8192, 256),
]


@pytest.fixture(params=["pair", "single"])
def tiles(request, monkeypatch):
    monkeypatch.setenv("ORDA_GEMM_CTA_PAIR", "1" if request.param == "pair" else "0")
    return request.param


@pytest.mark.parametrize("a_kind,b_kind", [(0, 0), (0, 1), (1, 1), (1, 0)])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_layouts(ctx, tiles, a_kind, b_kind, m, n, k):
    from orda_b200.device import gemm_bf16

    gen = torch.Generator(device="cuda").manual_seed(m * 7 + n * 13 + k)
    a = _operand(m, k, gen) if a_kind == 0 else _operand(k, m, gen)
    b = _operand(n, k, gen) if b_kind == 0 else _operand(k, n, gen)
    c = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float32)
    gemm_bf16(ctx, a, a_kind, b, b_kind, c, m, n, k)
    torch.cuda.synchronize()
    ctx.check()
    A = (a if a_kind == 0 else a.t()).double()
    B = (b.t() if b_kind == 0 else b).double()
    ref = A @ B
    assert torch.isfinite(c).all()
    err = (c.double() - ref).norm() / ref.norm()
    assert err < 1e-5, f"rel L2 {err:.3e}"


def test_gemm_alpha_beta_accumulate(ctx, tiles):
    from orda_b200.device import gemm_bf16

    gen = torch.Generator(device="cuda").manual_seed(5)
    m, n, k = 384, 640, 192
    a = _operand(m, k, gen)
    b = _operand(k, n, gen)
    c0 = torch.randn(m, n, generator=gen, device="cuda")
    c = c0.clone()
    gemm_bf16(ctx, a, 0, b, 1, c, m, n, k, alpha=0.25, beta=1.0)
    torch.cuda.synchronize()
    ref = 0.25 * (a.double() @ b.double()) + c0.double()
    assert ((c.double() - ref).norm() / ref.norm()) < 1e-5


def test_gemm_long_k(ctx, tiles):
    """Long-K shape of the dgrad GEMM (K = vocabulary)."""
    from orda_b200.device import gemm_bf16

    gen = torch.Generator(device="cuda").manual_seed(9)
    m, n, k = 256, 512, 32000
    a = _operand(m, k, gen)
    b = _operand(k, n, gen)
    c = torch.empty(m, n, device="cuda")
    gemm_bf16(ctx, a, 0, b, 1, c, m, n, k)
    torch.cuda.synchronize()
    ref = a.double() @ b.double()
    # fp32 accumulation of 32000 products: observed 3.7e-5 relative
    assert ((c.double() - ref).norm() / ref.norm()) < 1e-4
