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


# Wide pair tiles (256 x 512, two N = 256 MMAs per K slice, one accumulator
# over all 512 TMEM columns): ORDA_GEMM_WIDE=2 forces them for every
# store-epilogue GEMM with N > 256. (3328, 4096) gives 104 tiles, i.e. one
# full wave of 74 pairs and a last wave of 30 tiles, which is split into two
# K halves reduce-added into the zeroed output; (256, 768) and (200, 1000)
# give fewer tiles than pairs (split when K has two blocks or more) with N
# and M tails.
WIDE_SHAPES = [
    (3328, 4096, 512),
    (3300, 4000, 520),
    (256, 768, 64),
    (200, 1000, 1000),
]


@pytest.mark.parametrize("a_kind,b_kind", [(0, 0), (0, 1), (1, 1), (1, 0)])
@pytest.mark.parametrize("m,n,k", WIDE_SHAPES)
def test_gemm_wide_tiles(ctx, monkeypatch, a_kind, b_kind, m, n, k):
    from orda_b200.device import gemm_bf16

    monkeypatch.setenv("ORDA_GEMM_CTA_PAIR", "1")
    monkeypatch.setenv("ORDA_GEMM_WIDE", "2")
    gen = torch.Generator(device="cuda").manual_seed(m * 3 + n * 5 + k)
    a = _operand(m, k, gen) if a_kind == 0 else _operand(k, m, gen)
    b = _operand(n, k, gen) if b_kind == 0 else _operand(k, n, gen)
    outs = []
    for _ in range(2):
        c = torch.full((m, n), float("nan"), device="cuda", dtype=torch.float32)
        gemm_bf16(ctx, a, a_kind, b, b_kind, c, m, n, k)
        outs.append(c)
    torch.cuda.synchronize()
    ctx.check()
    A = (a if a_kind == 0 else a.t()).double()
    B = (b.t() if b_kind == 0 else b).double()
    ref = A @ B
    assert torch.isfinite(outs[0]).all()
    err = (outs[0].double() - ref).norm() / ref.norm()
    assert err < 1e-5, f"rel L2 {err:.3e}"
    # the split halves land in either order with the same sum
    assert torch.equal(outs[0], outs[1])


def test_gemm_wide_alpha_beta_accumulate(ctx, monkeypatch):
    """beta = 1 accumulates through TMA reduce-add, so no tile is split."""
    from orda_b200.device import gemm_bf16

    monkeypatch.setenv("ORDA_GEMM_CTA_PAIR", "1")
    monkeypatch.setenv("ORDA_GEMM_WIDE", "2")
    gen = torch.Generator(device="cuda").manual_seed(6)
    m, n, k = 640, 1536, 192
    a = _operand(m, k, gen)
    b = _operand(k, n, gen)
    c0 = torch.randn(m, n, generator=gen, device="cuda")
    c = c0.clone()
    gemm_bf16(ctx, a, 0, b, 1, c, m, n, k, alpha=0.25, beta=1.0)
    torch.cuda.synchronize()
    ref = 0.25 * (a.double() @ b.double()) + c0.double()
    assert ((c.double() - ref).norm() / ref.norm()) < 1e-5


def test_gemm_large_selects_wide_tiles(ctx, monkeypatch):
    """A store GEMM with two waves of wide tiles (19 x 8 = 152 tiles for 74
    pairs) and 128 K blocks takes wide tiles by default; its last wave of 4
    tiles is split into K halves. Against ORDA_GEMM_WIDE=0 and the float64
    product: unsplit tiles sum K in the same order either way, so only the
    split tiles differ."""
    from orda_b200.device import gemm_bf16

    monkeypatch.setenv("ORDA_GEMM_CTA_PAIR", "1")
    gen = torch.Generator(device="cuda").manual_seed(10)
    m, n, k = 19 * 256, 4096, 8192
    a = _operand(m, k, gen)
    b = _operand(k, n, gen)
    res = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("ORDA_GEMM_WIDE", mode)
        c = torch.empty(m, n, device="cuda")
        gemm_bf16(ctx, a, 0, b, 1, c, m, n, k)
        res[mode] = c
    torch.cuda.synchronize()
    ctx.check()
    ref = a.double() @ b.double()
    for mode, c in res.items():
        assert ((c.double() - ref).norm() / ref.norm()) < 1e-4, mode
    d = (res["1"].double() - res["0"].double()).norm() / ref.norm()
    assert 0 < d < 1e-4, d
