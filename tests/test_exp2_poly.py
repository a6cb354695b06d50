"""The FMA-pipe exp2 of the Fast profile (csrc/fastmath.cuh), on the CPU:
its coefficients are refitted here by the stated procedure and compared with
the constants in the source, and the algorithm (rint by the 1.5 * 2^23
constant, degree-6 Horner with fused multiply-adds, exponent add) is run in
float32 arithmetic with numpy and held to 2 ulp of float64 2^x."""
from __future__ import annotations

import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parent.parent / "orda-cutile-rs_b200" / "csrc" / "fastmath.cuh"


def _constants():
    c = dict(re.findall(r"constexpr float kExp2C(\d) = ([0-9.eE+-]+)f;", SRC.read_text()))
    return np.array([float(c[str(i)]) for i in range(7)], dtype=np.float32)


def test_coefficients_are_the_stated_fit():
    k = np.arange(4000)
    f = 0.5 * np.cos(np.pi * (k + 0.5) / 4000)  # Chebyshev nodes of [-1/2, 1/2]
    y = np.exp2(f)
    a = np.vander(f, 7, increasing=True) / y[:, None]  # relative error
    c, *_ = np.linalg.lstsq(a, np.ones_like(f), rcond=None)
    assert np.array_equal(c.astype(np.float32), _constants())


def _fma32(a, b, c):
    # a * b is exact in float64 for float32 operands; one rounding to float32
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def exp2_fma_emulated(x):
    x = np.clip(np.asarray(x, dtype=np.float32), np.float32(-125.0), np.float32(126.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    n = t.view(np.int32) - np.int32(0x4B400000)
    f = (x - (t - magic).astype(np.float32)).astype(np.float32)
    c = _constants()
    p = np.full_like(f, c[6])
    for i in range(5, -1, -1):
        p = _fma32(p, f, np.full_like(f, c[i]))
    return (p.view(np.int32) + (n << 23)).view(np.float32)


def test_emulated_exp2_within_two_ulp():
    """Over the supported range [-125, 126] (arguments outside are clamped)."""
    rng = np.random.default_rng(5)
    x = np.concatenate([np.linspace(-125.0, 126.0, 400001), rng.uniform(-30, 0, 200000),
                        np.arange(-125, 126, dtype=np.float64) + 0.5,
                        np.arange(-125, 127, dtype=np.float64)]).astype(np.float32)
    got = exp2_fma_emulated(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got / ref - 1.0)
    assert rel.max() < 2 * 2.0 ** -23, rel.max()
    # exact at integers (f = 0: p = 1)
    xi = np.arange(-125, 127, dtype=np.float32)
    assert np.array_equal(exp2_fma_emulated(xi), np.exp2(xi.astype(np.float64)).astype(np.float32))
