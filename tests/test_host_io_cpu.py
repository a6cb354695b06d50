"""The host-side passes of the host-Mat entry (host_io.cc), on the CPU: the
fp32 -> bf16 rounding that must equal the device's, the exact narrowing of
teacher logits that hold bf16 values, and the dequantisation of grad_W,
each in every instruction-set version this CPU runs, against the scalar
definitions (orda_selftest_host_io); and the scalar rounding rule itself
against numpy's round-to-nearest-even on the bit patterns."""
from __future__ import annotations

import ctypes as C

import numpy as np


def test_host_io_versions_agree_with_the_scalar_definitions(ob):
    lib = ob.load_library()
    buf = C.create_string_buffer(256)
    rc = lib.orda_selftest_host_io(buf, len(buf))
    assert rc == 0, buf.value.decode()
    assert buf.value.decode().startswith("checked: scalar")


def test_bf16_rounding_rule_is_round_to_nearest_even():
    """bf16_bits.h on finite values: the high half of the value rounded to 8
    significant bits, ties to even; checked against an independent integer
    restatement (round half to even on the dropped 16 bits)."""
    rng = np.random.default_rng(3)
    b = rng.integers(0, 2 ** 32, 200000, dtype=np.uint64).astype(np.uint32)
    b = b[(b & 0x7FFFFFFF) < 0x7F800000]  # finite
    hi, lo = (b >> 16).astype(np.uint64), (b & 0xFFFF).astype(np.uint64)
    up = (lo > 0x8000) | ((lo == 0x8000) & (hi & 1 == 1))
    want = (hi + up).astype(np.uint64) & 0xFFFF
    got = ((b.astype(np.uint64) + 0x7FFF + ((b >> 16) & 1)) >> 16) & 0xFFFF
    assert np.array_equal(got, want)
