"""Pins the CPU oracle to the reference's own unit tests.

Each test restates one `#[test]` of malcolmgreaves/orda-cutile-rs (the file and
line are in the docstring) and runs it against oracle/liborda_oracle.so. The
reference ships no stored output files, so these known-answer tests and
identities are the golden vectors for this path.
"""
from __future__ import annotations

import math

import numpy as np
import pytest


# ------------------------------------------------------------------ mat.rs
def test_matmul_nt_basic(oracle):
    """src/mat.rs:151-159."""
    c = oracle.matmul_nt(np.array([[1, 2, 3]]), np.array([[1, 0, 0], [0, 1, 1]]))
    assert c.shape == (1, 2)
    assert c.tolist() == [[1.0, 5.0]]


def test_matmul_nn_and_tn_consistent(oracle):
    """src/mat.rs:161-176."""
    a = np.array([[1.0, 2.0], [3.0, 4.0]])
    b = np.array([[1.0, 0.0, 1.0], [0.0, 1.0, 0.0]])
    c = oracle.matmul_tn(a, b)
    assert c.shape == (2, 3)
    assert c[0].tolist() == [1.0, 3.0, 1.0]
    assert c[1].tolist() == [2.0, 4.0, 2.0]
    d = oracle.matmul_nn(a, b)
    assert d[0].tolist() == [1.0, 2.0, 1.0]
    assert d[1].tolist() == [3.0, 4.0, 3.0]


def test_matmul_thread_count_is_bit_identical(oracle):
    rng = np.random.default_rng(0)
    a = rng.standard_normal((17, 33)).astype(np.float32)
    b = rng.standard_normal((29, 33)).astype(np.float32)
    assert np.array_equal(oracle.matmul_nt(a, b, 1), oracle.matmul_nt(a, b, 4))
    g = rng.standard_normal((17, 29)).astype(np.float32)
    g[3, :] = 0.0
    assert np.array_equal(oracle.matmul_nn(g, b, 1), oracle.matmul_nn(g, b, 4))
    assert np.array_equal(oracle.matmul_tn(g, a, 1), oracle.matmul_tn(g, a, 4))
    # sequential f32 accumulation, no FMA contraction: compare to an explicit loop
    acc = np.float32(0.0)
    for p in range(33):
        acc = np.float32(acc + np.float32(a[2, p] * b[5, p]))
    assert oracle.matmul_nt(a, b)[2, 5] == acc


# ---------------------------------------------------------- reference/kl.rs
def test_identical_distributions_have_zero_kl(oracle):
    """src/reference/kl.rs:159-164."""
    row = [0.3, 1.2, -0.7, 2.1, 0.0]
    assert abs(oracle.forward_kl_row(row, row, 1.5)) < 1e-12


def test_kl_is_nonnegative(oracle):
    """src/reference/kl.rs:166-174."""
    s = [0.1, 0.2, 0.3, -1.0, 2.0]
    t = [1.0, -0.5, 0.0, 0.7, 0.2]
    for temp in [0.5, 1.0, 1.5, 4.0]:
        assert oracle.forward_kl_row(s, t, temp) >= -1e-12


def test_kl_matches_closed_form_two_class(oracle):
    """src/reference/kl.rs:176-196."""
    temperature = 2.0
    inv_t = 1.0 / temperature
    s = np.array([0.7, -0.4], np.float32)
    t = np.array([-0.2, 1.1], np.float32)

    def sig(a, b):
        za, zb = float(a) * inv_t, float(b) * inv_t
        m = max(za, zb)
        d = math.exp(za - m) + math.exp(zb - m)
        return math.exp(za - m) / d, math.exp(zb - m) / d

    ps0, ps1 = sig(s[0], s[1])
    pt0, pt1 = sig(t[0], t[1])
    expected = pt0 * (math.log(pt0) - math.log(ps0)) + pt1 * (math.log(pt1) - math.log(ps1))
    assert abs(oracle.forward_kl_row(s, t, temperature) - expected) < 1e-12


def test_kl_ignored_rows_contribute_zero(oracle):
    """src/reference/kl.rs:198-206."""
    logits = np.array([[1.0, 2.0, 3.0], [0.5, -0.5, 0.0]], np.float32)
    kl, grad = oracle.kl_reference_chunk(logits, [-100], 1, 0.4, 1.5, 1, -100, True)
    assert kl == 0.0
    assert np.all(grad == 0.0)


def test_kl_grad_matches_temperature_scaling(oracle):
    """src/reference/kl.rs:208-223."""
    logits = np.array([[0.2, 0.5, -0.1], [1.0, -1.0, 0.3]], np.float32)
    kw, temp = np.float32(0.4), np.float32(1.5)
    _kl, grad = oracle.kl_reference_chunk(logits, [1], 1, kw, temp, 1, -100, True)
    inv_t = 1.0 / float(temp)
    ps, _ = oracle.softmax_logsoftmax(logits[0], inv_t)
    pt, _ = oracle.softmax_logsoftmax(logits[1], inv_t)
    gs = np.float32(kw * temp / np.float32(1.0))
    for j in range(3):
        expected = gs * np.float32(ps[j] - pt[j])
        assert abs(grad[0, j] - expected) < 1e-6


# ------------------------------------------------ reference/cross_entropy.rs
def _softmax(x):
    m = float(np.max(np.asarray(x, np.float32)))
    d = sum(math.exp(float(v) - m) for v in x)
    return [math.exp(float(v) - m) / d for v in x]


def test_nll_equals_negative_log_softmax_of_target(oracle):
    """src/reference/cross_entropy.rs:91-99."""
    x = [1.0, 2.0, 0.5, -1.0]
    nll = oracle.ce_loss_row(x, 1, -100, 0.0)
    assert abs(float(nll) - (-math.log(_softmax(x)[1]))) < 1e-6


def test_grad_is_softmax_minus_onehot(oracle):
    """src/reference/cross_entropy.rs:101-121."""
    x = [0.3, -0.7, 1.1, 0.0]
    _nll, grad = oracle.ce_fwdbwd_row(x, 2, -100, 0.0, 1.0)
    p = _softmax(x)
    for j in range(4):
        expected = p[j] - (1.0 if j == 2 else 0.0)
        assert abs(float(grad[j]) - expected) < 1e-6
    assert abs(sum(float(g) for g in grad)) < 1e-5


def test_ce_ignored_row_is_zero(oracle):
    """src/reference/cross_entropy.rs:123-129."""
    nll, grad = oracle.ce_fwdbwd_row([3.0, 1.0, -2.0], -100, -100, 0.0, 1.0)
    assert nll == 0.0
    assert np.all(grad == 0.0)


def test_scale_scales_gradient(oracle):
    """src/reference/cross_entropy.rs:131-139."""
    x = [0.5, -0.5, 1.0]
    _n1, g1 = oracle.ce_fwdbwd_row(x, 0, -100, 0.0, 1.0)
    _n2, g2 = oracle.ce_fwdbwd_row(x, 0, -100, 0.0, 2.5)
    assert np.all(np.abs(g2 - np.float32(2.5) * g1) < 1e-6)


def test_label_smoothing_grad_sums_to_zero(oracle):
    """src/reference/cross_entropy.rs:141-148."""
    _nll, grad = oracle.ce_fwdbwd_row([0.2, 1.3, -0.4, 0.9, 0.0], 3, -100, 0.1, 1.0)
    assert abs(float(np.sum(grad.astype(np.float64)))) < 1e-5


# ---------------------------------------------------------------- quant.rs
def test_round_half_even_cases(oracle):
    """src/quant.rs:208-216."""
    cases = {0.5: 0.0, 1.5: 2.0, 2.5: 2.0, -1.5: -2.0, 2.4: 2.0, 2.6: 3.0}
    for x, want in cases.items():
        assert oracle.round_half_even(x) == want


def test_deterministic_roundtrip_bounded_error(oracle):
    """src/quant.rs:218-231."""
    m = np.array([[1.0, -2.0, 0.5, 3.0], [-0.1, 0.2, -0.3, 0.05]], np.float32)
    q, s = oracle.quantize_rowwise_int8(m)
    deq = q.astype(np.float32) * s[:, None]
    for r in range(2):
        assert np.all(np.abs(m[r] - deq[r]) <= 0.5 * s[r] + 1e-6)


def test_stochastic_is_unbiased(oracle):
    """src/quant.rs:233-255: 20000 draws from one SplitMix64 stream (seed
    12345). Consecutive calls on a 1x3 matrix consume the stream in the same
    order as one call on the 20000x3 matrix of repeated rows."""
    row = np.array([0.37, -1.23, 2.71], np.float32)
    m = np.tile(row, (20000, 1))
    q, s = oracle.quantize_rowwise_int8_stochastic(m, 12345)
    deq = q.astype(np.float32) * s[:, None]
    mean = (deq.astype(np.float64).sum(axis=0) / 20000).astype(np.float32)
    assert np.all(np.abs(mean - row) < 1e-2)


def test_grad_w_target_rows_are_exact(oracle):
    """src/quant.rs:257-275."""
    grad_w = np.array([[10.0, -10.0], [0.123, 0.456], [-7.0, 7.0], [0.01, -0.02]], np.float32)
    target = [0, 2, -100]
    assert oracle.unique_targets(target, -100, 4) == [0, 2]
    _q, _s, deq = oracle.quantize_grad_w(grad_w, target, -100)
    assert np.array_equal(deq[0], grad_w[0])
    assert np.array_equal(deq[2], grad_w[2])
    assert np.all(np.abs(deq[1] - grad_w[1]) < 0.02)


def test_rng_matches_splitmix64_definition(oracle):
    """SplitMix64 of src/quant.rs:18-44 recomputed in Python from its
    definition: state = seed + (k+2)*golden before the k-th mix."""
    mask = (1 << 64) - 1
    golden = 0x9E3779B97F4A7C15
    seed = 12345
    got = oracle.rng_f32_stream(seed, 5)
    for k in range(5):
        z = (seed + (k + 2) * golden) & mask
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & mask
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & mask
        z ^= z >> 31
        assert got[k] == np.float32(z >> 40) * np.float32(1.0 / (1 << 24))


# ------------------------------------------------------------- resolver.rs
def test_fixed_chunking(oracle, ob):
    """src/resolver.rs:132-146."""
    p = oracle.resolve_chunk_size(1000, ob.ChunkSize.Fixed(256))
    assert (p.chunk_size, p.num_chunks) == (256, 4)
    p = oracle.resolve_chunk_size(100, ob.ChunkSize.Fixed(4096))
    assert (p.chunk_size, p.num_chunks) == (100, 1)


def test_auto_without_vocab_is_single_chunk(oracle, ob):
    """src/resolver.rs:148-157."""
    p = oracle.resolve_chunk_size(8192, ob.ChunkSize.Auto())
    assert (p.chunk_size, p.num_chunks) == (8192, 1)


def test_chunks_from_raw_matches_python_rule(oracle):
    """src/resolver.rs:159-169."""
    assert [oracle.chunks_from_raw(r) for r in (0.0, 1.49, 1.5, 3.0, 6.0)] == [1, 1, 2, 4, 8]


def test_auto_large_vocab_example(oracle, ob):
    """src/resolver.rs:171-181: BT=8192, V=131072 -> 16 chunks x 512 rows."""
    p = oracle.resolve_chunk_size(8192, ob.ChunkSize.Auto(), 131072)
    assert (p.num_chunks, p.chunk_size) == (16, 512)


def test_doubling_schedule_escalates_to_limit(oracle):
    """src/resolver.rs:183-189."""
    assert oracle.chunk_doubling_schedule(10_000, 4, 32) == [4, 8, 16, 32]
    assert oracle.chunk_doubling_schedule(20, 4, 1000) == [4, 8, 16, 20]


# --------------------------------------------------------- config / teacher
def test_profiles_and_pow2(oracle):
    """src/config.rs:131-153."""
    from orda_b200 import _abi
    import ctypes as C

    for prof, fast in ((0, False), (1, True), (2, False)):
        c = _abi.OrdaKernelConfig()
        oracle.lib().oref_kernel_config_from_profile(prof, C.byref(c))
        assert bool(c.fast_math) == fast
    for p in [1, 2, 4, 8, 1024, 32768]:
        assert oracle.lib().oref_is_power_of_two(p)
    for n in [0, 3, 6, 100, 65535]:
        assert not oracle.lib().oref_is_power_of_two(n)
    c = _abi.OrdaKernelConfig()
    oracle.lib().oref_kernel_config_from_profile(0, C.byref(c))
    c.max_fused_size = 100
    buf = C.create_string_buffer(256)
    assert oracle.lib().oref_kernel_config_validate(C.byref(c), buf, 256) != 0


def test_teacher_default_weights(oracle):
    """src/teacher.rs:66-86."""
    assert oracle.lib().oref_default_teacher_ce_weight(0) == 1.0
    assert oracle.lib().oref_default_teacher_ce_weight(1) == 0.0
    assert oracle.lib().oref_default_teacher_ce_weight(2) == 0.0


@pytest.mark.parametrize(
    "x,want",
    [(1.5, "1.5"), (2.0, "2"), (-0.1, "-0.1"), (0.0, "0"), (1e-7, "0.0000001"), (1e20, "100000000000000000000"),
     (float("nan"), "NaN"), (float("inf"), "inf"), (-2.5, "-2.5"), (123.25, "123.25")],
)
def test_rust_float_display(oracle, x, want):
    """Error messages print f32 with Rust `Display` (shortest round trip,
    never exponent notation)."""
    assert oracle.format_f32(x) == want
