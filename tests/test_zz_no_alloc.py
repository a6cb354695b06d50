"""The allocation-free quantiser entry point, through the C ABI.

orda_quantize_grad_w_device_noalloc serves callers that cannot call
cudaMalloc (allocator hooks, out-of-memory handlers, runtimes that forbid
device allocations after start-up): its scratch is a fixed device array in
the library instead of a context workspace. These tests check that its output
equals the regular entry point's (orda_quantize_grad_w_device) and, bit for
bit, the oracle's restatement of the reference quantiser, each on two calls in
a row, the second with different labels so stale scratch from the first call
would show, and that a V above the stated limit is rejected.

The file name sorts last so a run that stops at the first failure has already
run every other test; it also passes alone in a fresh process.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _call_noalloc(lib, g, labels, stochastic, seed, q, sc):
    from orda_b200 import _abi

    v, h = g.shape
    buf = _abi.err_buf()
    rc = lib.orda_quantize_grad_w_device_noalloc(
        g.data_ptr(), v, h, g.stride(0), labels.data_ptr(), labels.numel(), -100, int(stochastic), seed,
        q.data_ptr(), sc.data_ptr(), torch.cuda.current_stream().cuda_stream, buf, len(buf))
    return rc, buf.value.decode()


@pytest.mark.parametrize("stochastic", [False, True])
def test_noalloc_quantizer_matches_regular_entry_twice(stochastic):
    import orda_b200 as ob
    from orda_b200.device import DeviceContext, quantize_grad_w

    lib = ob.load_library()
    gen = torch.Generator(device="cuda").manual_seed(3)
    v, h = 4099, 700
    base = torch.randn(v, h, generator=gen, device="cuda") * 1e-3
    with DeviceContext(0) as ctx:
        for call, n_labels in enumerate((500, 37)):
            labels = torch.randint(0, v, (n_labels,), generator=gen, device="cuda")
            labels[::5] = -100
            ref = base.clone()
            q_ref = torch.empty(v, h, dtype=torch.int8, device="cuda")
            s_ref = torch.empty(v, device="cuda")
            quantize_grad_w(ctx, ref, labels, -100, stochastic, 99 + call, q_ref, s_ref)

            got = base.clone()
            q = torch.empty(v, h, dtype=torch.int8, device="cuda")
            s = torch.empty(v, device="cuda")
            rc, msg = _call_noalloc(lib, got, labels, stochastic, 99 + call, q, s)
            assert rc == 0, msg
            torch.cuda.synchronize()
            ctx.check()
            # same kernels on the same inputs: bit-identical outputs
            assert torch.equal(q, q_ref)
            assert torch.equal(s.view(torch.int32), s_ref.view(torch.int32))
            assert torch.equal(got.view(torch.int32), ref.view(torch.int32))
            # target rows of this call (and only those) are kept exact
            tgt = sorted({int(t) for t in labels.tolist() if t != -100})
            kept = (got == base).all(dim=1).nonzero().flatten().tolist()
            assert set(tgt) <= set(kept)


@pytest.mark.parametrize("stochastic", [False, True])
def test_noalloc_quantizer_bit_exact_with_oracle(oracle, stochastic):
    """The allocation-free entry against the oracle's restatement of
    `quantize_grad_w` + `dequantize_grad_w` (src/quant.rs:157-202) directly:
    INT8 codes, scales and the dequantised matrix bit-identical on the same
    fp32 grad_W, on two calls in a row with different target rows."""
    import orda_b200 as ob

    lib = ob.load_library()
    gen = torch.Generator().manual_seed(17)
    v, h = 2053, 384
    base = (torch.randn(v, h, generator=gen) * torch.rand(v, 1, generator=gen) ** 3 * 1e-3).numpy()
    base[11, :] = 0.0  # amax 0: the scale comes from the 1e-12 floor
    for call, n_labels in enumerate((700, 23)):
        labels = torch.randint(0, v, (n_labels,), generator=gen)
        labels[::6] = -100
        seed = 4242 + call
        q_ref, s_ref, deq_ref = oracle.quantize_grad_w(base, labels.numpy(), -100, stochastic=stochastic, seed=seed)
        g = torch.from_numpy(base).cuda()
        q = torch.empty(v, h, dtype=torch.int8, device="cuda")
        s = torch.empty(v, device="cuda")
        rc, msg = _call_noalloc(lib, g, labels.cuda(), stochastic, seed, q, s)
        assert rc == 0, msg
        torch.cuda.synchronize()
        assert np.array_equal(q.cpu().numpy(), q_ref)
        assert np.array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))
        assert np.array_equal(g.cpu().numpy().view(np.uint32), deq_ref.view(np.uint32))


def test_noalloc_rejects_v_above_limit():
    import orda_b200 as ob

    lib = ob.load_library()
    limit = 262144  # ORDA_NOALLOC_MAX_V in include/orda.h
    g = torch.zeros(limit + 1, 8, device="cuda")
    labels = torch.zeros(4, dtype=torch.int64, device="cuda")
    q = torch.empty(limit + 1, 8, dtype=torch.int8, device="cuda")
    s = torch.empty(limit + 1, device="cuda")
    rc, msg = _call_noalloc(lib, g, labels, False, 0, q, s)
    assert rc != 0
    assert "exceeds the no-allocation limit" in msg
