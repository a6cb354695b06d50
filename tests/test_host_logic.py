"""Host logic of liborda_b200.so, checked on CPU against the oracle: the
library loads, exports every entry point of include/orda.h, and its
configuration defaults, chunk resolver, OOM ladder and argument validation
(messages included) agree with the reference restatement. No device compute
is called here.
"""
from __future__ import annotations

import ctypes as C
import itertools
import re
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent


def declared_entry_points():
    names = []
    for h in sorted((REPO / "include").glob("*.h")):
        names += re.findall(r"^ORDA_API\s+[\w\s\*]+?\b(orda_\w+)\(", h.read_text(), flags=re.M)
    return names


def test_library_exports_every_declared_symbol(ob):
    lib = ob.load_library()
    names = declared_entry_points()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ but not exported"
    from orda_b200 import _abi

    assert set(names) == set(_abi.SIGNATURES), "ctypes signature table out of sync with include/orda.h"


def test_loss_options_defaults_match_reference(ob, oracle):
    """`LossOptions::default` src/api.rs:49-64 and KernelConfig defaults."""
    from orda_b200 import _abi

    a, b = _abi.OrdaLossOptions(), _abi.OrdaLossOptions()
    ob.load_library().orda_loss_options_default(C.byref(a))
    oracle.lib().oref_loss_options_default(C.byref(b))
    assert bytes(a) == bytes(b)
    py = ob.LossOptions()
    assert bytes(py._c()) == bytes(a)
    assert a.student_ce_weight == 1.0 and a.has_teacher_ce_weight == 0 and a.kd_weight == 0.0
    assert a.temperature == 1.0 and a.ignore_index == -100 and a.label_smoothing == 0.0
    assert a.config.max_fused_size == 32768


@pytest.mark.parametrize("profile", [0, 1, 2])
def test_kernel_config_from_profile(ob, oracle, profile):
    from orda_b200 import _abi

    a, b = _abi.OrdaKernelConfig(), _abi.OrdaKernelConfig()
    ob.load_library().orda_kernel_config_from_profile(profile, C.byref(a))
    oracle.lib().oref_kernel_config_from_profile(profile, C.byref(b))
    assert bytes(a) == bytes(b)
    assert ob.KernelConfig.from_profile(ob.Profile(profile)).fast_math == (profile == 1)


def test_kernel_config_validate_messages(ob):
    c = ob.KernelConfig(max_fused_size=100)
    with pytest.raises(ob.OrdaError, match=r"^max_fused_size must be a power of two >= 1, got 100$"):
        c.validate()
    with pytest.raises(ob.OrdaError, match=r"^max_chunks must be >= 1, got 0$"):
        ob.KernelConfig(max_chunks=0).validate()
    ob.KernelConfig().validate()


def test_chunks_from_raw_grid(ob, oracle):
    for raw in [0.0, 1.0, 1.49, 1.5, 2.99, 3.0, 6.0, 128.0, 1e6, 1e30, float("inf")]:
        assert ob.chunks_from_raw(raw) == oracle.chunks_from_raw(raw)


def test_resolver_grid_matches_oracle(ob, oracle):
    bts = [1, 7, 100, 256, 511, 512, 1000, 2048, 4097, 8192, 65536]
    vs = [None, 7, 8192, 32000, 128256, 131072, 152064]
    mcs = [None, 1, 3, 32]
    for bt, v, mc in itertools.product(bts, vs, mcs):
        for cs in (ob.ChunkSize.Auto(), ob.ChunkSize.Fixed(0), ob.ChunkSize.Fixed(64), ob.ChunkSize.Fixed(10**9)):
            assert ob.resolve_chunk_size(bt, cs, v, mc) == oracle.resolve_chunk_size(bt, cs, v, mc), (bt, v, mc, cs)


def test_resolver_known_answers(ob):
    """The golden integers of src/resolver.rs:132-181 and the BASELINE plans."""
    assert ob.resolve_chunk_size(1000, ob.ChunkSize.Fixed(256), None, None) == ob.ChunkPlan(256, 4)
    assert ob.resolve_chunk_size(100, ob.ChunkSize.Fixed(4096), None, None) == ob.ChunkPlan(100, 1)
    assert ob.resolve_chunk_size(8192, ob.ChunkSize.Auto(), None, None) == ob.ChunkPlan(8192, 1)
    assert ob.resolve_chunk_size(8192, ob.ChunkSize.Auto(), 131072, None) == ob.ChunkPlan(512, 16)
    assert ob.resolve_chunk_size(2048, ob.ChunkSize.Auto(), 32000, None) == ob.ChunkPlan(1024, 2)
    assert ob.resolve_chunk_size(256, ob.ChunkSize.Auto(), 8192, None) == ob.ChunkPlan(256, 1)
    assert ob.resolve_chunk_size(8192, ob.ChunkSize.Auto(), 152064, None) == ob.ChunkPlan(512, 16)


def test_doubling_schedule_grid(ob, oracle):
    assert ob.chunk_doubling_schedule(10_000, 4, 32) == [4, 8, 16, 32]
    assert ob.chunk_doubling_schedule(20, 4, 1000) == [4, 8, 16, 20]
    for bt, start, limit in itertools.product([1, 5, 20, 512, 8192], [0, 1, 3, 16, 100], [0, 1, 7, 32, 10**6]):
        assert ob.chunk_doubling_schedule(bt, start, limit) == oracle.chunk_doubling_schedule(bt, start, limit)
    for bt in [1, 511, 512, 8192]:
        assert ob.default_max_chunks_limit(bt) == oracle.default_max_chunks_limit(bt)


def test_oom_ladder_with_failing_allocator(ob):
    """The OOM retry ladder (the upstream dispatcher's `dynamic_chunk` loop,
    documented at src/resolver.rs:107-126) driven by an injected allocator
    that fails the first k requests -- no device involved."""
    tried = []

    def fail_first(k):
        def f(nc, cs):
            tried.append((nc, cs))
            return len(tried) > k

        return f

    assert ob.chunk_retry(8192, 16, 32, fail_first(0)) == ob.ChunkPlan(512, 16)
    tried.clear()
    assert ob.chunk_retry(8192, 16, 32, fail_first(1)) == ob.ChunkPlan(256, 32)
    assert tried == [(16, 512), (32, 256)]
    tried.clear()
    assert ob.chunk_retry(8192, 16, 32, fail_first(5)) is None
    tried.clear()
    assert ob.chunk_retry(20, 4, 1000, fail_first(2)) == ob.ChunkPlan(2, 16)


def test_teacher_default_weight(ob):
    assert ob.Teacher.Tied(ob.Mat.zeros(2, 3)).default_teacher_ce_weight() == 1.0
    assert ob.Teacher.Separate(ob.Mat.zeros(2, 3), ob.Mat.zeros(5, 3)).default_teacher_ce_weight() == 0.0
    assert ob.Teacher.Precomputed(ob.Mat.zeros(2, 5)).default_teacher_ce_weight() == 0.0


def _base(ob):
    bt, h, v = 4, 3, 5
    s = ob.Mat.zeros(bt, h)
    w = ob.Mat.zeros(v, h)
    return bt, h, v, s, w


VALIDATION_CASES = [
    # (description, builder) -> expected message (src/api.rs:104-181)
    ("bt0", "student_hidden has 0 rows (BT must be > 0)"),
    ("wshape", "weight must have shape (V, 3), got (5, 4)"),
    ("nlabels", "labels must have length BT=4, got 3"),
    ("label_range", "label 5 out of range [0, 5) and != ignore_index -100"),
    ("label_neg", "label -1 out of range [0, 5) and != ignore_index -100"),
    ("smoothing", "label_smoothing must be in [0,1], got 1.5"),
    ("smoothing_nan", "label_smoothing must be in [0,1], got NaN"),
    ("kd", "kd_weight must be >= 0, got -0.1"),
    ("temp", "temperature must be > 0, got 0"),
    ("tied", "Tied teacher hidden must be (4, 3), got (4, 2)"),
    ("sep_rows", "Separate teacher hidden must have BT=4 rows"),
    ("sep_w", "Separate teacher weight must be (5, 2), got (5, 3)"),
    ("pre", "Precomputed teacher logits must be (4, 5), got (4, 4)"),
    ("fused", "max_fused_size must be a power of two >= 1, got 100"),
]


def _case(ob, name):
    bt, h, v, s, w = _base(ob)
    labels = [0, 1, 2, 3]
    teacher = ob.Teacher.Tied(ob.Mat.zeros(bt, h))
    opts = ob.LossOptions()
    if name == "bt0":
        s = ob.Mat.zeros(0, h)
        labels = []
    elif name == "wshape":
        w = ob.Mat.zeros(5, 4)
    elif name == "nlabels":
        labels = [0, 1, 2]
    elif name == "label_range":
        labels = [0, 1, 5, 2]
    elif name == "label_neg":
        labels = [0, -1, 2, 3]
    elif name == "smoothing":
        opts.label_smoothing = 1.5
    elif name == "smoothing_nan":
        opts.label_smoothing = float("nan")
    elif name == "kd":
        opts.kd_weight = -0.1
    elif name == "temp":
        opts.temperature = 0.0
    elif name == "tied":
        teacher = ob.Teacher.Tied(ob.Mat.zeros(bt, 2))
    elif name == "sep_rows":
        teacher = ob.Teacher.Separate(ob.Mat.zeros(3, 2), ob.Mat.zeros(v, 2))
    elif name == "sep_w":
        teacher = ob.Teacher.Separate(ob.Mat.zeros(bt, 2), ob.Mat.zeros(v, 3))
    elif name == "pre":
        teacher = ob.Teacher.Precomputed(ob.Mat.zeros(bt, 4))
    elif name == "fused":
        opts.config = ob.KernelConfig(max_fused_size=100)
    return s, w, labels, teacher, opts


@pytest.mark.parametrize("name,msg", VALIDATION_CASES)
def test_validation_messages_match_reference(ob, oracle, name, msg):
    s, w, labels, teacher, opts = _case(ob, name)
    with pytest.raises(ob.OrdaError) as e:
        from orda_b200 import validate

        validate(s, w, labels, teacher, opts)
    assert e.value.message == msg
    with pytest.raises(oracle.OracleError) as e2:
        oracle.validate(s, w, labels, teacher, opts)
    assert e2.value.message == msg


def test_validation_accepts_ignore_index_and_valid_input(ob):
    from orda_b200 import validate

    bt, h, v, s, w = _base(ob)
    assert validate(s, w, [0, -100, 4, 3], ob.Teacher.Tied(ob.Mat.zeros(bt, h)), ob.LossOptions()) == (v, h, bt)
    opts = ob.LossOptions(ignore_index=7)
    with pytest.raises(ob.OrdaError, match="label -100 out of range"):
        validate(s, w, [0, -100, 4, 3], ob.Teacher.Tied(ob.Mat.zeros(bt, h)), opts)


def test_backend_cpu_is_rejected(ob):
    """The B200 library has no CPU path: Backend::Cpu is an error."""
    bt, h, v, s, w = _base(ob)
    opts = ob.LossOptions(backend=ob.Backend.Cpu)
    with pytest.raises(ob.OrdaError, match="Backend::Cpu is not available"):
        ob.distillation_loss(s, w, [0, 1, 2, 3], ob.Teacher.Tied(ob.Mat.zeros(bt, h)), opts)


def test_negative_teacher_weight_is_rejected(ob):
    """src/api.rs:214-216."""
    bt, h, v, s, w = _base(ob)
    opts = ob.LossOptions(teacher_ce_weight=-1.0)
    with pytest.raises(ob.OrdaError, match=r"^teacher_ce_weight must be >= 0, got -1$"):
        ob.distillation_loss(s, w, [0, 1, 2, 3], ob.Teacher.Tied(ob.Mat.zeros(bt, h)), opts)


def test_no_gpu_fails_loudly_without_fallback(ob):
    """Without a B200 the library reports an error instead of computing on
    the CPU."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert not ob.is_available()
    bt, h, v, s, w = _base(ob)
    with pytest.raises(ob.OrdaError, match="no sm_100 CUDA device"):
        ob.distillation_loss(s, w, [0, 1, 2, 3], ob.Teacher.Tied(ob.Mat.zeros(bt, h)), ob.LossOptions())
