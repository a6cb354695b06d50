"""Row-sharded (data-parallel over tokens) distillation across GPUs.

Each rank owns a contiguous block of the BT rows and a replica of W. Ranks
compute their rows' loss terms and gradients with the global mean
denominator (the token count of all ranks), so the per-rank scalar sums and
grad_W partials add up to the single-GPU result. The only cross-rank traffic
is one reduction of grad_W (reduce-scatter: rank r keeps the vocabulary rows
owner_rows(V, N, r)), a 4-float all-reduce of the loss scalars and, for the
INT8 round trip, an all-gather of the labels so every rank knows the target
rows of its vocabulary slice. grad_hidden stays local.

The collective flow is written against a `compute` callable so the same code
drives the B200 path (NCCL, CUDA tensors) and the CPU tests (gloo, with the
oracle as compute).

SlotReduceScatter replaces the NCCL reduce-scatter of grad_W on one node:
the wgrad GEMM writes each owner's rows into the owner's memory itself.

vocab_sharded_step is the other partitioning, for the largest vocabularies:
W is split by vocabulary rows and every rank sees all tokens.
"""
from __future__ import annotations

import contextlib
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist


def on_stream(stream):
    """Makes `stream` torch's current stream for a block (None keeps the
    current one). torch.distributed orders each NCCL collective after the work
    queued on the current stream when the collective is issued, and makes the
    current stream wait for it; running a step's collectives on the stream
    that carries its device calls is what makes the all-reduce that serves as
    a barrier come after this rank's peer stores, and the slot reduction come
    after the barrier."""
    if stream is None:
        return contextlib.nullcontext()
    if not isinstance(stream, torch.cuda.Stream):
        stream = torch.cuda.ExternalStream(int(stream))
    return torch.cuda.stream(stream)


def shard_rows(bt_total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous row block of `rank` (the first bt_total % world ranks take
    one extra row)."""
    base, extra = divmod(bt_total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def owner_rows(total: int, world: int, rank: int, align: int = 8) -> tuple[int, int]:
    """Rows [r0, r1) of `total` owned by `rank`: slices of ceil(total / world)
    rows rounded up to `align` (so a bf16 or fp32 row block stays 16-byte
    aligned), the last owner taking the remainder. The slot buffers of the
    library (orda_context_slots_create) use the same rule."""
    n = -(-total // world)
    n = -(-n // align) * align
    r0 = min(rank * n, total)
    r1 = min(r0 + n, total)
    if r1 <= r0:
        raise ValueError(f"{total} rows leave rank {rank} of {world} no rows in slices of {n}")
    return r0, r1


def vocab_slice(v: int, world: int, rank: int) -> tuple[int, int]:
    """Vocabulary rows of grad_W owned by `rank` after the reduce-scatter."""
    return owner_rows(v, world, rank)


def gather_labels(labels_local: torch.Tensor, ignore_index: int, capacity: Optional[int] = None,
                  group=None) -> torch.Tensor:
    """Every rank's labels, concatenated by rank. Ranks may hold different
    row counts: each contributes `capacity` entries (default: its own count,
    which must then be equal on all ranks), padded with ignore_index, which
    marks no target row."""
    world = dist.get_world_size(group)
    n = labels_local.numel()
    cap = n if capacity is None else capacity
    if n > cap:
        raise ValueError(f"{n} labels exceed the gather capacity {cap}")
    padded = labels_local
    if n < cap:
        padded = torch.full((cap,), ignore_index, dtype=labels_local.dtype, device=labels_local.device)
        padded[:n] = labels_local
    gathered = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(gathered, padded, group=group)
    return torch.cat(gathered)


def global_non_ignore(labels_local: torch.Tensor, ignore_index: int, group=None) -> int:
    cnt = (labels_local != ignore_index).sum().to(torch.int64).reshape(1)
    dist.all_reduce(cnt, group=group)
    return int(cnt.item())


@dataclass
class ShardResult:
    scalars: torch.Tensor          # global [loss, student_ce, teacher_ce, kl]
    grad_student_hidden: torch.Tensor  # local rows
    grad_weight_slice: torch.Tensor    # this rank's vocabulary slice of grad_W
    vocab_range: tuple[int, int]


def reduce_grad_weight(grad_w: torch.Tensor, group=None) -> torch.Tensor:
    """Sum of grad_W over ranks, returning this rank's vocabulary slice
    (NCCL reduce-scatter when the slices are equal, else an all-reduce)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    v0, v1 = vocab_slice(grad_w.shape[0], world, rank)
    if dist.get_backend(group) == "nccl" and (v1 - v0) * world == grad_w.shape[0]:
        out = torch.empty(v1 - v0, grad_w.shape[1], dtype=grad_w.dtype, device=grad_w.device)
        dist.reduce_scatter_tensor(out, grad_w, group=group)
        return out
    dist.all_reduce(grad_w, group=group)
    return grad_w[v0:v1]


def row_sharded_step(
    compute: Callable[[int], tuple[torch.Tensor, torch.Tensor, torch.Tensor]],
    labels_local: torch.Tensor,
    ignore_index: int,
    n_global: int,
    quantize: Optional[Callable[[torch.Tensor, torch.Tensor], None]] = None,
    group=None,
    label_capacity: Optional[int] = None,
) -> ShardResult:
    """One row-sharded step.

    compute(n_global) -> (scalars[4], grad_student_hidden, grad_weight) runs
    the local rows with the global denominator. quantize(grad_w_slice,
    labels_shifted) applies the INT8 round trip to the reduced slice, with
    labels shifted so the slice's first row is 0. label_capacity: the most
    rows any rank holds, when ranks hold different row counts.
    """
    scalars, gsh, gw = compute(n_global)
    dist.all_reduce(scalars, group=group)
    sl = reduce_grad_weight(gw, group)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    v0, v1 = vocab_slice(gw.shape[0], world, rank)
    if quantize is not None:
        labels_all = gather_labels(labels_local, ignore_index, label_capacity, group)
        shifted = torch.where(labels_all == ignore_index, torch.full_like(labels_all, -1), labels_all - v0)
        quantize(sl, shifted)
    return ShardResult(scalars=scalars, grad_student_hidden=gsh, grad_weight_slice=sl, vocab_range=(v0, v1))


class SlotReduceScatter:
    """The fused grad_W reduce-scatter over the GPUs of one node.

    Every rank allocates a slot buffer fp32 [world][slice][H] for the grad_W
    rows it owns (owner_rows: V need not divide by the world size) and maps
    the other ranks' buffers (CUDA IPC handles exchanged with an all-gather).
    The device entry then runs with scatter_grad_weight: its wgrad GEMM
    stores this rank's partial of every owner's rows straight into that
    owner's buffer while the GEMM runs, so no separate reduce-scatter pass
    over grad_W is left. After a barrier the owner sums the partials in rank
    order (deterministic) and applies the INT8 round trip in the same pass.

    int8_wire (opt-in, lossy): the partials travel as row-wise INT8 codes and
    scales (4x fewer bytes); the device calls must pass int8_wire=True too.
    """

    def __init__(self, ctx, v: int, h: int, group=None, label_capacity: Optional[int] = None,
                 int8_wire: bool = False):
        """label_capacity: the most rows any rank holds in a step, when ranks
        hold different row counts (labels are gathered padded to it)."""
        self.ctx = ctx
        self.group = group
        self.label_capacity = label_capacity
        self.int8_wire = int8_wire
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.v0, self.v1 = vocab_slice(v, self.world, self.rank)
        handle = ctx.slots_create(self.world, self.rank, v, h, 1)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        ctx.slots_attach(handles)
        dev = torch.device("cuda", torch.cuda.current_device())
        self._token = torch.zeros(1, device=dev)
        dist.barrier(group=group)

    def step(
        self,
        compute: Callable[[int], tuple[torch.Tensor, torch.Tensor]],
        labels_local: torch.Tensor,
        ignore_index: int,
        n_global: int,
        grad_weight_slice: torch.Tensor,
        quantize: bool = False,
        stochastic: bool = False,
        seed: int = 0,
        q: Optional[torch.Tensor] = None,
        scale: Optional[torch.Tensor] = None,
        stream=None,
        marks: Optional[list] = None,
    ) -> ShardResult:
        """compute(n_global) -> (scalars[4], grad_student_hidden) runs the
        local rows with scatter_grad_weight; grad_weight_slice [v1 - v0, H]
        receives this rank's reduced (and, with quantize, dequantised) rows.
        marks (optional): two CUDA events, recorded after the barrier and
        after the reduction, for timing. stream: the stream the device calls
        of `compute` use (default: the current stream); the step's
        collectives run on it too."""
        with on_stream(stream):
            return self._step(compute, labels_local, ignore_index, n_global, grad_weight_slice, quantize,
                              stochastic, seed, q, scale, stream, marks)

    def _step(self, compute, labels_local, ignore_index, n_global, grad_weight_slice, quantize, stochastic, seed,
              q, scale, stream, marks):
        labels_all = gather_labels(labels_local, ignore_index, self.label_capacity, self.group)
        scalars, gsh = compute(n_global)
        # the scalar all-reduce is also the barrier after which every rank's
        # partials have landed in this rank's slot buffer
        dist.all_reduce(scalars, group=self.group)
        if marks is not None:
            marks[0].record(stream)
        self.ctx.reduce_slots(grad_weight_slice, labels_all, ignore_index, quantize, stochastic, seed, q, scale,
                              stream=stream, int8_wire=self.int8_wire)
        if marks is not None:
            marks[1].record(stream)
        # the slot buffers are read; the next step's GEMMs may write them
        dist.all_reduce(self._token, group=self.group)
        return ShardResult(scalars=scalars, grad_student_hidden=gsh, grad_weight_slice=grad_weight_slice,
                           vocab_range=(self.v0, self.v1))


# ------------------------------------------------------------------ vocabulary sharding

def vocab_slice_bounds(v_total: int, world: int, rank: int, align: int = 8) -> tuple[int, int]:
    """Vocabulary rows [v0, v1) held by `rank` when V is sharded: near-equal
    contiguous slices whose starts are multiples of `align` (so a bf16 column
    slice of teacher logits stays 16-byte aligned)."""
    return owner_rows(v_total, world, rank, align)


class HiddenSlots:
    """Slot buffers for the vocabulary-sharded grad_hidden reduce-scatter:
    rank r owns hidden rows owner_rows(BT, world, r); set 0 receives the
    student's partials, set 1 the teacher's (when teacher hidden gradients
    exist). The dgrad GEMMs store each owner's rows into its buffer."""

    def __init__(self, ctx, bt: int, h: int, teacher: bool, group=None):
        self.ctx = ctx
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.r0, self.r1 = owner_rows(bt, self.world, self.rank)
        self.teacher = teacher
        handle = ctx.slots_create(self.world, self.rank, bt, h, 2 if teacher else 1)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        ctx.slots_attach(handles)
        dev = torch.device("cuda", torch.cuda.current_device())
        self._token = torch.zeros(1, device=dev)
        self.grad_student_hidden = torch.empty(self.r1 - self.r0, h, device=dev)
        self.grad_teacher_hidden = torch.empty(self.r1 - self.r0, h, device=dev) if teacher else None
        dist.barrier(group=group)


def vocab_sharded_step(ctx, student_hidden, weight_slice, labels, teacher_mode, v_total: int, v0: int,
                       teacher_hidden=None, teacher_weight_slice=None, teacher_logits_slice=None, opts=None,
                       out: Optional[dict] = None, want_int8: bool = False, stream=None, group=None,
                       hidden_slots: Optional[HiddenSlots] = None):
    """One vocabulary-sharded step (tensor parallel over the output head).

    Every rank holds all rows of the hidden states and labels and the
    vocabulary rows [v0, v0 + len(weight_slice)) of W (of a Separate
    teacher's W, or those columns of Precomputed teacher logits). The ranks
    exchange one small tuple of row statistics per row (all-gather) between
    the two device phases, then combine grad_hidden and the scalars.
    grad_weight of the result is this rank's slice, complete; the scalars are
    the full-vocabulary values on every rank. grad_hidden is all-reduced (the
    full [BT, H] on every rank), or, with hidden_slots, reduce-scattered by
    the dgrad GEMMs themselves: the result then holds this rank's rows
    hidden_slots.r0:r1 of the full-vocabulary grad_hidden. stream: the
    stream of the device calls (default: the current stream); the
    collectives run on it too.
    """
    with on_stream(stream):
        return _vocab_sharded_step(ctx, student_hidden, weight_slice, labels, teacher_mode, v_total, v0,
                                   teacher_hidden, teacher_weight_slice, teacher_logits_slice, opts, out, want_int8,
                                   stream, group, hidden_slots)


def _vocab_sharded_step(ctx, student_hidden, weight_slice, labels, teacher_mode, v_total, v0, teacher_hidden,
                        teacher_weight_slice, teacher_logits_slice, opts, out, want_int8, stream, group,
                        hidden_slots):
    from .device import vocab_backward_device, vocab_forward_device

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    kw = dict(teacher_hidden=teacher_hidden, teacher_weight_slice=teacher_weight_slice,
              teacher_logits_slice=teacher_logits_slice, opts=opts, stream=stream)
    part = vocab_forward_device(ctx, student_hidden, weight_slice, labels, teacher_mode, v_total, v0, **kw)
    every = torch.empty((world,) + tuple(part.shape), device=part.device, dtype=part.dtype)
    dist.all_gather_into_tensor(every, part, group=group)
    res = vocab_backward_device(ctx, student_hidden, weight_slice, labels, teacher_mode, v_total, v0, every,
                                include_rows=(rank == 0), out=out, want_int8=want_int8,
                                scatter_grad_hidden=hidden_slots is not None, **kw)
    # with hidden_slots this all-reduce is also the barrier after which every
    # rank's grad_hidden partials have landed in the owners' slot buffers
    dist.all_reduce(res.scalars, group=group)
    if hidden_slots is not None:
        ctx.reduce_slot_set(0, hidden_slots.grad_student_hidden, stream=stream)
        res.grad_student_hidden = hidden_slots.grad_student_hidden
        if hidden_slots.teacher:
            ctx.reduce_slot_set(1, hidden_slots.grad_teacher_hidden, stream=stream)
            res.grad_teacher_hidden = hidden_slots.grad_teacher_hidden
        # the slot buffers are read; the next step's GEMMs may write them
        dist.all_reduce(hidden_slots._token, group=group)
        return res
    dist.all_reduce(res.grad_student_hidden, group=group)
    if res.grad_teacher_hidden is not None:
        dist.all_reduce(res.grad_teacher_hidden, group=group)
    return res
