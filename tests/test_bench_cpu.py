"""Host-side helpers of bench.py (no GPU)."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
import bench  # noqa: E402


@pytest.mark.parametrize("speeds", [[1.0] * 8, [1.0, 1.2, 0.9, 1.1, 1.0, 0.95, 1.05, 1.3], [2.0, 1.0], [1.0]])
def test_balanced_rows_sum_bounds_and_order(speeds):
    bt, world = 8192, len(speeds)
    rows = bench.balanced_rows(bt * world, speeds, 16, bt - bt // 4, bt + bt // 4)
    assert sum(rows) == bt * world
    assert all(r % 16 == 0 and bt - bt // 4 <= r <= bt + bt // 4 for r in rows)
    # faster ranks never get fewer rows than slower ones
    for i in range(world):
        for j in range(world):
            if speeds[i] > speeds[j]:
                assert rows[i] >= rows[j]
    if len(set(speeds)) == 1:
        assert rows == [bt] * world


def test_balanced_rows_proportional_when_unclamped():
    rows = bench.balanced_rows(16384, [1.0, 1.25], 16, 6144, 10240)
    assert abs(rows[1] / rows[0] - 1.25) < 0.01


class _Ev:
    """A recorded CUDA event stand-in: a time stamp in ms."""

    def __init__(self, t):
        self.t = t

    def synchronize(self):
        pass

    def elapsed_time(self, end):
        return end.t - self.t


class _SimDist:
    """all_gather_object over simulated ranks: every rank's measured rows/ms
    for the step being gathered."""

    def __init__(self):
        self.values = None

    def all_gather_object(self, out, mine, group=None):
        out[:] = self.values


def test_row_balancer_converges_to_speed_proportional_rows():
    """Ranks whose GPUs run at different speeds: the feedback controller moves
    to rows proportional to speed (within one 256-row quantum), keeps the
    global batch and the bounds, and stays there."""
    world, per, q = 4, 8192, 256
    speed = [1.00, 0.90, 1.12, 0.85]  # rows per ms relative
    sim = _SimDist()
    bals = [bench.RowBalancer(sim, None, world, r, per, q, per - per // 4, per + per // 4) for r in range(world)]
    t = 0.0
    hist = []
    for step in range(30):
        rows = bals[0].rows
        assert all(b.rows == rows for b in bals)  # every rank computes the same allocation
        assert sum(rows) == per * world and all(x % q == 0 for x in rows)
        dur = [rows[r] / (speed[r] * 350.0) for r in range(world)]  # ms
        # each rank records its step; the gather of a lagged step sees every
        # rank's rows/ms of that step
        hist.append([rows[r] / dur[r] for r in range(world)])
        if len(hist) > bals[0].lag:
            sim.values = hist[len(hist) - 1 - bals[0].lag]
        for r, b in enumerate(bals):
            b.record(_Ev(t), _Ev(t + dur[r]), rows[r])
        t += max(dur) + 1.0
    want = [per * world * s / sum(speed) for s in speed]
    assert all(abs(x - w) <= q for x, w in zip(bals[0].rows, want)), (bals[0].rows, want)
    steps = [max(r / s for r, s in zip(rows_, speed)) for rows_ in bals[0].history[-5:]]
    assert max(steps) / min(steps) < 1.01  # settled

