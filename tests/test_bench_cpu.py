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
