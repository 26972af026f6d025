"""Pipeline schedule tables on CPU: the interleaved 1F1B order of every rank holds
each (chunk, micro-batch) forward and backward exactly once with forwards before
their backwards; the lock-step timetable respects every data dependency
(a chunk's forward after the previous chunk's, its backward after the next
chunk's backward), never stalls, and its length shows the bubble shrinking with
more virtual stages (reference test strategy: tests/test_pipeline*.py)."""
from __future__ import annotations

import pytest

from avgen_b200.parallel.pipeline import (PipelineConfig, balanced_split_points, interleaved_order,
                                          interleaved_timetable)

CASES = [(2, 2, 2), (2, 2, 4), (2, 3, 4), (4, 2, 4), (4, 2, 8), (3, 3, 6), (4, 4, 8), (8, 2, 8)]


@pytest.mark.parametrize("p,v,m", CASES)
def test_each_rank_runs_every_action_once(p: int, v: int, m: int) -> None:
    for r in range(p):
        order = interleaved_order(r, p, v, m)
        fwd = [(j, k) for kind, j, k in order if kind == "F"]
        bwd = [(j, k) for kind, j, k in order if kind == "B"]
        want = sorted((j, k) for j in range(v) for k in range(m))
        assert sorted(fwd) == want and sorted(bwd) == want
        seen = set()
        for kind, j, k in order:
            if kind == "B":
                assert (j, k) in seen, f"rank {r}: backward of {(j, k)} before its forward"
            else:
                seen.add((j, k))


@pytest.mark.parametrize("p,v,m", CASES)
def test_timetable_respects_dependencies(p: int, v: int, m: int) -> None:
    table = interleaved_timetable(p, v, m)
    last = p * v - 1
    fwd, bwd = {}, {}
    for t, row in enumerate(table):
        assert len(row) == p and any(a is not None for a in row)
        for r, action in enumerate(row):
            if action is None:
                continue
            kind, j, k = action
            (fwd if kind == "F" else bwd)[(j * p + r, k)] = t
    assert len(fwd) == len(bwd) == p * v * m
    for (g, k), t in fwd.items():
        if g > 0:
            assert fwd[(g - 1, k)] < t
    for (g, k), t in bwd.items():
        assert fwd[(g, k)] < t
        if g < last:
            assert bwd[(g + 1, k)] < t
    # never longer than running the chunks one after another with no overlap at all
    assert len(table) <= 2 * p * v * m


@pytest.mark.parametrize("p,m", [(2, 4), (4, 8), (8, 16)])
def test_more_virtual_stages_shrink_the_relative_bubble(p: int, m: int) -> None:
    def bubble(v: int) -> float:
        ticks = len(interleaved_timetable(p, v, m))
        busy = 2 * m * v  # each rank's own work in ticks
        return (ticks - busy) / busy

    assert bubble(2) < bubble(1)


def test_order_requires_whole_microbatch_groups() -> None:
    with pytest.raises(ValueError, match="multiple"):
        interleaved_order(0, 4, 2, 6)


@pytest.mark.parametrize("blocks,stages", [(4, 4), (8, 4), (32, 8), (40, 16), (12, 5)])
def test_balanced_split_points_cover_and_balance(blocks: int, stages: int) -> None:
    points = balanced_split_points(blocks, stages)
    bounds = [0, *points, blocks]
    sizes = [b - a for a, b in zip(bounds, bounds[1:])]
    assert len(sizes) == stages and all(s >= 1 for s in sizes) and sum(sizes) == blocks
    assert max(sizes) - min(sizes) <= 2  # the ends carry the embeddings and the head
    with pytest.raises(ValueError):
        balanced_split_points(3, 4)


@pytest.mark.parametrize("kw", [{"schedule": "dualpipe"}, {"microbatches": 0}, {"stages_per_rank": 0},
                                {"schedule": "1f1b", "stages_per_rank": 2}])
def test_pipeline_config_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        PipelineConfig(**kw)


def test_pipeline_config_bubble_fraction() -> None:
    assert PipelineConfig(microbatches=8).bubble_fraction(4) == pytest.approx(3 / 11)
    assert PipelineConfig(schedule="interleaved_1f1b", stages_per_rank=2, microbatches=8).bubble_fraction(8) == \
        pytest.approx(3 / 11)
    assert PipelineConfig().bubble_fraction(1) == 0.0
