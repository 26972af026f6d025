"""The analytic simulator against this framework's measured B200 step times for the
flagship model (1, 2 and 8 GPUs): the predicted step stays within 15 % of the
measurement and the predicted exposed communication (wire time the overlap does
not hide plus the ring barriers' wait for the slowest rank) within a factor of
two of the measured one, so a cost-model change that drifts away from the
hardware fails here."""
from __future__ import annotations

import json
from pathlib import Path

import pytest

import avgen_b200.simulate as sim
from avgen_b200.parallel import ParallelDims

MEASURED = json.loads((Path(sim.__file__).parent / "measured_b200.json").read_text())


@pytest.mark.parametrize("run", MEASURED["runs"], ids=lambda r: f"n{r['world_size']}")
def test_simulated_step_tracks_the_measured_step(run: dict) -> None:
    shape = sim.ModelShape(**MEASURED["model"])
    dims = ParallelDims(world_size=run["world_size"], dp_shard=run["dp_shard"], context=run["context"])
    data_parallel = run["dp_shard"]
    accumulation = run["samples_per_step"] // data_parallel
    report = sim.simulate_config(shape, dims, gradient_accumulation=accumulation)
    predicted_ms = report.step_seconds * 1e3
    assert abs(predicted_ms / run["ms_per_step"] - 1.0) < 0.15, (predicted_ms, run["ms_per_step"])
    exposed_ms = report.communication.exposed_seconds * 1e3 * accumulation
    measured = run["exposed_comm_ms"]
    assert measured / 2 - 1.0 <= exposed_ms <= 2 * measured + 1.0, (exposed_ms, measured)


@pytest.mark.parametrize("n,want", [(1, 0.0), (2, 0.5642), (3, 0.8463), (4, 1.0294), (8, 1.4236), (16, 1.7660)])
def test_expected_normal_maximum(n: int, want: float) -> None:
    from avgen_b200.simulate.comms import expected_max_normal

    assert expected_max_normal(n) == pytest.approx(want, abs=2e-4)
