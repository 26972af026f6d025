"""The analytic simulator against this framework's measured B200 step times for the
flagship model (1, 2 and 8 GPUs): the predicted step stays within 15 % of the
measurement, and the predicted exposed communication stays below the measured one
(the model counts wire time, not rank skew), so a cost-model change that drifts
away from the hardware fails here."""
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
    assert exposed_ms <= run["exposed_comm_ms"] + 1.0, (exposed_ms, run["exposed_comm_ms"])
