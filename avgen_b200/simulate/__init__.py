"""Capacity planning: memory, compute and communication models, plan search,
fake-world sharding checks and trace capture (avgen/simulate/__init__.py)."""
from avgen_b200.simulate.chakra import TraceArtifacts, capture_execution_trace, capture_with_timing
from avgen_b200.simulate.comms import (ETHERNET_200G, INFINIBAND_NDR, NVLINK4, NVLINK5, CollectiveCost,
                                       CommunicationEstimate, Interconnect, calibrate_from_busbw, count_collectives,
                                       estimate_step_communication)
from avgen_b200.simulate.compute import (A100_80GB, ACCELERATORS, B200, H100_SXM, H200_SXM, Accelerator,
                                         ComputeEstimate, KernelEfficiency, estimate_compute, measure_runtime,
                                         suggest_activation_policy, transformer_flops)
from avgen_b200.simulate.memory import (OPTIMIZER_BYTES, MemoryEstimate, ModelShape, calibration_error,
                                        estimate_memory, measure_memory)
from avgen_b200.simulate.plan import PlanCandidate, SearchSpace, render_plan_table, search_parallel_plan
from avgen_b200.simulate.report import SimulationReport, simulate_config
from avgen_b200.simulate.world import FakeWorld, fake_tensors, fake_world, meta_init, simulate_rank

__all__ = ["A100_80GB", "ACCELERATORS", "B200", "ETHERNET_200G", "H100_SXM", "H200_SXM", "INFINIBAND_NDR", "NVLINK4",
           "NVLINK5", "OPTIMIZER_BYTES", "Accelerator", "CollectiveCost", "CommunicationEstimate", "ComputeEstimate",
           "FakeWorld", "Interconnect", "KernelEfficiency", "MemoryEstimate", "ModelShape", "PlanCandidate",
           "SearchSpace", "SimulationReport", "TraceArtifacts", "calibrate_from_busbw", "calibration_error",
           "capture_execution_trace", "capture_with_timing", "count_collectives", "estimate_compute",
           "estimate_memory", "estimate_step_communication", "fake_tensors", "fake_world", "measure_memory",
           "measure_runtime", "meta_init", "render_plan_table", "search_parallel_plan", "simulate_config",
           "simulate_rank", "suggest_activation_policy", "transformer_flops"]
