"""Telemetry: loggers, on-device metric accumulation, throughput / MFU, memory, profiling."""
from avgen_b200.telemetry.logger import (ConsoleLogger, JSONLLogger, Logger, MultiLogger, NoOpLogger,
                                         RankGatedLogger, TensorBoardLogger, WandbLogger, build_logger)
from avgen_b200.telemetry.metrics import (MemoryReport, MemoryReporter, MetricAccumulator, ThroughputMeter,
                                          ThroughputReport, merge_metrics)
from avgen_b200.telemetry.profiler import (DeviceTimer, flight_recorder_dump, memory_snapshot, nvtx_range,
                                           profile_steps, should_profile_rank)

__all__ = ["ConsoleLogger", "DeviceTimer", "JSONLLogger", "Logger", "MemoryReport", "MemoryReporter",
           "MetricAccumulator", "MultiLogger", "NoOpLogger", "RankGatedLogger", "TensorBoardLogger",
           "ThroughputMeter", "ThroughputReport", "WandbLogger", "build_logger", "flight_recorder_dump",
           "memory_snapshot", "merge_metrics", "nvtx_range", "profile_steps", "should_profile_rank"]
