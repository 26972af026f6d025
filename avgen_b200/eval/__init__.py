"""Evaluation: running metrics over generated media, prompt sharding, exact
cross-rank merging and pinned, comparable reports (avgen/eval/__init__.py API)."""
from avgen_b200.eval import av, conditional, video  # noqa: F401  (registers the built-in metrics)
from avgen_b200.eval.av import AudioBandwidth, AudioSilence, AVSyncProxy
from avgen_b200.eval.conditional import FirstFrameFidelity, InpaintBoundaryConsistency, SeamContinuity
from avgen_b200.eval.learned import (LearnedMetricSpec, MissingBackendError, available_learned_metrics,
                                     build_learned_metric, describe_learned_metrics, frechet_distance,
                                     learned_metric_available, learned_metric_summary, list_learned_metrics,
                                     merge_feature_banks, register_learned_metric, require_backend)
from avgen_b200.eval.protocols import (Metric, MetricError, RunningMetric, build_metric, describe_metrics,
                                       list_metrics, metric_class, register_metric, require_audio, require_video)
from avgen_b200.eval.report import (REPORT_VERSION, EvalPin, EvalReport, IncomparableReports, capture_environment,
                                    compare_reports, format_comparison, prompt_set_digest)
from avgen_b200.eval.suite import (DEFAULT_PROMPTS, EvalBatch, MetricBundle, build_metrics, run_eval_suite,
                                   shard_prompts, torch_gather)
from avgen_b200.eval.video import (FlickerIndex, MotionMagnitude, SaturationClipping, SharpnessProxy,
                                   StaticFrameRatio, TemporalConsistency)

__all__ = ["AVSyncProxy", "AudioBandwidth", "AudioSilence", "DEFAULT_PROMPTS", "EvalBatch", "EvalPin", "EvalReport",
           "FirstFrameFidelity", "FlickerIndex", "IncomparableReports", "InpaintBoundaryConsistency",
           "LearnedMetricSpec", "Metric", "MetricBundle", "MetricError", "MissingBackendError", "MotionMagnitude",
           "REPORT_VERSION", "RunningMetric", "SaturationClipping", "SeamContinuity", "SharpnessProxy",
           "StaticFrameRatio", "TemporalConsistency", "available_learned_metrics", "build_learned_metric",
           "build_metric", "build_metrics", "capture_environment", "compare_reports", "describe_learned_metrics",
           "describe_metrics", "format_comparison", "frechet_distance", "learned_metric_available",
           "learned_metric_summary", "list_learned_metrics", "list_metrics", "merge_feature_banks", "metric_class",
           "prompt_set_digest", "register_learned_metric", "register_metric", "require_audio", "require_backend",
           "require_video", "run_eval_suite", "shard_prompts", "torch_gather"]
