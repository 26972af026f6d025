"""Data: protocols, procedural synthetic source, latent shards, buckets, loader, packing, ingest."""
from avgen_b200.data.bucket import BucketBatch, BucketCurriculum, BucketSampler, CurriculumPhase, largest_remainder
from avgen_b200.data.ingest import (ClipProbe, ClipQA, ClipReport, ClipSpec, IngestSummary, QualityGate,
                                    RejectionReason, build_latent_sample, content_fingerprint, plan_clip_spec,
                                    probe_clip, summarise_reports, tensor_fingerprint)
from avgen_b200.data.loader import (LoaderConfig, LoaderCursor, ShardedLoader, assign_buckets,
                                    bucket_from_descriptor, build_loader)
from avgen_b200.data.packing import PackedLayout, PackPlan, pack_streams, plan_packing, split_packed
from avgen_b200.data.protocols import (DATA_SCHEMA_VERSION, Bucket, BucketPlan, DataSource, LatentSample,
                                       SampleDescriptor, SampleStore, collate_samples)
from avgen_b200.data.shard import (ConcatShardReader, ShardCorruptionError, ShardManifest, ShardReader, ShardRecord,
                                   validate_shard, write_shard)
from avgen_b200.data.synthetic import AlignmentTruth, SyntheticConfig, SyntheticSource
from avgen_b200.data.synthetic_batch import random_batch

__all__ = [
    "DATA_SCHEMA_VERSION", "AlignmentTruth", "Bucket", "BucketBatch", "BucketCurriculum", "BucketPlan",
    "BucketSampler", "ClipProbe", "ClipQA", "ClipReport", "ClipSpec", "ConcatShardReader", "CurriculumPhase",
    "DataSource", "IngestSummary", "LatentSample", "LoaderConfig", "LoaderCursor", "PackPlan", "PackedLayout",
    "QualityGate", "RejectionReason", "SampleDescriptor", "SampleStore", "ShardCorruptionError", "ShardManifest",
    "ShardReader", "ShardRecord", "ShardedLoader", "SyntheticConfig", "SyntheticSource", "assign_buckets",
    "bucket_from_descriptor", "build_latent_sample", "build_loader", "collate_samples", "content_fingerprint",
    "largest_remainder", "pack_streams", "plan_clip_spec", "plan_packing", "probe_clip", "random_batch",
    "split_packed", "summarise_reports", "tensor_fingerprint", "validate_shard", "write_shard",
]

from avgen_b200.data.ingest import iter_clip_table  # noqa: E402

__all__ += ["iter_clip_table"]
