"""Rank-sharded, resumable, prefetching loader (avgen/data/loader.py:83-843).

:class:`ShardedLoader` assigns every stored sample to its nearest bucket, plans
epochs with a :class:`~avgen_b200.data.bucket.BucketSampler`, collates batches
into page-locked host memory on a background thread (``prefetch_batches``
ahead) so the trainer's host->device copies are asynchronous, and keeps a
:class:`LoaderCursor` (epoch, batch index, samples seen) that checkpoints and
resumes exactly. ``build_loader`` wires a loader from a run config.
"""
from __future__ import annotations

import queue
import threading
from collections.abc import Iterator, Mapping, Sequence
from dataclasses import dataclass
from typing import Any

import torch

from avgen_b200.core.batch import MediaBatch
from avgen_b200.data.bucket import BucketBatch, BucketCurriculum, BucketSampler
from avgen_b200.data.protocols import Bucket, BucketPlan, SampleDescriptor, SampleStore, collate_samples

__all__ = ["LoaderConfig", "LoaderCursor", "ShardedLoader", "assign_buckets", "bucket_from_descriptor",
           "build_loader"]


def bucket_from_descriptor(desc: SampleDescriptor, plan: BucketPlan) -> Bucket | None:
    """The exact-shape bucket of a sample, else ``None``."""
    for b in plan.buckets:
        if (b.frames, b.height, b.width) == (desc.frames, desc.height, desc.width) and \
                b.audio_frames == desc.audio_frames:
            return b
    return None


def assign_buckets(store: SampleStore, plan: BucketPlan) -> tuple[int, ...]:
    """Bucket id per sample (``-1`` when no bucket has its exact shape)."""
    out = []
    for i in range(len(store)):
        b = bucket_from_descriptor(store.descriptor(i), plan)
        out.append(b.bucket_id if b is not None else -1)
    return tuple(out)


@dataclass(frozen=True, slots=True)
class LoaderConfig:
    seed: int = 0
    prefetch_batches: int = 2
    pin_memory: bool = True
    drop_last: bool = True
    text_tokens: int | None = None

    def __post_init__(self) -> None:
        if self.prefetch_batches < 0:
            raise ValueError("prefetch_batches must be non-negative")


@dataclass
class LoaderCursor:
    epoch: int = 0
    batch_index: int = 0
    samples_seen: int = 0

    def advance(self, samples: int) -> None:
        self.batch_index += 1
        self.samples_seen += samples

    def state_dict(self) -> dict[str, int]:
        return {"epoch": self.epoch, "batch_index": self.batch_index, "samples_seen": self.samples_seen}

    def load_state_dict(self, state: Mapping[str, Any]) -> None:
        self.epoch = int(state["epoch"])
        self.batch_index = int(state["batch_index"])
        self.samples_seen = int(state.get("samples_seen", 0))


_STOP = object()


class ShardedLoader:
    def __init__(self, store: SampleStore, plan: BucketPlan, *, config: LoaderConfig | None = None,
                 data_rank: int = 0, data_world: int = 1, weights: Sequence[float] | None = None,
                 curriculum: BucketCurriculum | None = None) -> None:
        self._store = store
        self._plan = plan
        self._config = config or LoaderConfig()
        self._rank = data_rank
        self._world = data_world
        self._sampler = BucketSampler(plan, assign_buckets(store, plan), weights=weights, curriculum=curriculum,
                                      seed=self._config.seed, data_rank=data_rank, data_world=data_world,
                                      drop_last=self._config.drop_last)
        self._cursor = LoaderCursor()
        self._step = 0
        self._thread: threading.Thread | None = None
        self._stop = threading.Event()

    @property
    def cursor(self) -> LoaderCursor:
        return self._cursor

    @property
    def sampler(self) -> BucketSampler:
        return self._sampler

    @property
    def config(self) -> LoaderConfig:
        return self._config

    @property
    def data_coordinates(self) -> tuple[int, int]:
        return self._rank, self._world

    def set_step(self, step: int) -> None:
        """Curriculum step used when the next epoch is planned."""
        self._step = step

    def set_curriculum(self, stage: object) -> None:  # Trainer hook; weights come from the sampler's curriculum
        del stage

    def batches_per_epoch(self) -> int:
        return self._sampler.batches_per_epoch()

    def epoch_plan(self, epoch: int | None = None) -> tuple[BucketBatch, ...]:
        return self._sampler.plan_epoch(epoch=self._cursor.epoch if epoch is None else epoch, step=self._step)

    def build_batch(self, planned: BucketBatch) -> MediaBatch:
        samples = [self._store[i] for i in planned.indices]
        return collate_samples(samples, bucket_id=planned.bucket_id, text_tokens=self._config.text_tokens,
                               pin=self._config.pin_memory and torch.cuda.is_available())

    def _produce(self, out: queue.Queue) -> None:
        try:
            while not self._stop.is_set():
                plan = self.epoch_plan()
                if not plan:
                    raise RuntimeError("the loader has no batches to produce")
                for i in range(self._cursor.batch_index, len(plan)):
                    if self._stop.is_set():
                        return
                    out.put((self._cursor.epoch, i, self.build_batch(plan[i])))
                self._cursor.epoch += 1
                self._cursor.batch_index = 0
        except BaseException as exc:  # noqa: BLE001 - forwarded to the consumer
            out.put(exc)
        finally:
            out.put(_STOP)

    def __iter__(self) -> Iterator[MediaBatch]:
        if self._config.prefetch_batches == 0:
            while True:
                plan = self.epoch_plan()
                while self._cursor.batch_index < len(plan):
                    batch = self.build_batch(plan[self._cursor.batch_index])
                    self._cursor.advance(batch.spec.batch_size)
                    yield batch
                self._cursor.epoch += 1
                self._cursor.batch_index = 0
        q: queue.Queue = queue.Queue(maxsize=self._config.prefetch_batches)
        start = (self._cursor.epoch, self._cursor.batch_index, self._cursor.samples_seen)
        self._stop.clear()
        self._thread = threading.Thread(target=self._produce, args=(q,), daemon=True, name="avgen-loader")
        self._thread.start()
        self._cursor.epoch, self._cursor.batch_index, self._cursor.samples_seen = start
        try:
            while True:
                item = q.get()
                if item is _STOP:
                    return
                if isinstance(item, BaseException):
                    raise item
                epoch, index, batch = item
                self._cursor.epoch, self._cursor.batch_index = epoch, index
                self._cursor.advance(batch.spec.batch_size)
                yield batch
        finally:
            self.close()

    def close(self) -> None:
        self._stop.set()
        if self._thread is not None and self._thread.is_alive():
            self._thread.join(timeout=5.0)
        self._thread = None

    def state_dict(self) -> dict[str, Any]:
        return {"cursor": self._cursor.state_dict(), "data_rank": self._rank, "data_world": self._world,
                "step": self._step}

    def load_state_dict(self, state: Mapping[str, Any]) -> None:
        if int(state.get("data_world", self._world)) != self._world:
            raise ValueError("cannot resume the loader cursor on a different data_world")
        self._cursor.load_state_dict(state["cursor"])
        self._step = int(state.get("step", 0))


def build_loader(config: Any, *, data_rank: int = 0, data_world: int = 1, batch_size: int | None = None):  # noqa: ANN201
    """A data source for a :class:`~avgen_b200.config.RunConfig`: synthetic or latent shards."""
    data = config.data
    bucket = data.largest_bucket()
    bsz = batch_size or config.micro_batch_size
    if data.source == "synthetic":
        from avgen_b200.data.synthetic import SyntheticConfig, SyntheticSource

        syn = SyntheticConfig(seed=data.seed, num_samples=max(64, bsz * data_world * 4),
                              video_channels=data.latent_channels, frames=bucket.frames, height=bucket.height,
                              width=bucket.width, audio_channels=data.audio_channels, audio_frames=data.audio_frames,
                              text_tokens=data.text_tokens, text_width=data.text_width,
                              video_timebase_num=max(8, bucket.frames), video_timebase_den=1,
                              audio_timebase_num=max(32, data.audio_frames or 32), drive_frequency_hz=0.5,
                              drive_harmonic_gain=0.0 if data.audio_frames else 0.6)
        return SyntheticSource(syn, batch_size=bsz, data_rank=data_rank, data_world=data_world)
    from avgen_b200.data.shard import ConcatShardReader

    store = ConcatShardReader.from_root(data.root)
    model = config.model
    plan = BucketPlan(tuple(Bucket(bucket_id=i, frames=b.frames, height=b.height, width=b.width,
                                   micro_batch_size=bsz, audio_frames=data.audio_frames,
                                   patch_frames=model.patch_frames, patch_height=model.patch_height,
                                   patch_width=model.patch_width, name=b.name)
                            for i, b in enumerate(data.buckets)))
    return ShardedLoader(store, plan, config=LoaderConfig(seed=data.seed, prefetch_batches=data.prefetch_batches,
                                                          text_tokens=data.text_tokens),
                         data_rank=data_rank, data_world=data_world, weights=[b.weight for b in data.buckets])
