"""Data layer on CPU: largest-remainder quotas, curricula, bucket sampling
(disjoint per-rank slices, exact quotas, seeded order), packing layouts and
first-fit packing, shard writing/validation/corruption detection, the
synthetic source's contracts and the ingest quality gate (reference test
strategy: tests/test_data*.py -- quota arithmetic, resume, corruption, QA)."""
from __future__ import annotations

import itertools
import json
from pathlib import Path

import pytest
import torch

from avgen_b200.data import (Bucket, BucketPlan, ConcatShardReader, PackedLayout, SyntheticConfig, SyntheticSource,
                             largest_remainder, plan_packing, validate_shard, write_shard)
from avgen_b200.data.bucket import BucketCurriculum, BucketSampler, CurriculumPhase
from avgen_b200.data.ingest import (ClipProbe, ClipQA, QualityGate, RejectionReason, build_latent_sample,
                                    content_fingerprint, plan_clip_spec, summarise_reports, tensor_fingerprint)
from avgen_b200.data.loader import assign_buckets, bucket_from_descriptor
from avgen_b200.data.packing import split_packed
from avgen_b200.data.shard import ShardCorruptionError, ShardReader

# ----------------------------------------------------------------------------- quotas


@pytest.mark.parametrize("total,weights,expect", [
    (10, [0.5, 0.3, 0.2], (5, 3, 2)), (7, [1, 1, 1], (3, 2, 2)), (0, [1, 2], (0, 0)), (5, [0, 1], (0, 5)),
    (3, [0.2, 0.2, 0.6], (1, 0, 2)), (100, [1, 1, 1], (34, 33, 33)), (1, [3, 3], (1, 0)),
])
def test_largest_remainder_cases(total: int, weights: list[float], expect: tuple[int, ...]) -> None:
    assert largest_remainder(total, weights) == expect


@pytest.mark.parametrize("total", [0, 1, 7, 31, 1000])
@pytest.mark.parametrize("weights", [[1.0], [0.1, 0.9], [3, 1, 1, 5], [0.33, 0.33, 0.34], [1e-3, 1, 1e3]])
def test_largest_remainder_sums_and_is_within_one(total: int, weights: list[float]) -> None:
    q = largest_remainder(total, weights)
    assert sum(q) == total
    s = sum(weights)
    for qi, w in zip(q, weights):
        assert abs(qi - total * w / s) < 1.0


@pytest.mark.parametrize("total,weights", [(-1, [1]), (3, [0, 0]), (3, [1, -1]), (3, [])])
def test_largest_remainder_rejects(total: int, weights: list[float]) -> None:
    with pytest.raises(ValueError):
        largest_remainder(total, weights)


# ----------------------------------------------------------------------------- curricula


def test_curriculum_step_and_interpolated() -> None:
    c = BucketCurriculum((CurriculumPhase(10, (1.0, 0.0)), CurriculumPhase(20, (0.0, 1.0))))
    assert c.weights_at(0) == (1.0, 0.0) and c.weights_at(9) == (1.0, 0.0)
    assert c.weights_at(10) == (0.0, 1.0) and c.weights_at(10_000) == (0.0, 1.0)
    lerp = BucketCurriculum(c.phases, interpolate=True)
    assert lerp.weights_at(5) == (1.0, 0.0)  # inside the first phase nothing blends
    assert lerp.weights_at(15) == pytest.approx((0.5, 0.5))
    assert lerp.bucket_count == 2


@pytest.mark.parametrize("phases", [
    (), (CurriculumPhase(10, (1.0,)), CurriculumPhase(5, (1.0,))),
    (CurriculumPhase(10, (1.0,)), CurriculumPhase(10, (1.0,))),
    (CurriculumPhase(10, (1.0,)), CurriculumPhase(20, (1.0, 1.0))),
])
def test_curriculum_rejects(phases: tuple) -> None:
    with pytest.raises(ValueError):
        BucketCurriculum(phases)


@pytest.mark.parametrize("kw", [{"until_step": 0, "weights": (1.0,)}, {"until_step": 1, "weights": ()},
                                {"until_step": 1, "weights": (0.0, 0.0)}, {"until_step": 1, "weights": (-1.0, 2.0)}])
def test_curriculum_phase_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        CurriculumPhase(**kw)


# ----------------------------------------------------------------------------- bucket sampler


def _plan(mbs: tuple[int, ...] = (2, 2, 1)) -> BucketPlan:
    return BucketPlan(tuple(Bucket(i, 4 * (i + 1), 8, 8, micro_batch_size=m) for i, m in enumerate(mbs)))


@pytest.mark.parametrize("world", [1, 2, 3, 4])
def test_bucket_sampler_ranks_get_disjoint_same_bucket_batches(world: int) -> None:
    plan = _plan()
    assignments = [i % 3 for i in range(60)]
    batches = [BucketSampler(plan, assignments, seed=5, data_rank=r, data_world=world).plan_epoch(epoch=0)
               for r in range(world)]
    seen: list[int] = []
    for rank_batches in batches:
        for b in rank_batches:
            assert all(assignments[i] == b.bucket_id for i in b.indices)
            assert len(b.indices) == plan.get(b.bucket_id).micro_batch_size
            seen += b.indices
    assert len(seen) == len(set(seen))  # no sample twice in one epoch
    counts = [len(b) for b in batches]
    assert len(set(counts)) == 1  # every rank steps the same number of times


def test_bucket_sampler_epochs_differ_and_repeat_with_seed() -> None:
    plan = _plan()
    assignments = [i % 3 for i in range(30)]
    s = BucketSampler(plan, assignments, seed=1)
    e0, e1 = s.plan_epoch(epoch=0), s.plan_epoch(epoch=1)
    assert e0 != e1
    assert e0 == BucketSampler(plan, assignments, seed=1).plan_epoch(epoch=0)
    assert e0 != BucketSampler(plan, assignments, seed=2).plan_epoch(epoch=0)
    assert s.state_dict() == {"seed": 1, "data_rank": 0, "data_world": 1}


def test_bucket_sampler_weights_quotas_and_upsampling() -> None:
    plan = _plan((1, 1, 1))
    assignments = [0] * 10 + [1] * 2 + [2] * 0
    s = BucketSampler(plan, assignments, weights=(0.5, 0.5, 1.0))
    assert s.pool_size(0) == 10 and s.pool_size(1) == 2 and s.pool_size(2) == 0
    assert s.weights_at(0) == (0.5, 0.5, 0.0)  # an empty bucket is never drawn
    assert s.batches_per_epoch() == 12
    assert s.quotas_at(0) == (6, 6, 0)
    epoch = s.plan_epoch(epoch=0)
    per = {b: sum(1 for x in epoch if x.bucket_id == b) for b in (0, 1, 2)}
    assert per == {0: 6, 1: 6, 2: 0}  # the 2-sample bucket is upsampled to honour its weight
    assert s.quotas_at(0, batches=4) == (2, 2, 0)


def test_bucket_sampler_curriculum_and_errors() -> None:
    plan = _plan((1, 1, 1))
    assignments = [i % 3 for i in range(30)]
    cur = BucketCurriculum((CurriculumPhase(5, (1.0, 0.0, 0.0)), CurriculumPhase(10, (0.0, 0.0, 1.0))))
    s = BucketSampler(plan, assignments, curriculum=cur)
    assert {b.bucket_id for b in s.plan_epoch(epoch=0, step=0)} == {0}
    assert {b.bucket_id for b in s.plan_epoch(epoch=0, step=7)} == {2}
    with pytest.raises(ValueError):
        BucketSampler(plan, assignments, curriculum=BucketCurriculum((CurriculumPhase(5, (1.0, 1.0)),)))
    with pytest.raises(ValueError):
        BucketSampler(plan, assignments, data_rank=2, data_world=2)
    assert BucketSampler(plan, assignments, batch_size=3).batch_size == 3


def test_bucket_plan_and_bucket_contracts() -> None:
    plan = _plan()
    assert plan.index_of(2) == 2 and plan.get(1).frames == 8
    with pytest.raises(KeyError):
        plan.get(9)
    with pytest.raises(ValueError):
        BucketPlan(())
    with pytest.raises(ValueError):
        BucketPlan((Bucket(0, 4, 8, 8), Bucket(0, 8, 8, 8)))
    b = Bucket(3, 8, 16, 32, micro_batch_size=2, audio_frames=10, name="wide")
    assert b.video_tokens == 8 * 8 * 16 and b.tokens == b.video_tokens + 10 and b.has_audio
    assert b.aspect_ratio == 2.0 and b.latent_cells == 8 * 16 * 32
    assert b.duration_seconds(timebase_num=8, timebase_den=1) == 1.0
    assert "wide" in b.describe() and "+a10" in b.describe()
    assert plan.token_budget == max(x.tokens * x.micro_batch_size for x in plan.buckets)
    with pytest.raises(ValueError):
        Bucket(0, 4, 7, 8)  # height not divisible by the 2x2 patch
    assert plan.nearest(frames=12, height=8, width=8).bucket_id == 2


# ----------------------------------------------------------------------------- packing


@pytest.mark.parametrize("lengths,capacity", [([5, 3, 7, 2], 10), ([1] * 20, 4), ([10, 10, 10], 10),
                                              ([9, 1, 8, 2, 7, 3], 10), ([3, 3, 3, 3], 7)])
def test_plan_packing_is_a_valid_partition(lengths: list[int], capacity: int) -> None:
    plan = plan_packing(lengths, capacity)
    used = sorted(i for r in plan.rows for i in r.sources)
    assert used == list(range(len(lengths)))
    for r in plan.rows:
        assert r.used <= capacity and r.lengths == tuple(lengths[i] for i in r.sources)
    # first-fit decreasing never needs more than 11/9 OPT + 1 rows; OPT >= ceil(sum / capacity)
    lower = -(-sum(lengths) // capacity)
    assert len(plan.rows) <= 11 * lower // 9 + 1
    assert 0 < plan.occupancy <= 1


def test_plan_packing_limits_segments_and_rejects_long_streams() -> None:
    plan = plan_packing([1] * 10, 100, max_segments=3)
    assert all(r.segment_count <= 3 for r in plan.rows) and len(plan.rows) == 4
    with pytest.raises(ValueError):
        plan_packing([11], 10)
    assert plan.layout_for(0) is plan.rows[0]


@pytest.mark.parametrize("capacity,lengths", [(10, (4, 3)), (8, (8,)), (16, (1, 2, 3, 4)), (5, ())])
def test_packed_layout_views(capacity: int, lengths: tuple[int, ...]) -> None:
    layout = PackedLayout(capacity, lengths)
    ids = layout.segment_ids()
    assert ids.shape == (capacity,)
    assert int((ids >= 0).sum()) == sum(lengths) == layout.used
    cu = layout.cu_seqlens()
    assert cu.tolist() == [0, *itertools.accumulate(lengths)] and cu.dtype == torch.int32
    mask = layout.attention_mask()
    # block diagonal: the mask equals the union of per-segment squares
    ref = torch.zeros(capacity, capacity, dtype=torch.bool)
    for off, n in zip(layout.offsets, lengths):
        ref[off:off + n, off:off + n] = True
    assert torch.equal(mask, ref)
    w = layout.segment_weights()
    assert float(w.sum()) == pytest.approx(len(lengths))
    assert torch.equal(layout.valid_mask(), ids >= 0)
    assert layout.occupancy == pytest.approx(sum(lengths) / capacity)
    packed = torch.arange(capacity).reshape(1, capacity)
    parts = split_packed(packed, layout)
    assert [p.shape[1] for p in parts] == list(lengths)


@pytest.mark.parametrize("kw", [{"capacity": 0, "lengths": ()}, {"capacity": 4, "lengths": (0,)},
                                {"capacity": 4, "lengths": (3, 2)}])
def test_packed_layout_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        PackedLayout(**kw)


# ----------------------------------------------------------------------------- shards


def _samples(n: int, audio: int = 0, seed: int = 0) -> list:
    src = SyntheticSource(SyntheticConfig(seed=seed, num_samples=n, audio_frames=audio, drive_harmonic_gain=0.0))
    return [src.sample(i) for i in range(n)]


def test_shard_write_rules(tmp_path: Path) -> None:
    samples = _samples(3)
    write_shard(tmp_path / "a", samples)
    with pytest.raises(FileExistsError):
        write_shard(tmp_path / "a", samples)
    with pytest.raises(ValueError):
        write_shard(tmp_path / "empty", [])
    with pytest.raises(ValueError, match="duplicate"):
        write_shard(tmp_path / "dup", [samples[0], samples[0]])
    m = validate_shard(tmp_path / "a")
    assert len(m) == 3


def test_shard_reader_round_trip_every_field(tmp_path: Path) -> None:
    samples = _samples(4, audio=32)
    write_shard(tmp_path / "s", samples)
    reader = ShardReader(tmp_path / "s")
    assert len(reader) == 4 and reader.path == tmp_path / "s"
    for i, s in enumerate(samples):
        got = reader[i]
        assert got.descriptor == s.descriptor
        torch.testing.assert_close(got.video, s.video)
        torch.testing.assert_close(got.audio, s.audio)
        torch.testing.assert_close(got.text, s.text)
        assert torch.equal(got.text_mask, s.text_mask)
        assert reader.descriptor(i) == s.descriptor
    reader.close()
    with pytest.raises(RuntimeError):
        reader[0]


def test_shard_detects_flipped_bytes(tmp_path: Path) -> None:
    write_shard(tmp_path / "s", _samples(2))
    validate_shard(tmp_path / "s")
    data = [p for p in (tmp_path / "s").iterdir() if p.suffix in (".safetensors", ".pt", ".bin")]
    assert data, list((tmp_path / "s").iterdir())
    raw = bytearray(data[0].read_bytes())
    raw[-5] ^= 0xFF  # flip bits inside the last tensor's payload
    data[0].write_bytes(bytes(raw))
    with pytest.raises(ShardCorruptionError):
        validate_shard(tmp_path / "s")
    validate_shard(tmp_path / "s", check_data=False)  # manifest-only validation still passes


def test_shard_manifest_corruption_and_newer_schema(tmp_path: Path) -> None:
    write_shard(tmp_path / "s", _samples(2))
    manifests = [p for p in (tmp_path / "s").iterdir() if p.suffix == ".json" and "manifest" in p.name.lower()]
    assert manifests, list((tmp_path / "s").iterdir())
    path = manifests[0]
    doc = json.loads(path.read_text())
    doc["schema_version"] = doc.get("schema_version", 1) + 100
    path.write_text(json.dumps(doc))
    with pytest.raises(ShardCorruptionError, match="newer"):
        validate_shard(tmp_path / "s")
    path.write_text("{not json")
    with pytest.raises(ShardCorruptionError):
        validate_shard(tmp_path / "s")


def test_concat_reader_locates_and_rejects_mixed_codecs(tmp_path: Path) -> None:
    write_shard(tmp_path / "s0", _samples(3))
    write_shard(tmp_path / "s1", _samples(5)[3:])
    store = ConcatShardReader.from_root(tmp_path)
    assert len(store) == 5 and len(store.readers) == 2
    assert store.locate(0) == (0, 0) and store.locate(3) == (1, 0) and store.locate(4) == (1, 1)
    with pytest.raises(IndexError):
        store.locate(5)
    assert store.descriptor(4).sample_id == 4
    with pytest.raises(ValueError):
        ConcatShardReader([])
    other = SyntheticSource(SyntheticConfig(num_samples=1, audio_frames=0, video_codec_id="other-codec"))
    write_shard(tmp_path / "x", [other.sample(0)])
    with pytest.raises(ValueError, match="disagree"):
        ConcatShardReader.from_paths([tmp_path / "s0", tmp_path / "x"])


def test_bucket_assignment_from_descriptors(tmp_path: Path) -> None:
    write_shard(tmp_path / "s", _samples(4))
    store = ConcatShardReader.from_root(tmp_path)
    d = store.descriptor(0)
    plan = BucketPlan((Bucket(0, d.frames, d.height, d.width), Bucket(1, d.frames * 2, d.height, d.width)))
    assert bucket_from_descriptor(d, plan).bucket_id == 0
    assert assign_buckets(store, plan) == (0, 0, 0, 0)
    none = BucketPlan((Bucket(0, d.frames * 2, d.height * 2, d.width * 2),))
    assert bucket_from_descriptor(d, none) is None


# ----------------------------------------------------------------------------- synthetic source


@pytest.mark.parametrize("world", [1, 2, 4])
def test_synthetic_ranks_partition_the_epoch(world: int) -> None:
    cfg = SyntheticConfig(num_samples=16, audio_frames=0)
    ids: list[int] = []
    for r in range(world):
        src = SyntheticSource(cfg, batch_size=2, data_rank=r, data_world=world)
        for batch in itertools.islice(iter(src), 16 // (2 * world)):
            ids += batch.sample_ids.tolist()
    assert sorted(ids) == list(range(16))


def test_synthetic_samples_are_pure_functions_of_seed_and_index() -> None:
    a = SyntheticSource(SyntheticConfig(seed=3, num_samples=4, audio_frames=16, drive_harmonic_gain=0.0))
    b = SyntheticSource(SyntheticConfig(seed=3, num_samples=4, audio_frames=16, drive_harmonic_gain=0.0))
    c = SyntheticSource(SyntheticConfig(seed=4, num_samples=4, audio_frames=16, drive_harmonic_gain=0.0))
    torch.testing.assert_close(a.sample(2).video, b.sample(2).video)
    assert not torch.allclose(a.sample(2).video, c.sample(2).video)
    assert not torch.allclose(a.sample(1).video, a.sample(2).video)
    s = a.sample(0)
    s.validate()
    assert s.video.shape == (4, 8, 8, 8) and s.audio.shape == (2, 16)
    assert a.sample_params(1) == b.sample_params(1)


@pytest.mark.parametrize("kw", [{"num_samples": 0}, {"frames": 0}, {"drive_frequency_hz": 0.0},
                                {"drive_frequency_jitter": 1.0}, {"drive_harmonic_gain": -1.0},
                                {"video_codec_id": ""}, {"audio_frames": -1},
                                {"drive_frequency_hz": 3.0, "video_timebase_num": 8}])
def test_synthetic_config_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        SyntheticConfig(**kw)


def test_synthetic_config_rates() -> None:
    cfg = SyntheticConfig(video_timebase_num=24, audio_timebase_num=48, audio_frames=0)
    assert cfg.video_fps == 24.0 and cfg.audio_fps == 48.0 and not cfg.has_audio
    assert cfg.max_drive_frequency_hz == pytest.approx(0.5 * 1.6 * 2.0)


# ----------------------------------------------------------------------------- ingest


def _probe(**kw) -> ClipProbe:  # noqa: ANN003
    base = dict(path="clip.mp4", width=1280, height=720, frames=240, frame_rate_num=24, frame_rate_den=1,
                duration_seconds=10.0, has_audio=True, audio_sample_rate=48000, audio_rms_dbfs=-20.0,
                fingerprint="")
    base.update(kw)
    return ClipProbe(**base)


@pytest.mark.parametrize("kw,reason", [
    ({"duration_seconds": 0.5}, RejectionReason.TOO_SHORT), ({"duration_seconds": 120.0}, RejectionReason.TOO_LONG),
    ({"width": 200, "height": 200}, RejectionReason.LOW_RESOLUTION),
    ({"width": 3000, "height": 400}, RejectionReason.BAD_ASPECT),
    ({"frame_rate_num": 8}, RejectionReason.LOW_FRAME_RATE),
    ({"audio_rms_dbfs": -90.0}, RejectionReason.SILENT_AUDIO),
])
def test_quality_gate_rejections(kw: dict, reason: RejectionReason) -> None:
    report = QualityGate().evaluate(_probe(**kw))
    assert not report.admitted and reason in report.reasons


def test_quality_gate_audio_requirement_dedup_and_summary() -> None:
    gate = QualityGate(ClipQA(require_audio=True))
    assert RejectionReason.NO_AUDIO in gate.evaluate(_probe(has_audio=False)).reasons
    first = gate.evaluate(_probe(fingerprint="abc"))
    second = gate.evaluate(_probe(fingerprint="abc"))
    assert first.admitted and not second.admitted and second.reasons == (RejectionReason.DUPLICATE,)
    assert gate.admitted == 1
    reports = [first, second, gate.evaluate(_probe(duration_seconds=0.1))]
    summary = summarise_reports(reports)
    assert summary.total == 3 and summary.admitted == 1
    assert summary.rejections == {"duplicate": 1, "too_short": 1}
    assert summary.acceptance_rate == pytest.approx(1 / 3) and "1/3 admitted" in summary.describe()
    gate.reset()
    assert gate.admitted == 0 and gate.evaluate(_probe(fingerprint="abc")).admitted


def test_probe_properties_and_fingerprints() -> None:
    p = _probe(width=720, height=1280, frame_rate_num=30000, frame_rate_den=1001)
    assert p.short_side == 720 and p.aspect_ratio == pytest.approx(0.5625)
    assert p.frame_rate == pytest.approx(29.97, rel=1e-4)
    assert content_fingerprint(b"ab") == content_fingerprint([b"a", b"b"])
    assert content_fingerprint(b"ab") != content_fingerprint(b"ba")
    t = torch.arange(6.0)
    assert tensor_fingerprint(t) == tensor_fingerprint(t.clone())
    assert tensor_fingerprint(t) != tensor_fingerprint(t.reshape(2, 3))  # shape is part of the identity
    assert tensor_fingerprint(t) != tensor_fingerprint(t.double())


@pytest.mark.parametrize("frames,stride,expect_n", [(240, 1, 33), (20, 1, 17), (3, 1, 1), (240, 2, 33), (50, 4, 13)])
def test_plan_clip_spec_frames(frames: int, stride: int, expect_n: int) -> None:
    spec = plan_clip_spec(_probe(frames=frames), frames=33, height=720, width=1280, stride=stride)
    assert spec.frames == expect_n and (spec.frames - 1) % 4 == 0
    assert spec.start_frame >= 0 and spec.start_frame + (spec.frames - 1) * stride < frames
    assert spec.height % 16 == 0 and spec.width % 16 == 0
    assert spec.frame_rate == pytest.approx(24.0 / stride)


def test_build_latent_sample_descriptor() -> None:
    s = build_latent_sample(7, video_latent=torch.zeros(16, 5, 8, 12), text=torch.zeros(3, 32),
                            audio_latent=torch.zeros(8, 40), caption="a cat")
    d = s.descriptor
    assert (d.sample_id, d.channels, d.frames, d.height, d.width) == (7, 16, 5, 8, 12)
    assert (d.audio_channels, d.audio_frames, d.text_tokens, d.text_width) == (8, 40, 3, 32)
    assert d.caption == "a cat" and bool(s.text_mask.all())
    silent = build_latent_sample(8, video_latent=torch.zeros(4, 1, 2, 2), text=torch.zeros(1, 4))
    assert silent.descriptor.audio_frames == 0 and silent.descriptor.audio_channels == 0


def test_synthetic_descriptor_matches_generated_sample() -> None:
    source = SyntheticSource(SyntheticConfig(num_samples=5))
    for i in (0, 4):
        assert source.descriptor(i) == source.sample(i).descriptor
    with pytest.raises(IndexError):
        source.descriptor(5)
    with pytest.raises(IndexError):
        source.descriptor(-1)
