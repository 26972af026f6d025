"""Data layer: synthetic source determinism and sharding, shards, buckets, loader, packing."""
from __future__ import annotations

import torch

from avgen_b200.data import (Bucket, BucketPlan, ConcatShardReader, LoaderConfig, PackedLayout, ShardedLoader,
                             SyntheticConfig, SyntheticSource, largest_remainder, plan_packing, validate_shard,
                             write_shard)


def test_synthetic_deterministic_disjoint_and_aligned() -> None:
    cfg = SyntheticConfig(num_samples=16, audio_frames=32, drive_harmonic_gain=0.0)
    a = SyntheticSource(cfg, batch_size=2, data_rank=0, data_world=2)
    b = SyntheticSource(cfg, batch_size=2, data_rank=1, data_world=2)
    ba, bb = next(iter(a)), next(iter(b))
    assert set(ba.sample_ids.tolist()).isdisjoint(bb.sample_ids.tolist())
    again = next(iter(SyntheticSource(cfg, batch_size=2, data_rank=0, data_world=2)))
    torch.testing.assert_close(ba.video, again.video)
    truth = a.alignment_truth()
    assert float(truth.correlation(ba).min()) > 0.9
    ba.validate()


def test_synthetic_resume() -> None:
    src = SyntheticSource(SyntheticConfig(num_samples=8, audio_frames=0), batch_size=2)
    it = iter(src)
    next(it)
    state = src.state_dict()
    want = next(it).sample_ids
    other = SyntheticSource(SyntheticConfig(num_samples=8, audio_frames=0), batch_size=2)
    other.load_state_dict(state)
    assert torch.equal(next(iter(other)).sample_ids, want)


def test_shard_roundtrip_and_corruption(tmp_path) -> None:
    src = SyntheticSource(SyntheticConfig(num_samples=6, audio_frames=32, drive_harmonic_gain=0.0))
    samples = [src.sample(i) for i in range(6)]
    write_shard(tmp_path / "s0", samples[:3])
    write_shard(tmp_path / "s1", samples[3:])
    validate_shard(tmp_path / "s0")
    store = ConcatShardReader.from_root(tmp_path)
    assert len(store) == 6
    torch.testing.assert_close(store[4].video, samples[4].video)
    (tmp_path / "s1" / "COMMIT").unlink()
    try:
        validate_shard(tmp_path / "s1")
        raise AssertionError("an uncommitted shard must not validate")
    except RuntimeError:
        pass


def test_loader_quota_and_resume(tmp_path) -> None:
    src = SyntheticSource(SyntheticConfig(num_samples=12, audio_frames=0))
    write_shard(tmp_path / "s", [src.sample(i) for i in range(12)])
    store = ConcatShardReader.from_root(tmp_path)
    plan = BucketPlan((Bucket(0, 8, 8, 8, micro_batch_size=2),))
    loader = ShardedLoader(store, plan, config=LoaderConfig(prefetch_batches=2, pin_memory=False), data_world=1)
    it = iter(loader)
    first = [next(it).sample_ids.tolist() for _ in range(2)]
    state = loader.state_dict()
    third = next(it).sample_ids.tolist()
    loader.close()
    resumed = ShardedLoader(store, plan, config=LoaderConfig(prefetch_batches=0, pin_memory=False))
    resumed.load_state_dict(state)
    assert next(iter(resumed)).sample_ids.tolist() == third
    assert first[0] != first[1]
    assert largest_remainder(10, [0.5, 0.3, 0.2]) == (5, 3, 2)
    assert sum(largest_remainder(7, [1, 1, 1])) == 7


def test_packing_layout() -> None:
    plan = plan_packing([5, 3, 7, 2], capacity=10)
    assert all(r.used <= 10 for r in plan.rows)
    layout = PackedLayout(10, (4, 3))
    assert layout.cu_seqlens().tolist() == [0, 4, 7]
    mask = layout.attention_mask()
    assert bool(mask[0, 3]) and not bool(mask[0, 4]) and not bool(mask[8, 8])
    assert abs(float(layout.segment_weights().sum()) - 2.0) < 1e-6
