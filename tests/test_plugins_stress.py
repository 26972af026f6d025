"""Entry-point plugins and large fake worlds on CPU.

Plugins: every registry loads third-party components from its entry-point
group once; a plugin that fails to import raises naming the entry point, never
a silently missing component (reference test strategy: tests/test_plugins.py).
Stress: meshes of up to 4096 ranks built on the fake process group give every
rank consistent data / sequence coordinates (reference:
tests/test_distributed_stress.py:60-66)."""
from __future__ import annotations

import math
import multiprocessing as mp
from importlib import metadata

import pytest
import torch

from avgen_b200 import _plugins
from avgen_b200.parallel.dims import ParallelDims


class _FakeEntryPoint:
    def __init__(self, name: str, obj: object = None, error: Exception | None = None) -> None:
        self.name, self.value, self._obj, self._error = name, f"fake:{name}", obj, error

    def load(self) -> object:
        if self._error is not None:
            raise self._error
        return self._obj


def _install(monkeypatch: pytest.MonkeyPatch, group: str, points: list[_FakeEntryPoint]) -> None:
    real = metadata.entry_points

    def fake(**kw):  # noqa: ANN003, ANN202
        if kw.get("group") == group:
            return points
        return real(**kw)

    monkeypatch.setattr(_plugins.metadata, "entry_points", fake)
    _plugins._LOADED.discard(group)  # noqa: SLF001


def test_loader_hands_each_point_once_in_name_order(monkeypatch: pytest.MonkeyPatch) -> None:
    _install(monkeypatch, "avgen.test_group", [_FakeEntryPoint("b", 2), _FakeEntryPoint("a", 1),
                                               _FakeEntryPoint("skipme", 3)])
    seen: list[tuple[str, object]] = []
    n = _plugins.load_entry_points("avgen.test_group", lambda name, obj: seen.append((name, obj)), skip={"skipme"})
    assert n == 2 and seen == [("a", 1), ("b", 2)]
    assert _plugins.load_entry_points("avgen.test_group", lambda *a: seen.append(a)) == 0  # loaded once
    assert _plugins.load_entry_points("avgen.test_group", lambda *a: None, force=True) == 3


def test_failing_plugin_names_the_entry_point(monkeypatch: pytest.MonkeyPatch) -> None:
    _install(monkeypatch, "avgen.test_broken", [_FakeEntryPoint("broken", error=ImportError("no module x"))])
    with pytest.raises(RuntimeError, match="broken"):
        _plugins.load_entry_points("avgen.test_broken", lambda *a: None)


def test_sampler_plugin_is_buildable(monkeypatch: pytest.MonkeyPatch) -> None:
    from avgen_b200.infer import sampler as S

    class Custom(S.EulerSampler):
        pass

    _install(monkeypatch, S.SAMPLER_ENTRY_POINT_GROUP, [_FakeEntryPoint("custom_euler", Custom)])
    assert "custom_euler" in S.list_samplers()
    assert isinstance(S.build_sampler("custom_euler"), Custom)
    S._REGISTRY.pop("custom_euler", None)  # noqa: SLF001
    _install(monkeypatch, S.SAMPLER_ENTRY_POINT_GROUP, [_FakeEntryPoint("bad", 42)])
    with pytest.raises(TypeError, match="callable"):
        S.list_samplers()


def test_reward_plugin_is_buildable(monkeypatch: pytest.MonkeyPatch) -> None:
    from avgen_b200.rl import rewards as R

    class Constant:
        name = "const"

        def score(self, media, prompts):  # noqa: ANN001, ANN201
            return torch.ones(len(prompts))

    _install(monkeypatch, R.REWARD_ENTRY_POINT_GROUP, [_FakeEntryPoint("const_reward", Constant)])
    assert "const_reward" in R.list_rewards()
    r = R.build_reward("const_reward")
    assert r.score(None, ["a", "b"]).tolist() == [1.0, 1.0]
    R._REWARDS.pop("const_reward", None)  # noqa: SLF001


def test_model_plugin_registers(monkeypatch: pytest.MonkeyPatch) -> None:
    from avgen_b200.models import registry

    group = "avgen.models"
    points = list(metadata.entry_points(group=group))
    assert all(hasattr(p, "load") for p in points)  # installed plugins, if any, expose load()
    assert "video_dit" in registry.list_models()
    assert group in _plugins.ENTRY_POINT_GROUPS


# ----------------------------------------------------------------------------- large fake worlds


def _probe(world: int, kw: dict, ranks: list[int]) -> list[tuple]:
    from avgen_b200.simulate.world import fake_world

    dims = ParallelDims(world_size=world, **kw)
    out = []
    for rank in ranks:
        with fake_world(dims, rank=rank, device_type="cpu") as w:
            mesh = w.mesh
            out.append((rank, tuple(mesh.shape), dims.data_coordinates(mesh), dims.sequence_coordinates(mesh)))
    return out


@pytest.mark.parametrize("world,kw", [
    (2048, {"dp_replicate": 16, "context": 8, "tensor": 4}),
    (4096, {"dp_replicate": 32, "context": 8, "tensor": 8}),
    (4096, {"dp_replicate": 4, "dp_shard": 16, "context": 8, "tensor": 8}),
])
def test_fake_world_coordinates_at_scale(world: int, kw: dict) -> None:
    dims = ParallelDims(world_size=world, **kw)
    tp, cp = dims.tensor, dims.context
    # first, last, and a rank with its tp and cp neighbours
    base = world // 2 + 3 * tp
    ranks = [0, world - 1, base, base + 1, base + tp]
    ctx = mp.get_context("spawn")
    with ctx.Pool(1) as pool:
        rows = pool.apply(_probe, (world, kw, ranks))
    by_rank = {r: (shape, data, seq) for r, shape, data, seq in rows}
    for r, (shape, (d, dw), (s, sw)) in by_rank.items():
        assert math.prod(shape) == world
        assert dw == dims.dp_replicate * dims.dp_shard and 0 <= d < dw
        assert sw == cp and 0 <= s < sw
    assert by_rank[0][1][0] == 0 and by_rank[world - 1][1][0] == by_rank[world - 1][1][1] - 1
    # a tp neighbour shares data and sequence shard; a cp neighbour shares data only
    assert by_rank[base][1] == by_rank[base + 1][1] and by_rank[base][2] == by_rank[base + 1][2]
    if (base // tp) % cp + 1 < cp:
        assert by_rank[base][1] == by_rank[base + tp][1] and by_rank[base][2] != by_rank[base + tp][2]
