"""Core contracts on CPU: patch layouts, patchify / unpatchify as exact inverses
at many geometries, token coordinates, per-pixel reductions, seed mixing and
RNG stream independence / state round trips (reference test strategy:
tests/test_core*.py -- geometry tables, inverse pairs, determinism)."""
from __future__ import annotations

import pytest
import torch

from avgen_b200.core.patchify import (GridPatchifier, build_spatial_coords, build_temporal_coords, patchify_grid,
                                      unpatchify_grid)
from avgen_b200.core.rng import RNGStreams, mix_seed
from avgen_b200.core.tokens import PatchLayout

GEOMETRIES = [
    # frames, height, width, pt, ph, pw, channels
    (1, 2, 2, 1, 2, 2, 1), (4, 8, 8, 1, 2, 2, 16), (8, 16, 32, 2, 2, 2, 4), (3, 6, 9, 1, 3, 3, 2),
    (16, 4, 4, 4, 1, 1, 8), (2, 2, 2, 2, 2, 2, 3), (5, 10, 15, 5, 5, 5, 1),
]


@pytest.mark.parametrize("f,h,w,pt,ph,pw,c", GEOMETRIES)
def test_layout_geometry(f: int, h: int, w: int, pt: int, ph: int, pw: int, c: int) -> None:
    layout = PatchLayout(f, h, w, pt, ph, pw, c)
    assert layout.grid == (f // pt, h // ph, w // pw)
    assert layout.num_tokens == (f // pt) * (h // ph) * (w // pw)
    assert layout.patch_dim == c * pt * ph * pw
    assert layout.num_tokens * layout.patch_dim == c * f * h * w


@pytest.mark.parametrize("f,h,w,pt,ph,pw,c", GEOMETRIES)
def test_patchify_round_trip(f: int, h: int, w: int, pt: int, ph: int, pw: int, c: int) -> None:
    layout = PatchLayout(f, h, w, pt, ph, pw, c)
    grid = torch.randn(2, c, f, h, w, generator=torch.Generator().manual_seed(f * 100 + h))
    tokens = patchify_grid(grid, layout)
    assert tokens.shape == (2, layout.num_tokens, layout.patch_dim)
    assert torch.equal(unpatchify_grid(tokens, layout), grid)


@pytest.mark.parametrize("f,h,w,pt,ph,pw,c", GEOMETRIES)
def test_patchify_token_order_is_frame_row_column(f: int, h: int, w: int, pt: int, ph: int, pw: int, c: int) -> None:
    layout = PatchLayout(f, h, w, pt, ph, pw, c)
    gf, gh, gw = layout.grid
    # encode each cell's patch-grid coordinate in the value and check where it lands
    t_idx = torch.arange(f)[:, None, None] // pt
    r_idx = torch.arange(h)[None, :, None] // ph
    c_idx = torch.arange(w)[None, None, :] // pw
    code = (t_idx * gh * gw + r_idx * gw + c_idx).float()
    grid = code.expand(1, c, f, h, w).contiguous()
    tokens = patchify_grid(grid, layout)
    expect = torch.arange(layout.num_tokens, dtype=torch.float32)[:, None].expand(-1, layout.patch_dim)
    assert torch.equal(tokens[0], expect)


@pytest.mark.parametrize("kw", [{"frames": 0, "height": 2, "width": 2}, {"frames": 3, "height": 2, "width": 2,
                                                                          "patch_frames": 2},
                                {"frames": 2, "height": 3, "width": 2}, {"frames": 2, "height": 2, "width": 2,
                                                                         "channels": 0}])
def test_layout_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        PatchLayout(**kw)


def test_layout_temporal_and_empty() -> None:
    t = PatchLayout.temporal(12, 8, patch_frames=3)
    assert t.grid == (4, 1, 1) and t.patch_dim == 24 and t.is_temporal_only()
    e = PatchLayout.empty()
    assert e.num_tokens == 1 and e.patch_dim == 1


def test_patchify_rejects_wrong_shapes() -> None:
    layout = PatchLayout(2, 4, 4, 1, 2, 2, 3)
    with pytest.raises(ValueError):
        patchify_grid(torch.zeros(1, 3, 2, 4, 6), layout)
    with pytest.raises(ValueError):
        unpatchify_grid(torch.zeros(1, 5, 12), layout)


@pytest.mark.parametrize("normalize", [False, True])
def test_temporal_coords(normalize: bool) -> None:
    layout = PatchLayout(4, 4, 6, 2, 2, 2, 1)
    positions = torch.tensor([[0.0, 0.5, 1.0, 1.5], [10.0, 10.0, 11.0, 11.0]])
    coords = build_temporal_coords(positions, layout, normalize_space=normalize)
    assert coords.shape == (2, layout.num_tokens, 3) and coords.dtype == torch.float32
    grid = coords.reshape(2, 2, 2, 3, 3)
    # time is the mean of each patch's frames
    torch.testing.assert_close(grid[0, :, 0, 0, 0], torch.tensor([0.25, 1.25]))
    torch.testing.assert_close(grid[1, :, 0, 0, 0], torch.tensor([10.0, 11.0]))
    rows, cols = grid[0, 0, :, 0, 1], grid[0, 0, 0, :, 2]
    if normalize:
        torch.testing.assert_close(rows, torch.tensor([0.0, 1.0]))
        torch.testing.assert_close(cols, torch.tensor([0.0, 0.5, 1.0]))
    else:
        torch.testing.assert_close(rows, torch.tensor([0.0, 2.0]))
        torch.testing.assert_close(cols, torch.tensor([0.0, 2.0, 4.0]))
    with pytest.raises(ValueError):
        build_temporal_coords(positions[:, :3], layout)


@pytest.mark.parametrize("fps,start", [(8.0, 0.0), (24.0, 2.5), (0.5, 0.0)])
def test_spatial_coords_follow_the_frame_rate(fps: float, start: float) -> None:
    layout = PatchLayout(4, 2, 2, 1, 2, 2, 1)
    coords = build_spatial_coords(layout, batch=3, fps=fps, start_seconds=start)
    torch.testing.assert_close(coords[0, :, 0], start + torch.arange(4.0) / fps)
    assert torch.equal(coords[0], coords[2])
    with pytest.raises(ValueError):
        build_spatial_coords(layout, batch=1, fps=0.0)


def test_grid_patchifier_reductions() -> None:
    p = GridPatchifier(patch_frames=1, patch_height=2, patch_width=2)
    b, c, f, h, w = 2, 3, 2, 4, 4
    grid = torch.randn(b, c, f, h, w)
    mask = torch.zeros(b, f, h, w, dtype=torch.bool)
    mask[:, :, 0, 0] = True  # one valid pixel in the first patch of each frame row
    cond = torch.ones(b, f, h, w, dtype=torch.bool)
    cond[:, 0, 0, 0] = False  # not every pixel of token 0 is conditioned
    noise = torch.arange(b * f * h * w, dtype=torch.float32).reshape(b, f, h, w)
    stream = p.to_tokens(grid, positions=torch.zeros(b, f), mask=mask, noise_level=noise, conditioned=cond)
    assert stream.tokens.shape == (b, f * 4, c * 4)
    assert stream.mask[:, 0].all() and not stream.mask[:, 1].any()
    assert not stream.conditioned[:, 0].any() and stream.conditioned[:, 1].all()
    # per-token noise is the patch mean of the per-pixel levels
    torch.testing.assert_close(stream.noise_level[0, 0], noise[0, 0, :2, :2].mean())
    assert torch.equal(p.to_grid(stream), grid)
    scalar = p.to_tokens(grid, positions=torch.zeros(b, f), mask=mask, noise_level=torch.tensor([0.1, 0.2]))
    assert scalar.noise_level.shape == (b,) and not scalar.conditioned.any()
    with pytest.raises(ValueError):
        p.layout_for((1, 2, 3))
    with pytest.raises(ValueError):
        p.to_tokens(grid, positions=torch.zeros(b, f), mask=mask[:, :1], noise_level=torch.zeros(b))


# ----------------------------------------------------------------------------- seeds and streams


@pytest.mark.parametrize("seed", [0, 1, 2**31, 2**62])
def test_mix_seed_is_deterministic_and_in_range(seed: int) -> None:
    a = mix_seed(seed, "noise", 3)
    assert a == mix_seed(seed, "noise", 3)
    assert 0 <= a < 2**63
    assert a != mix_seed(seed, "noise", 4) and a != mix_seed(seed, "timestep", 3) and a != mix_seed(seed + 1, "noise", 3)


def test_mix_seed_has_no_easy_collisions() -> None:
    seen = {mix_seed(s, r) for s in range(64) for r in range(64)}
    assert len(seen) == 64 * 64
    assert mix_seed(1, "ab") != mix_seed(1, "ba") and mix_seed(1, 2, 3) != mix_seed(1, 3, 2)


def test_rng_streams_are_independent_and_restorable() -> None:
    a = RNGStreams.from_seed(7)
    draws = {n: torch.rand(4, generator=getattr(a, n)) for n in RNGStreams.NAMES}
    for x, y in [(x, y) for x in RNGStreams.NAMES for y in RNGStreams.NAMES if x < y]:
        assert not torch.equal(draws[x], draws[y])
    state = a.state_dict()
    nxt = torch.rand(4, generator=a.noise)
    b = RNGStreams.from_seed(99)
    b.load_state_dict(state)
    assert torch.equal(torch.rand(4, generator=b.noise), nxt)
    with pytest.raises(ValueError):
        b.load_state_dict({"noise": state["noise"]})
    with pytest.raises(TypeError):
        b.load_state_dict({**state, "noise": state["noise"].float()})


@pytest.mark.parametrize("rank", [0, 1, 5])
def test_rng_for_rank_differs_per_rank_and_matches_across_calls(rank: int) -> None:
    a = RNGStreams.for_rank(3, data_rank=rank)
    b = RNGStreams.for_rank(3, data_rank=rank)
    c = RNGStreams.for_rank(3, data_rank=rank + 1)
    x = torch.rand(3, generator=a.timestep)
    assert torch.equal(x, torch.rand(3, generator=b.timestep))
    assert not torch.equal(x, torch.rand(3, generator=c.timestep))


def test_rng_fork_seed_for_and_validation() -> None:
    a = RNGStreams.from_seed(1)
    g1 = a.fork("dropout")
    g2 = a.fork("dropout")  # the noise stream advanced in between
    assert not torch.equal(torch.rand(2, generator=g1), torch.rand(2, generator=g2))
    s1, s2 = a.seed_for("kernel"), a.seed_for("kernel")
    assert s1 != s2 and 0 <= s1 < 2**63
    a.validate()
    for bad in (-1, True, 1.5):
        with pytest.raises(ValueError):
            RNGStreams.from_seed(bad)  # type: ignore[arg-type]
    with pytest.raises(ValueError):
        RNGStreams.for_rank(0, data_rank=-1)


def test_collective_timeout_restores_the_groups_own_timeout(monkeypatch: pytest.MonkeyPatch) -> None:
    """A temporary bound is undone to the timeout the group was created with, not to the library default."""
    from datetime import timedelta

    import torch.distributed as dist

    from avgen_b200.parallel import env

    calls: list[timedelta] = []
    c10d = dist.distributed_c10d
    monkeypatch.setattr(dist, "is_initialized", lambda: True)
    monkeypatch.setattr(c10d, "_get_default_group", lambda: "group")
    monkeypatch.setattr(c10d, "_set_pg_timeout", lambda t, g: calls.append(t))
    monkeypatch.setattr(env, "_group_timeout", timedelta(seconds=77))
    with env.collective_timeout(5):
        assert calls == [timedelta(seconds=5)]
    assert calls[-1] == timedelta(seconds=77)
