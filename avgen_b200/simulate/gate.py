"""Simulator regression gate over pinned parallelism plans
(.github/scripts/check_reference_plans.py role in the reference).

    python -m avgen_b200.simulate.gate [--plans PATH] [--update] [--json]

For each pinned plan: predicted MFU above its floor, per-rank memory below its
cap, scaling efficiency above its floor (when given), and the real device mesh
built at the plan's full world size on the fake process group with the mesh
dimension order (pp, dp_replicate, dp_shard, cp, tp). ``--update`` rewrites the
``observed`` values in the plans file. Exit code 1 on any violation.
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import sys
from pathlib import Path
from typing import Any

__all__ = ["DEFAULT_PLANS", "check_plan", "check_plans", "main"]

DEFAULT_PLANS = Path(__file__).with_name("reference_plans.json")
_ORDER = ("pp", "dp_replicate", "dp_shard", "cp", "tp")


def _mesh_names(dims_kwargs: dict[str, int], world: int) -> tuple[str, ...]:
    from avgen_b200.parallel.dims import ParallelDims
    from avgen_b200.simulate.world import fake_world

    with fake_world(ParallelDims(world_size=world, **dims_kwargs), device_type="cpu") as w:
        return tuple(w.mesh.mesh_dim_names or ()) if w.mesh is not None else ()


def _mesh_names_isolated(dims_kwargs: dict[str, int], world: int) -> tuple[str, ...]:
    """Build the mesh in a child process (the fake process group is process-global)."""
    ctx = mp.get_context("spawn")
    with ctx.Pool(1) as pool:
        return pool.apply(_mesh_names, (dims_kwargs, world))


def check_plan(plan: dict[str, Any], models: dict[str, Any], defaults: dict[str, Any], *,
               build_mesh: bool = True) -> tuple[dict[str, float], list[str]]:
    from avgen_b200.parallel.dims import ParallelDims
    from avgen_b200.simulate import ACCELERATORS, ModelShape, simulate_config

    shape = ModelShape(**models[plan["model"]])
    world = int(plan.get("world_size", 8))
    dims_kwargs = {k: int(v) for k, v in plan.get("dims", {}).items()}
    others = 1
    for k in ("dp_replicate", "tensor", "context", "pipeline"):
        others *= dims_kwargs.get(k, 1)
    if "dp_shard" not in dims_kwargs:
        dims_kwargs["dp_shard"] = world // others
    dims = ParallelDims(world_size=world, **dims_kwargs)
    acc = ACCELERATORS[defaults.get("accelerator", "b200")]
    rep = simulate_config(shape, dims, accelerator=acc)
    observed = {"mfu": round(rep.mfu, 4), "memory_gib": round(rep.memory.total_gib, 2),
                "scaling": round(rep.communication.scaling_efficiency, 4), "step_seconds": round(rep.step_seconds, 4)}
    problems = []
    if observed["mfu"] < plan.get("min_mfu", 0.0):
        problems.append(f"{plan['name']}: MFU {observed['mfu']:.3f} below floor {plan['min_mfu']}")
    if observed["memory_gib"] > plan.get("max_memory_gib", float("inf")):
        problems.append(f"{plan['name']}: {observed['memory_gib']:.1f} GiB per rank above {plan['max_memory_gib']}")
    if observed["scaling"] < plan.get("min_scaling", 0.0):
        problems.append(f"{plan['name']}: scaling {observed['scaling']:.3f} below floor {plan['min_scaling']}")
    if build_mesh:
        names = _mesh_names_isolated(dims_kwargs, world)
        want = tuple(n for n in _ORDER if n in names)
        if names != want:
            problems.append(f"{plan['name']}: mesh order {names} is not {want}")
    return observed, problems


def check_plans(path: str | Path = DEFAULT_PLANS, *, update: bool = False,
                build_mesh: bool = True) -> tuple[dict[str, dict[str, float]], list[str]]:
    spec = json.loads(Path(path).read_text(encoding="utf-8"))
    results: dict[str, dict[str, float]] = {}
    problems: list[str] = []
    for plan in spec["plans"]:
        obs, probs = check_plan(plan, spec["models"], spec.get("defaults", {}), build_mesh=build_mesh)
        results[plan["name"]] = obs
        problems += probs
        if update:
            plan["observed"] = obs
    if update:
        Path(path).write_text(json.dumps(spec, indent=2) + "\n", encoding="utf-8")
    return results, problems


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(prog="python -m avgen_b200.simulate.gate", description=__doc__,
                                formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--plans", default=str(DEFAULT_PLANS))
    p.add_argument("--update", action="store_true")
    p.add_argument("--no-mesh", action="store_true", help="skip building the fake-world meshes")
    p.add_argument("--json", action="store_true")
    a = p.parse_args(argv)
    results, problems = check_plans(a.plans, update=a.update, build_mesh=not a.no_mesh)
    if a.json:
        sys.stdout.write(json.dumps({"results": results, "problems": problems}, indent=2) + "\n")
    else:
        for name, obs in results.items():
            sys.stdout.write(f"{name:22s} mfu {obs['mfu']:.3f}  mem {obs['memory_gib']:7.1f} GiB  "
                             f"scaling {obs['scaling']:.3f}  step {obs['step_seconds']:.3f} s\n")
        for msg in problems:
            sys.stdout.write(f"FAIL {msg}\n")
    return 1 if problems else 0


if __name__ == "__main__":
    raise SystemExit(main())
