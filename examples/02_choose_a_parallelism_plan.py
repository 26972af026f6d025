"""Rank parallelism plans for B200 jobs without a GPU.

The simulator prices memory, compute (calibrated to measured B200 GEMM and
attention rates) and communication (NVLink 5 inside a node, InfiniBand between
nodes) for every mesh that divides the world, and keeps the plans that fit in
180 GB with headroom.

    python examples/02_choose_a_parallelism_plan.py
"""
from __future__ import annotations

from avgen_b200.simulate.compute import B200
from avgen_b200.simulate.memory import ModelShape
from avgen_b200.simulate.plan import SearchSpace, render_plan_table, search_parallel_plan


def show(title: str, shape: ModelShape, space: SearchSpace) -> None:
    plans = search_parallel_plan(shape, space, accelerator=B200, top_k=5)
    print(f"== {title}: {len(plans)} plans fit")
    print(render_plan_table(plans, B200))
    print()


def main() -> None:
    two_b = dict(parameters=4_250_000_000, depth=32, width=2560, num_heads=20, text_tokens=512)
    # the benchmark's headline: 64k-token clips on one 8-GPU node
    show("2B-class DiT, 64k tokens, 8 x B200", ModelShape(sequence_length=65536, **two_b),
         SearchSpace(world_size=8, global_batch_size=8))
    # long clips: 131k tokens per sample need the attention ring
    show("14B-class DiT, 131k tokens, 8 x B200",
         ModelShape(parameters=17_000_000_000, depth=40, width=5120, num_heads=40, sequence_length=131072,
                    text_tokens=512, ffn_hidden=13824), SearchSpace(world_size=8, global_batch_size=1))
    # scale out: hybrid sharding keeps the parameter gathers on NVLink
    show("2B-class DiT, 64k tokens, 1024 x B200", ModelShape(sequence_length=65536, **two_b),
         SearchSpace(world_size=1024, global_batch_size=1024))


if __name__ == "__main__":
    main()
