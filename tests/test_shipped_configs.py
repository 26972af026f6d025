"""The YAML configs shipped under ``configs/`` (counterpart of the reference's
``configs/`` tree): every fragment parses, every complete run validates, its
parallel degrees resolve on the world size it is written for, GPU-sized models
keep the head dim the sm_100a attention kernels take, the simulator predicts each
GPU run fits a B200, and the CPU smoke run trains end to end."""
from __future__ import annotations

import json
from pathlib import Path

import pytest

from avgen_b200.cli.main import main
from avgen_b200.config import load_config
from avgen_b200.config.loader import load_mapping
from avgen_b200.config.resolve import build_parallel_dims, gradient_accumulation

ROOT = Path(__file__).resolve().parents[1] / "configs"
FRAGMENT_DIRS = ("model", "data", "eval")
RUN_DIRS = ("train", "finetune", "rl")
# complete run -> the world size it is written for
WORLD = {"train/smoke_cpu.yaml": 1, "train/single_gpu.yaml": 1, "train/node_8gpu.yaml": 8,
         "train/node_8gpu_tp8.yaml": 8, "train/long_context_14b.yaml": 8, "train/multinode_64.yaml": 64,
         "train/multinode_512.yaml": 512, "train/multinode_1024.yaml": 1024, "finetune/lora.yaml": 8,
         "finetune/full.yaml": 8, "finetune/control.yaml": 8, "rl/grpo.yaml": 8, "rl/dpo.yaml": 8}
# values a user must supply for a run to validate
REQUIRED = ["data.root=/data/shards", "finetune.base_checkpoint=/ckpt/export", "rl.prompts_file=/data/prompts.txt"]


def _runs() -> list[str]:
    return sorted(str(p.relative_to(ROOT)) for d in RUN_DIRS for p in (ROOT / d).glob("*.yaml"))


def test_every_shipped_run_is_listed() -> None:
    assert set(_runs()) == set(WORLD)


@pytest.mark.parametrize("path", sorted(str(p.relative_to(ROOT)) for d in FRAGMENT_DIRS
                                        for p in (ROOT / d).glob("*.yaml")))
def test_fragments_parse_and_set_only_their_sections(path: str) -> None:
    mapping = load_mapping(ROOT / path)
    assert mapping and set(mapping) <= {"model", "data", "eval"}
    # a fragment composes into a complete, valid run on its own (defaults elsewhere)
    load_config(mapping=mapping, overrides=["data.root=/data/shards"])


@pytest.mark.parametrize("path", sorted(WORLD))
def test_complete_runs_validate_and_resolve(path: str) -> None:
    config = load_config(ROOT / path, REQUIRED)
    world = WORLD[path]
    dims = build_parallel_dims(config, world_size=world)
    assert dims.world_size == world
    accumulation = gradient_accumulation(config, world_size=world)
    assert accumulation >= 1
    if world > 1:
        # sharding and context parallelism stay inside one NVLink domain
        assert dims.tensor * dims.context * (dims.dp_shard if dims.dp_replicate > 1 else 1) <= config.parallel.gpus_per_node
    if config.parallel.precision.param_dtype == "bfloat16":
        assert config.model.width // config.model.num_heads == 128, "sm_100a attention kernels take head dim 128"


def test_headline_run_is_the_benchmark_configuration() -> None:
    config = load_config(ROOT / "train/node_8gpu.yaml", REQUIRED)
    m = config.model
    assert (m.depth, m.width, m.num_heads, m.mlp_ratio, m.ffn) == (32, 2560, 20, 4, "swiglu")
    assert (config.data.text_tokens, config.data.text_width) == (512, 4096)
    assert config.data.largest_bucket().tokens(m) == 65536
    dims = build_parallel_dims(config, world_size=8)
    assert (dims.dp_shard, dims.context, dims.tensor) == (2, 4, 1) and config.train.global_batch_size == 8
    big = load_config(ROOT / "train/long_context_14b.yaml", REQUIRED)
    assert big.data.largest_bucket().tokens(big.model) == 131072 and big.model.extra["ffn_hidden"] == 13824
    tp = load_config(ROOT / "train/node_8gpu_tp8.yaml", REQUIRED)
    assert tp.parallel.tensor == 8 and tp.data.largest_bucket().tokens(tp.model) == 32768


@pytest.mark.parametrize("path", ["train/node_8gpu.yaml", "train/node_8gpu_tp8.yaml", "train/long_context_14b.yaml",
                                  "finetune/lora.yaml"])
def test_simulator_predicts_gpu_runs_fit_a_b200(path: str, capsys: pytest.CaptureFixture[str]) -> None:
    assert main(["simulate", "--json", "--gpu", "b200", "--world-size", str(WORLD[path]), "--config",
                 str(ROOT / path), *REQUIRED]) == 0
    report = json.loads(capsys.readouterr().out)
    assert report["fits"], report


def test_smoke_cpu_config_trains(tmp_path: Path) -> None:
    out = tmp_path / "smoke"
    assert main(["train", "--config", str(ROOT / "train/smoke_cpu.yaml"), "train.steps=2", "train.warmup_steps=1",
                 f"output_dir={out}",
                 "telemetry.loggers=[jsonl]", "telemetry.log_every=1"]) == 0
    assert (out / "config.yaml").is_file()
    lines = (out / "metrics.jsonl").read_text().splitlines()
    assert len(lines) == 2
