"""Run-config schema, loader, resolvers and diffs on CPU: every validation rule
names its dotted field, YAML values are coerced by annotation, and the
resolvers turn a config into the runtime objects the trainer consumes
(reference test strategy: tests/test_config.py -- per-field validation,
coercion, overrides, composition, resolve helpers)."""
from __future__ import annotations

from dataclasses import replace
from pathlib import Path
from typing import Any, Optional

import pytest
import yaml

from avgen_b200.config import load_config
from avgen_b200.config import schema as S
from avgen_b200.config.diff import config_diff, config_to_dict, render_diff, save_config
from avgen_b200.config.loader import (ConfigError, apply_overrides, build_dataclass, coerce, deep_merge, load_mapping,
                                      parse_override)
from avgen_b200.config.resolve import (build_accelerator, build_activation_checkpoint, build_fsdp_config,
                                       build_interconnects, build_model_shape, build_parallel_config,
                                       build_parallel_dims, build_pipeline_config, build_precision_config,
                                       gradient_accumulation, model_kwargs, sequence_length_for)

# ----------------------------------------------------------------------------- section validation


@pytest.mark.parametrize("field,value", [
    ("depth", 0), ("depth", -1), ("width", 0), ("num_heads", 0), ("mlp_ratio", 0), ("patch_frames", 0),
    ("patch_height", 0), ("patch_width", 0), ("in_channels", 0), ("depth", 1.5), ("depth", True),
    ("audio_width", -1), ("parameters", -5), ("rope_theta", 0.0), ("rope_theta", -1.0), ("ffn", "relu"),
    ("out_channels", 0), ("out_channels", -2), ("name", ""),
])
def test_model_config_rejects(field: str, value: Any) -> None:
    with pytest.raises(ValueError) as err:
        S.ModelConfig(**{field: value})
    assert f"model.{field}" in str(err.value)


def test_model_config_heads_must_divide_width() -> None:
    with pytest.raises(ValueError, match="num_heads must divide"):
        S.ModelConfig(width=100, num_heads=3)
    with pytest.raises(TypeError):
        S.ModelConfig(extra=[1, 2])  # type: ignore[arg-type]


@pytest.mark.parametrize("width,heads,head_dim", [(768, 12, 64), (2560, 20, 128), (5120, 40, 128), (64, 1, 64)])
def test_model_config_head_dim(width: int, heads: int, head_dim: int) -> None:
    assert S.ModelConfig(width=width, num_heads=heads).head_dim == head_dim


@pytest.mark.parametrize("out,expect", [(-1, 16), (32, 32), (1, 1)])
def test_model_config_latent_out_channels(out: int, expect: int) -> None:
    assert S.ModelConfig(in_channels=16, out_channels=out).latent_out_channels == expect


@pytest.mark.parametrize("ffn,cross", [("swiglu", True), ("swiglu", False), ("gelu", True), ("gelu", False)])
def test_model_parameter_estimate_orders(ffn: str, cross: bool) -> None:
    small = S.ModelConfig(depth=4, width=256, num_heads=4, ffn=ffn, cross_attention=cross)
    deeper = replace(small, depth=8)
    wider = replace(small, width=512, num_heads=8)
    assert 0 < small.estimated_parameters() < deeper.estimated_parameters()
    assert small.estimated_parameters() < wider.estimated_parameters()
    # width dominates quadratically: doubling width roughly quadruples the block parameters
    assert wider.estimated_parameters() / small.estimated_parameters() > 3.5
    assert replace(small, parameters=123).estimated_parameters() == 123


def test_swiglu_estimate_exceeds_gelu_and_cross_adds_parameters() -> None:
    base = S.ModelConfig(depth=2, width=256, num_heads=4)
    assert base.estimated_parameters() > replace(base, ffn="gelu").estimated_parameters()
    assert base.estimated_parameters() > replace(base, cross_attention=False).estimated_parameters()


def test_model_has_audio() -> None:
    assert not S.ModelConfig().has_audio
    assert S.ModelConfig(audio_width=128).has_audio


@pytest.mark.parametrize("field,value", [("frames", 0), ("height", -1), ("width", 0), ("micro_batch_size", 0),
                                         ("weight", -0.5)])
def test_bucket_config_rejects(field: str, value: Any) -> None:
    with pytest.raises(ValueError) as err:
        S.BucketConfig(name="b0", **{field: value})
    assert "data.buckets[b0]" in str(err.value)


@pytest.mark.parametrize("frames,height,width,pt,ph,pw,tokens", [
    (16, 32, 32, 1, 2, 2, 16 * 16 * 16), (16, 128, 128, 1, 2, 2, 65536), (8, 64, 64, 2, 2, 2, 4 * 32 * 32),
    (1, 2, 2, 1, 2, 2, 1), (4, 4, 8, 4, 4, 4, 2),
])
def test_bucket_tokens(frames: int, height: int, width: int, pt: int, ph: int, pw: int, tokens: int) -> None:
    model = S.ModelConfig(patch_frames=pt, patch_height=ph, patch_width=pw)
    assert S.BucketConfig(frames=frames, height=height, width=width).tokens(model) == tokens


@pytest.mark.parametrize("frames,height,width", [(3, 32, 32), (16, 31, 32), (16, 32, 33)])
def test_bucket_tokens_require_divisible_patches(frames: int, height: int, width: int) -> None:
    model = S.ModelConfig(patch_frames=2, patch_height=2, patch_width=2)
    with pytest.raises(ValueError, match="not divisible"):
        S.BucketConfig(frames=frames, height=height, width=width).tokens(model)


@pytest.mark.parametrize("kw,needle", [
    ({"source": "webdataset"}, "data.source"), ({"num_workers": -1}, "data.num_workers"),
    ({"prefetch_batches": -1}, "data.prefetch_batches"), ({"shuffle_buffer": -2}, "data.shuffle_buffer"),
    ({"repeat": -1}, "data.repeat"), ({"seed": -3}, "data.seed"), ({"audio_frames": -1}, "data.audio_frames"),
    ({"latent_channels": 0}, "data.latent_channels"), ({"text_tokens": 0}, "data.text_tokens"),
    ({"text_width": 0}, "data.text_width"), ({"audio_channels": 0}, "data.audio_channels"),
    ({"caption_dropout": 1.5}, "data.caption_dropout"), ({"caption_dropout": -0.1}, "data.caption_dropout"),
    ({"buckets": ()}, "data.buckets"), ({"buckets": (S.BucketConfig(name="a"), S.BucketConfig(name="a"))},
                                        "duplicates"),
    ({"source": "latent_shards"}, "data.root"),
])
def test_data_config_rejects(kw: dict[str, Any], needle: str) -> None:
    with pytest.raises(ValueError) as err:
        S.DataConfig(**kw)
    assert needle in str(err.value)


def test_data_config_bucket_lookup_and_largest() -> None:
    a, b = S.BucketConfig(name="a", frames=4), S.BucketConfig(name="b", frames=8, height=16, width=64)
    data = S.DataConfig(buckets=(a, b))
    assert data.bucket("b") is b
    assert data.largest_bucket() is b
    with pytest.raises(KeyError, match="no bucket named 'c'"):
        data.bucket("c")
    assert not data.has_audio and S.DataConfig(audio_frames=4).has_audio
    assert S.DataConfig(source="latent_shards", root="/data").root == "/data"


@pytest.mark.parametrize("kw,needle", [
    ({"steps": 0}, "train.steps"), ({"global_batch_size": 0}, "train.global_batch_size"),
    ({"micro_batch_size": 0}, "train.micro_batch_size"), ({"optimizer": "lamb"}, "train.optimizer"),
    ({"schedule": "step"}, "train.schedule"), ({"timestep_sampler": "beta"}, "train.timestep_sampler"),
    ({"lr": 0.0}, "train.lr"), ({"eps": 0.0}, "train.eps"), ({"weight_decay": -1.0}, "train.weight_decay"),
    ({"max_grad_norm": -1.0}, "train.max_grad_norm"), ({"audio_loss_weight": -1.0}, "train.audio_loss_weight"),
    ({"beta1": 1.5}, "train.beta1"), ({"beta2": -0.1}, "train.beta2"), ({"decay_ratio": 2.0}, "train.decay_ratio"),
    ({"min_lr_ratio": -0.5}, "train.min_lr_ratio"), ({"ema_decay": 1.1}, "train.ema_decay"),
    ({"logit_normal_std": 0.0}, "train.logit_normal_std"), ({"base_shift": 0.0}, "train.base_shift"),
    ({"max_shift": -1.0}, "train.max_shift"), ({"base_seq_len": 0}, "train.base_seq_len"),
    ({"log_every": 0}, "train.log_every"), ({"warmup_steps": -1}, "train.warmup_steps"),
    ({"ema_warmup_steps": -1}, "train.ema_warmup_steps"), ({"eval_every": -1}, "train.eval_every"),
    ({"seed": -1}, "train.seed"), ({"steps": 10, "warmup_steps": 10}, "warmup_steps"),
    ({"base_seq_len": 4096, "max_seq_len": 4096}, "max_seq_len"), ({"beta1": 0.95, "beta2": 0.9}, "beta2"),
])
def test_train_config_rejects(kw: dict[str, Any], needle: str) -> None:
    with pytest.raises(ValueError) as err:
        S.TrainConfig(**kw)
    assert needle in str(err.value)


@pytest.mark.parametrize("name", S.OPTIMIZER_NAMES)
def test_train_config_accepts_every_optimizer(name: str) -> None:
    assert S.TrainConfig(optimizer=name).optimizer == name


@pytest.mark.parametrize("name", S.SCHEDULE_NAMES)
def test_train_config_accepts_every_schedule(name: str) -> None:
    assert S.TrainConfig(schedule=name).schedule == name


@pytest.mark.parametrize("name", S.TIMESTEP_SAMPLERS)
def test_train_config_accepts_every_timestep_sampler(name: str) -> None:
    assert S.TrainConfig(timestep_sampler=name).timestep_sampler == name


def test_train_config_properties() -> None:
    t = S.TrainConfig(beta1=0.8, beta2=0.99)
    assert t.betas == (0.8, 0.99)
    assert t.ema_enabled and not S.TrainConfig(ema_decay=0.0).ema_enabled


@pytest.mark.parametrize("kw,needle", [
    ({"param_dtype": "int8"}, "param_dtype"), ({"reduce_dtype": "fp64"}, "reduce_dtype"),
    ({"float8_recipe": "blockwise"}, "float8_recipe"), ({"float8_min_features": 0}, "float8_min_features"),
])
def test_precision_spec_rejects(kw: dict[str, Any], needle: str) -> None:
    with pytest.raises(ValueError, match=needle):
        S.PrecisionSpec(**kw)


@pytest.mark.parametrize("dtype,nbytes", [("float32", 4), ("bfloat16", 2), ("float16", 2)])
def test_precision_param_dtype_bytes(dtype: str, nbytes: int) -> None:
    assert S.PrecisionSpec(param_dtype=dtype).param_dtype_bytes == nbytes


@pytest.mark.parametrize("mode", S.AC_MODES)
def test_activation_spec_accepts_modes(mode: str) -> None:
    assert S.ActivationSpec(mode=mode).mode == mode


@pytest.mark.parametrize("kw", [{"mode": "partial"}, {"layer_interval": 0}, {"save_op_frequency": 0}])
def test_activation_spec_rejects(kw: dict[str, Any]) -> None:
    with pytest.raises(ValueError):
        S.ActivationSpec(**kw)


@pytest.mark.parametrize("schedule", S.PIPELINE_SCHEDULES)
def test_pipeline_spec_accepts_schedules(schedule: str) -> None:
    assert S.PipelineSpec(schedule=schedule).schedule == schedule


@pytest.mark.parametrize("kw,needle", [
    ({"schedule": "dualpipe"}, "schedule"), ({"microbatches": 0}, "microbatches"),
    ({"stages_per_rank": 0}, "stages_per_rank"), ({"schedule": "gpipe", "stages_per_rank": 2}, "single-stage"),
    ({"schedule": "1f1b", "stages_per_rank": 3}, "single-stage"),
])
def test_pipeline_spec_rejects(kw: dict[str, Any], needle: str) -> None:
    with pytest.raises(ValueError, match=needle):
        S.PipelineSpec(**kw)


def test_pipeline_spec_interleaved_allows_virtual_stages() -> None:
    assert S.PipelineSpec(schedule="interleaved_1f1b", stages_per_rank=2).stages_per_rank == 2


@pytest.mark.parametrize("kw,needle", [
    ({"dp_replicate": 0}, "dp_replicate"), ({"tensor": 0}, "tensor"), ({"context": 0}, "context"),
    ({"pipeline": 0}, "pipeline"), ({"gpus_per_node": 0}, "gpus_per_node"), ({"dp_shard": 0}, "dp_shard"),
    ({"dp_shard": -2}, "dp_shard"), ({"compile_mode": "fast"}, "compile_mode"),
    ({"tensor": 16, "gpus_per_node": 8}, "NVLink domain"),
])
def test_parallel_spec_rejects(kw: dict[str, Any], needle: str) -> None:
    with pytest.raises(ValueError, match=needle):
        S.ParallelConfigSpec(**kw)


@pytest.mark.parametrize("tp,cp,pp,degree", [(1, 1, 1, 1), (2, 4, 1, 8), (8, 1, 2, 16), (1, 8, 1, 8)])
def test_parallel_model_parallel_degree(tp: int, cp: int, pp: int, degree: int) -> None:
    assert S.ParallelConfigSpec(tensor=tp, context=cp, pipeline=pp).model_parallel_degree == degree


@pytest.mark.parametrize("kw", [{"save_every": -1}, {"keep_last_n": -1}, {"keep_every_n_steps": -1},
                                {"export_dtype": "int4"}])
def test_checkpoint_config_rejects(kw: dict[str, Any]) -> None:
    with pytest.raises(ValueError):
        S.CheckpointConfig(**kw)


@pytest.mark.parametrize("kw", [{"loggers": ("console", "console")}, {"loggers": ("mlflow",)}, {"log_every": 0},
                                {"profile_steps": -1}, {"profile_warmup": -1}, {"memory_report_every": -1}])
def test_telemetry_config_rejects(kw: dict[str, Any]) -> None:
    with pytest.raises(ValueError):
        S.TelemetryConfig(**kw)


@pytest.mark.parametrize("loggers", [(), ("noop",), ("console", "jsonl", "tensorboard"), ("wandb",)])
def test_telemetry_config_accepts(loggers: tuple[str, ...]) -> None:
    assert S.TelemetryConfig(loggers=loggers).loggers == loggers


@pytest.mark.parametrize("kw", [{"metrics": ()}, {"metrics": ("a", "a")}, {"sampler": "ddim"}, {"steps": 0},
                                {"batch_size": 0}, {"frames": 0}, {"height": 0}, {"width": 0}, {"num_prompts": -1},
                                {"seed": -1}, {"guidance": -1.0}])
def test_eval_config_rejects(kw: dict[str, Any]) -> None:
    with pytest.raises(ValueError):
        S.EvalConfig(**kw)


@pytest.mark.parametrize("sampler", S.SAMPLER_NAMES)
def test_inference_config_accepts_every_sampler(sampler: str) -> None:
    assert S.InferenceConfig(sampler=sampler).sampler == sampler


@pytest.mark.parametrize("kw", [{"sampler": "plms"}, {"dtype": "int8"}, {"steps": 0}, {"batch_size": 0},
                                {"frames": 0}, {"guidance": -0.1}, {"guidance_rescale": 1.2}, {"fps": 0.0}])
def test_inference_config_rejects(kw: dict[str, Any]) -> None:
    with pytest.raises(ValueError):
        S.InferenceConfig(**kw)


@pytest.mark.parametrize("kw", [{"mode": "prefix"}, {"lora_rank": 0}, {"lora_alpha": 0.0}, {"lora_dropout": 1.5},
                                {"control_channels": 0}, {"control_scale": -1.0}, {"control_blocks": 0},
                                {"lora_targets": ()}, {"lora_targets": ("q_proj", "q_proj")}])
def test_finetune_config_rejects(kw: dict[str, Any]) -> None:
    with pytest.raises(ValueError):
        S.FinetuneConfig(**kw)


def test_finetune_full_mode_allows_empty_targets() -> None:
    assert S.FinetuneConfig(mode="full", lora_targets=()).lora_targets == ()


@pytest.mark.parametrize("kw", [{"algorithm": "ppo"}, {"group_size": 0}, {"sampler_steps": 0},
                                {"kl_coefficient": -0.1}, {"clip_range": 0.0}, {"sde_noise_scale": -1.0},
                                {"dpo_beta": 0.0}, {"guidance": -1.0}, {"mixgrpo_window": -1},
                                {"rewards": ("a", "a")}, {"rewards": ("a", "b"), "reward_weights": (1.0,)},
                                {"algorithm": "grpo", "group_size": 1}])
def test_rl_config_rejects(kw: dict[str, Any]) -> None:
    with pytest.raises(ValueError):
        S.RLConfig(**kw)


def test_rl_config_dpo_allows_group_of_one() -> None:
    assert S.RLConfig(algorithm="dpo", group_size=1).group_size == 1


def test_run_config_cross_section_rules() -> None:
    with pytest.raises(ValueError, match="newer"):
        S.RunConfig(schema_version=S.SCHEMA_VERSION + 1)
    with pytest.raises(ValueError, match="audio tower"):
        S.RunConfig(model=S.ModelConfig(audio_width=64))
    ok = S.RunConfig(model=S.ModelConfig(audio_width=64), data=S.DataConfig(audio_frames=16))
    assert ok.model.has_audio
    with pytest.raises(ValueError, match="sequence-shard factor"):
        S.RunConfig(data=S.DataConfig(buckets=(S.BucketConfig(frames=3, height=2, width=2),)),
                    parallel=S.ParallelConfigSpec(context=2))
    with pytest.raises(ValueError, match="not divisible"):
        S.RunConfig(data=S.DataConfig(buckets=(S.BucketConfig(frames=16, height=31, width=32),)))


@pytest.mark.parametrize("cp,tp,sp,ok", [(2, 1, True, True), (4, 1, True, True), (1, 4, True, True),
                                         (1, 3, True, False), (1, 3, False, True), (3, 1, True, False)])
def test_run_config_sequence_shard_divisibility(cp: int, tp: int, sp: bool, ok: bool) -> None:
    # 16 x 32 x 32 latents with 1x2x2 patches: 4096 tokens, divisible by powers of two only
    kw = dict(parallel=S.ParallelConfigSpec(context=cp, tensor=tp, sequence_parallel=sp))
    if ok:
        assert S.RunConfig(**kw).sequence_length == 4096
    else:
        with pytest.raises(ValueError):
            S.RunConfig(**kw)


def test_run_config_micro_batch_and_name() -> None:
    cfg = S.RunConfig(data=S.DataConfig(buckets=(S.BucketConfig(micro_batch_size=3),)))
    assert cfg.micro_batch_size == 3
    assert replace(cfg, train=S.TrainConfig(micro_batch_size=5)).micro_batch_size == 5
    assert cfg.resolved_run_name().startswith("video_dit-") and "-d12" in cfg.resolved_run_name()
    assert replace(cfg, run_name="mine").resolved_run_name() == "mine"


# ----------------------------------------------------------------------------- coercion


@pytest.mark.parametrize("ann,value,expect", [
    (int, 3, 3), (int, 3.0, 3), (int, "7", 7), (int, "0x10", 16), (int, "1e3", 1000),
    (float, 1, 1.0), (float, "2.5", 2.5), (float, "1e-4", 1e-4),
    (bool, True, True), (bool, "yes", True), (bool, "off", False), (bool, "TRUE", True), (bool, 0, False),
    (bool, 1, True), (str, 5, "5"), (str, "x", "x"),
    (tuple[str, ...], "a", ("a",)), (tuple[str, ...], ["a", "b"], ("a", "b")), (tuple[int, ...], [1, "2"], (1, 2)),
    (tuple[int, int], [1, 2], (1, 2)), (Optional[int], None, None), (Optional[int], "4", 4), (Any, [1], [1]),
    (dict[str, Any], {"a": 1}, {"a": 1}), (list[int], ["1", 2], [1, 2]),
])
def test_coerce_accepts(ann: Any, value: Any, expect: Any) -> None:
    got = coerce(ann, value, "x")
    assert got == expect and type(got) is type(expect)


@pytest.mark.parametrize("ann,value", [
    (int, True), (int, 2.5), (int, "two"), (int, "2.5"), (int, [1]), (float, True), (float, "fast"), (float, None),
    (bool, "maybe"), (bool, 2), (str, {"a": 1}), (str, [1]), (tuple[int, int], [1, 2, 3]), (dict[str, Any], [1]),
])
def test_coerce_rejects(ann: Any, value: Any) -> None:
    with pytest.raises(ConfigError) as err:
        coerce(ann, value, "sec.key")
    assert "sec.key" in str(err.value)


def test_build_dataclass_suggests_close_keys() -> None:
    with pytest.raises(ConfigError, match="did you mean 'depth'"):
        build_dataclass(S.ModelConfig, {"detph": 3}, "model")
    with pytest.raises(ConfigError, match="unknown config key 'model.zzz'"):
        build_dataclass(S.ModelConfig, {"zzz": 3}, "model")
    with pytest.raises(ConfigError, match="model.depth"):
        build_dataclass(S.ModelConfig, {"depth": 0}, "model")


def test_build_dataclass_nested_sections() -> None:
    cfg = build_dataclass(S.RunConfig, {"parallel": {"precision": {"param_dtype": "float32"},
                                                     "activation": {"mode": "full"}},
                                        "data": {"buckets": [{"name": "x", "frames": 4}]}})
    assert cfg.parallel.precision.param_dtype == "float32"
    assert cfg.parallel.activation.mode == "full"
    assert cfg.data.buckets[0].name == "x" and cfg.data.buckets[0].frames == 4
    with pytest.raises(ConfigError, match="must be a mapping"):
        build_dataclass(S.RunConfig, {"train": 5})


# ----------------------------------------------------------------------------- overrides


@pytest.mark.parametrize("text,path,value", [
    # YAML 1.1 reads 1e-4 (no dot) as a string; the float annotation coerces it later
    ("train.lr=1e-4", ["train", "lr"], "1e-4"), ("train.lr=1.0e-4", ["train", "lr"], 1e-4), ("model.depth=12", ["model", "depth"], 12),
    ("run_name=abc", ["run_name"], "abc"), ("a.b=null", ["a", "b"], None), ("a.b=~", ["a", "b"], None),
    ("a.b=", ["a", "b"], ""), ("a.b=[1, 2]", ["a", "b"], [1, 2]), ("a.b={x: 1}", ["a", "b"], {"x": 1}),
    ("a.b=true", ["a", "b"], True), ("x[2].y=3", ["x", 2, "y"], 3), ("x[0][1]=4", ["x", 0, 1], 4),
    ("a.b= spaced ", ["a", "b"], "spaced"), ("a.b=a: b: c", ["a", "b"], "a: b: c"),
])
def test_parse_override(text: str, path: list, value: Any) -> None:
    got_path, got_value = parse_override(text)
    assert got_path == path and got_value == value


@pytest.mark.parametrize("text", ["no_equals", "=3", "a..b=1", "a.b-c.d=1", "a.[0]=1"])
def test_parse_override_rejects(text: str) -> None:
    with pytest.raises(ConfigError):
        parse_override(text)


def test_apply_overrides_creates_and_rejects() -> None:
    out = apply_overrides({}, ["new.section.key=1"])
    assert out == {"new": {"section": {"key": 1}}}
    base = {"l": [{"a": 1}], "s": 3}
    assert apply_overrides(base, ["l[0].a=2"])["l"][0]["a"] == 2
    assert base["l"][0]["a"] == 1  # input not mutated
    for bad in ("l[3].a=1", "s.x=1", "l[5]=1"):
        with pytest.raises(ConfigError):
            apply_overrides(base, [bad])


@pytest.mark.parametrize("a,b,expect", [
    ({}, {"x": 1}, {"x": 1}), ({"x": 1}, {}, {"x": 1}), ({"x": {"y": 1}}, {"x": {"z": 2}}, {"x": {"y": 1, "z": 2}}),
    ({"x": {"y": 1}}, {"x": 3}, {"x": 3}), ({"x": 3}, {"x": {"y": 1}}, {"x": {"y": 1}}),
    ({"x": [1, 2]}, {"x": [3]}, {"x": [3]}),
])
def test_deep_merge(a: dict, b: dict, expect: dict) -> None:
    assert deep_merge(a, b) == expect


# ----------------------------------------------------------------------------- files


def test_load_mapping_errors(tmp_path: Path) -> None:
    with pytest.raises(ConfigError, match="not found"):
        load_mapping(tmp_path / "missing.yaml")
    bad = tmp_path / "bad.yaml"
    bad.write_text("a: [1, 2\n")
    with pytest.raises(ConfigError, match="not valid YAML"):
        load_mapping(bad)
    scalar = tmp_path / "scalar.yaml"
    scalar.write_text("3\n")
    with pytest.raises(ConfigError, match="mapping at the top level"):
        load_mapping(scalar)
    base = tmp_path / "base_bad.yaml"
    base.write_text("_base_: {a: 1}\n")
    with pytest.raises(ConfigError, match="_base_"):
        load_mapping(base)
    empty = tmp_path / "empty.yaml"
    empty.write_text("")
    assert load_mapping(empty) == {}


def test_load_mapping_cycle_and_list_of_bases(tmp_path: Path) -> None:
    (tmp_path / "a.yaml").write_text("_base_: b.yaml\nx: 1\n")
    (tmp_path / "b.yaml").write_text("_base_: a.yaml\ny: 2\n")
    with pytest.raises(ConfigError, match="cyclic"):
        load_mapping(tmp_path / "a.yaml")
    (tmp_path / "p.yaml").write_text("x: 1\ny: 1\n")
    (tmp_path / "q.yaml").write_text("y: 2\nz: 2\n")
    (tmp_path / "r.yaml").write_text("_base_: [p.yaml, q.yaml]\nz: 3\n")
    assert load_mapping(tmp_path / "r.yaml") == {"x": 1, "y": 2, "z": 3}


def test_env_interpolation(tmp_path: Path, monkeypatch: pytest.MonkeyPatch) -> None:
    f = tmp_path / "e.yaml"
    f.write_text("output_dir: ${env:AVGEN_T_OUT:/tmp/x}/run\nnotes:\n  - ${env:AVGEN_T_N:a}\n  - b\n")
    monkeypatch.delenv("AVGEN_T_OUT", raising=False)
    assert load_mapping(f)["output_dir"] == "/tmp/x/run"
    monkeypatch.setenv("AVGEN_T_OUT", "/data")
    monkeypatch.setenv("AVGEN_T_N", "z")
    m = load_mapping(f)
    assert m["output_dir"] == "/data/run" and m["notes"] == ["z", "b"]
    g = tmp_path / "g.yaml"
    g.write_text("run_name: ${env:AVGEN_T_UNSET_VAR}\n")
    monkeypatch.delenv("AVGEN_T_UNSET_VAR", raising=False)
    with pytest.raises(ConfigError, match="AVGEN_T_UNSET_VAR"):
        load_mapping(g)


def test_pipeline_section_alias(tmp_path: Path) -> None:
    f = tmp_path / "pp.yaml"
    f.write_text("parallel:\n  pipeline: {schedule: gpipe, microbatches: 4}\n")
    cfg = load_config(f)
    assert cfg.parallel.pipeline_schedule.schedule == "gpipe" and cfg.parallel.pipeline_schedule.microbatches == 4
    assert cfg.parallel.pipeline == 1


def test_save_load_round_trip_and_diff(tmp_path: Path) -> None:
    cfg = load_config(None, ["model.depth=3", "train.lr=0.002", "telemetry.loggers=[console]",
                             "data.buckets=[{name: a, frames: 4, height: 8, width: 8}]"])
    path = save_config(cfg, tmp_path / "sub" / "resolved.yaml")
    assert path.exists() and not path.with_suffix(".yaml.tmp").exists()
    again = load_config(path)
    assert again == cfg
    assert config_diff(cfg, again) == {}
    assert render_diff({}) == "(no differences)"
    other = replace(cfg, seed=3)
    d = config_diff(cfg, other)
    assert d == {"seed": (0, 3)}
    assert "seed" in render_diff(d) and "0 -> 3" in render_diff(d)
    plain = config_to_dict(cfg)
    assert plain["data"]["buckets"][0]["name"] == "a" and isinstance(plain["telemetry"]["loggers"], list)
    assert yaml.safe_load(path.read_text())["model"]["depth"] == 3


def test_config_diff_on_mappings() -> None:
    d = config_diff({"a": {"b": 1}, "c": 2}, {"a": {"b": 2}, "d": 3})
    assert set(d) == {"a.b", "c", "d"}
    assert d["a.b"] == (1, 2)


# ----------------------------------------------------------------------------- resolvers


def _cfg(*overrides: str) -> S.RunConfig:
    return load_config(None, list(overrides))


@pytest.mark.parametrize("world,kw,shape", [
    (8, ["parallel.context=4"], {"dp_shard": 2, "cp": 4}), (8, ["parallel.tensor=8"], {"dp_shard": 1, "tp": 8}),
    (16, ["parallel.dp_replicate=2", "parallel.context=2"], {"dp_replicate": 2, "dp_shard": 4, "cp": 2}),
    (4, [], {"dp_shard": 4}), (8, ["parallel.pipeline=2", "parallel.tensor=2"], {"pp": 2, "tp": 2, "dp_shard": 2}),
])
def test_build_parallel_dims(world: int, kw: list[str], shape: dict[str, int]) -> None:
    dims = build_parallel_dims(_cfg(*kw), world_size=world)
    names = {"cp": "context", "tp": "tensor", "pp": "pipeline"}
    for k, v in shape.items():
        assert getattr(dims, names.get(k, k)) == v, (k, dims)


def test_build_parallel_dims_reads_world_size(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.setenv("WORLD_SIZE", "4")
    assert build_parallel_dims(_cfg("parallel.context=2")).dp_shard == 2


def test_resolved_parallel_settings() -> None:
    cfg = _cfg("parallel.precision.param_dtype=float32", "parallel.activation.mode=selective_layer",
               "parallel.activation.layer_interval=3", "parallel.fsdp.reshard_after_forward=false",
               "parallel.pipeline_schedule.schedule=gpipe", "parallel.pipeline_schedule.microbatches=6",
               "parallel.sequence_parallel=false")
    prec = build_precision_config(cfg)
    assert str(prec.param_dtype).endswith("float32")
    ac = build_activation_checkpoint(cfg)
    assert ac.mode == "selective_layer" and ac.layer_interval == 3
    assert build_fsdp_config(cfg).reshard_after_forward is False
    pp = build_pipeline_config(cfg)
    assert pp.schedule == "gpipe" and pp.microbatches == 6
    pc = build_parallel_config(cfg)
    assert pc.sequence_parallel is False and pc.activation_checkpoint.mode == "selective_layer"


@pytest.mark.parametrize("world,gbs,mbs,cp,accum", [(8, 8, 1, 4, 4), (8, 16, 1, 1, 2), (1, 4, 2, 1, 2),
                                                    (8, 2, 1, 4, 1)])
def test_gradient_accumulation(world: int, gbs: int, mbs: int, cp: int, accum: int) -> None:
    cfg = _cfg(f"train.global_batch_size={gbs}", f"train.micro_batch_size={mbs}", f"parallel.context={cp}")
    assert gradient_accumulation(cfg, world_size=world) == accum


def test_gradient_accumulation_rejects_indivisible_batch() -> None:
    with pytest.raises(ValueError):
        gradient_accumulation(_cfg("train.global_batch_size=3", "train.micro_batch_size=1"), world_size=2)


def test_model_shape_and_kwargs() -> None:
    cfg = _cfg("model.depth=4", "model.width=256", "model.num_heads=4", "data.text_tokens=77",
               "data.buckets=[{name: a, frames: 8, height: 16, width: 16, micro_batch_size: 2}]")
    assert sequence_length_for(cfg) == 8 * 8 * 8
    shape = build_model_shape(cfg)
    assert shape.sequence_length == 512 and shape.micro_batch_size == 2 and shape.depth == 4
    assert shape.text_tokens == 77 and shape.parameters == cfg.model.estimated_parameters()
    kw = model_kwargs(cfg)
    assert kw["depth"] == 4 and kw["text_context_length"] == 77 and kw["out_channels"] == 16
    assert "audio_width" not in kw
    no_cross = _cfg("model.cross_attention=false")
    assert "text_context_length" not in model_kwargs(no_cross)
    assert build_model_shape(no_cross).text_tokens == 0
    extra = _cfg("model.extra={qk_norm: false}")
    assert model_kwargs(extra)["qk_norm"] is False


def test_model_shape_adds_audio_tokens() -> None:
    cfg = _cfg("model.audio_width=64", "data.audio_frames=32")
    assert build_model_shape(cfg).sequence_length == sequence_length_for(cfg) + 32
    kw = model_kwargs(cfg)
    assert kw["audio_width"] == 64 and kw["audio_in_channels"] == 8


@pytest.mark.parametrize("name", ["b200", "B200", " h100 "])
def test_build_accelerator(name: str) -> None:
    acc = build_accelerator(name)
    assert acc is not None


def test_build_accelerator_unknown_and_interconnects() -> None:
    with pytest.raises(ValueError, match="unknown gpu"):
        build_accelerator("tpu-v5")
    intra, inter = build_interconnects("b200")
    intra_h, _ = build_interconnects("h100")
    assert intra is not intra_h and inter is not None


@pytest.mark.parametrize("ffn,cross,width,heads", [("swiglu", True, 256, 4), ("gelu", True, 192, 3),
                                                   ("swiglu", False, 128, 2), ("gelu", False, 320, 5)])
def test_parameter_estimate_matches_the_built_model(ffn: str, cross: bool, width: int, heads: int) -> None:
    """The closed form counts exactly what the model builds (on the meta device), so the
    simulator's memory and FLOP estimates start from the right parameter count."""
    from avgen_b200.config.loader import load_config
    from avgen_b200.config.resolve import build_model, counted_parameters

    cfg = load_config(None, overrides=[f"model.width={width}", f"model.num_heads={heads}", "model.depth=3",
                                       f"model.ffn={ffn}", f"model.cross_attention={str(cross).lower()}",
                                       "data.text_width=96"])
    built = sum(p.numel() for p in build_model(cfg, meta=True).parameters())
    assert counted_parameters(cfg) == built
    assert cfg.model.estimated_parameters(text_width=96) == built


def test_loader_build_keyword_form() -> None:
    from avgen_b200.config.loader import build

    built = build(S.TrainConfig, {"lr": "2e-4", "steps": 500}, where="train")
    assert built == build_dataclass(S.TrainConfig, {"lr": 2e-4, "steps": 500})
    with pytest.raises(ConfigError, match="train"):
        build(S.TrainConfig, {"learning_rat": 1.0}, where="train")
    with pytest.raises(ConfigError, match="warmup_steps"):  # the dataclass's own check, as a ConfigError
        build(S.TrainConfig, {"steps": 50}, where="train")
