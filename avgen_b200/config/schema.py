"""Run-configuration schema: frozen dataclasses, validated on construction.

The field names and sections are the YAML interface shared with avgen
(avgen/config/schema.py:112-1230): ``model``, ``data`` (with ``buckets``),
``train``, ``parallel`` (+ ``precision``, ``activation``, ``fsdp``,
``pipeline_schedule``), ``checkpoint``, ``telemetry``, ``eval``, ``inference``,
``finetune``, ``rl``. Every failure names the dotted field.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

__all__ = ["ActivationSpec", "BucketConfig", "CheckpointConfig", "DataConfig", "EvalConfig", "FSDPSpec",
           "FinetuneConfig", "InferenceConfig", "ModelConfig", "ParallelConfigSpec", "PipelineSpec", "PrecisionSpec",
           "RLConfig", "RunConfig", "SCHEMA_VERSION", "TelemetryConfig", "TrainConfig"]

SCHEMA_VERSION = 1
DTYPE_NAMES = ("float32", "bfloat16", "float16")
AC_MODES = ("fused", "none", "full", "selective_op", "selective_layer")
OPTIMIZER_NAMES = ("adamw", "adamw_8bit", "adafactor", "adamw_bf16_state", "sgd_momentum", "muon")
SCHEDULE_NAMES = ("constant", "cosine", "linear", "wsd")
TIMESTEP_SAMPLERS = ("uniform", "logit_normal", "shifted_logit_normal", "mode")
SAMPLER_NAMES = ("euler", "heun", "dpmpp_2m", "res_multistep", "euler_ancestral")
PIPELINE_SCHEDULES = ("gpipe", "1f1b", "interleaved_1f1b", "zero_bubble")
DATA_SOURCES = ("synthetic", "latent_shards")
LOGGER_NAMES = ("console", "jsonl", "tensorboard", "wandb", "noop")
FINETUNE_MODES = ("lora", "full", "control")
RL_ALGORITHMS = ("grpo", "dpo")
FFN_KINDS = ("swiglu", "gelu")


def _pos_int(name: str, v: Any) -> None:
    if isinstance(v, bool) or not isinstance(v, int) or v < 1:
        raise ValueError(f"{name} must be a positive integer; got {v!r}")


def _nonneg_int(name: str, v: Any) -> None:
    if isinstance(v, bool) or not isinstance(v, int) or v < 0:
        raise ValueError(f"{name} must be a non-negative integer; got {v!r}")


def _pos(name: str, v: Any) -> None:
    if isinstance(v, bool) or not isinstance(v, (int, float)) or not v > 0:
        raise ValueError(f"{name} must be positive; got {v!r}")


def _nonneg(name: str, v: Any) -> None:
    if isinstance(v, bool) or not isinstance(v, (int, float)) or v < 0:
        raise ValueError(f"{name} must be non-negative; got {v!r}")


def _frac(name: str, v: Any) -> None:
    if isinstance(v, bool) or not isinstance(v, (int, float)) or not 0.0 <= v <= 1.0:
        raise ValueError(f"{name} must lie in [0, 1]; got {v!r}")


def _choice(name: str, v: Any, options: tuple[str, ...]) -> None:
    if v not in options:
        raise ValueError(f"{name} must be one of {', '.join(options)}; got {v!r}")


def _unique(name: str, values: tuple[Any, ...]) -> None:
    if len(set(values)) != len(values):
        raise ValueError(f"{name} contains duplicates: {list(values)}")


@dataclass(frozen=True, slots=True)
class ModelConfig:
    name: str = "video_dit"
    depth: int = 12
    width: int = 768
    num_heads: int = 12
    mlp_ratio: int = 4
    patch_frames: int = 1
    patch_height: int = 2
    patch_width: int = 2
    in_channels: int = 16
    out_channels: int = -1
    cross_attention: bool = True
    audio_width: int = 0
    rope_theta: float = 10000.0
    ffn: str = "swiglu"
    parameters: int = 0
    extra: dict[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if not isinstance(self.name, str) or not self.name:
            raise ValueError("model.name must be a non-empty string")
        for n in ("depth", "width", "num_heads", "mlp_ratio", "patch_frames", "patch_height", "patch_width",
                  "in_channels"):
            _pos_int(f"model.{n}", getattr(self, n))
        _nonneg_int("model.audio_width", self.audio_width)
        _nonneg_int("model.parameters", self.parameters)
        _pos("model.rope_theta", self.rope_theta)
        _choice("model.ffn", self.ffn, FFN_KINDS)
        if self.out_channels != -1:
            _pos_int("model.out_channels", self.out_channels)
        if self.width % self.num_heads:
            raise ValueError(f"model.num_heads must divide model.width; got width={self.width} "
                             f"num_heads={self.num_heads}")
        if not isinstance(self.extra, dict):
            raise TypeError("model.extra must be a mapping")

    @property
    def head_dim(self) -> int:
        return self.width // self.num_heads

    @property
    def latent_out_channels(self) -> int:
        return self.in_channels if self.out_channels == -1 else self.out_channels

    @property
    def has_audio(self) -> bool:
        return self.audio_width > 0

    def estimated_parameters(self, *, text_width: int | None = None) -> int:
        """Closed-form parameter count of this framework's video DiT: per block q/k/v/out
        with their QK-norm weights, the MLP (three matrices for SwiGLU, two for GELU,
        hidden rounded up to 256), cross-attention (its k/v read the text after the
        root's ``text_width`` -> width projection), its norms and the block's
        modulation table; at the root the patch and text projections, the timestep MLP,
        the shared adaLN projection (6 x width outputs) and the output projection.
        ``parameters`` overrides it; :func:`avgen_b200.config.resolve.build_model_shape`
        counts the built model's parameters exactly when it can."""
        if self.parameters:
            return self.parameters
        w = self.width
        tw = text_width if text_width is not None else int(self.extra.get("text_width", 4096))
        hidden = -(-int(self.mlp_ratio * w) // 256) * 256
        mlp = (3 if self.ffn == "swiglu" else 2) * hidden * w
        attention = 4 * w * w + 2 * self.head_dim
        norms = (3 if self.cross_attention else 2) * w
        per_block = attention * (2 if self.cross_attention else 1) + mlp + 6 * w + norms
        patch = self.in_channels * self.patch_frames * self.patch_height * self.patch_width
        out = (self.out_channels if self.out_channels != -1 else self.in_channels) * (
            self.patch_frames * self.patch_height * self.patch_width)
        root = (patch + 1) * w + (tw + 1) * w + (256 * w + w * w + 2 * w) + (w + 1) * 6 * w + (w + 1) * out + w
        return int(per_block * self.depth + root)


@dataclass(frozen=True, slots=True)
class BucketConfig:
    name: str = "default"
    frames: int = 16
    height: int = 32
    width: int = 32
    micro_batch_size: int = 1
    weight: float = 1.0

    def __post_init__(self) -> None:
        for n in ("frames", "height", "width", "micro_batch_size"):
            _pos_int(f"data.buckets[{self.name}].{n}", getattr(self, n))
        _nonneg(f"data.buckets[{self.name}].weight", self.weight)

    def tokens(self, model: ModelConfig) -> int:
        for axis, patch in (("frames", model.patch_frames), ("height", model.patch_height),
                            ("width", model.patch_width)):
            if getattr(self, axis) % patch:
                raise ValueError(f"data.buckets[{self.name}].{axis}={getattr(self, axis)} is not divisible by "
                                 f"the model patch size {patch}")
        return (self.frames // model.patch_frames) * (self.height // model.patch_height) * (
            self.width // model.patch_width)


@dataclass(frozen=True, slots=True)
class DataConfig:
    source: str = "synthetic"
    root: str = ""
    manifest: str = ""
    buckets: tuple[BucketConfig, ...] = (BucketConfig(),)
    num_workers: int = 2
    prefetch_batches: int = 2
    shuffle_buffer: int = 1024
    seed: int = 0
    drop_last: bool = True
    latent_channels: int = 16
    text_tokens: int = 226
    text_width: int = 4096
    audio_frames: int = 0
    audio_channels: int = 8
    caption_dropout: float = 0.1
    repeat: int = 0

    def __post_init__(self) -> None:
        _choice("data.source", self.source, DATA_SOURCES)
        for n in ("num_workers", "prefetch_batches", "shuffle_buffer", "repeat", "seed", "audio_frames"):
            _nonneg_int(f"data.{n}", getattr(self, n))
        for n in ("latent_channels", "text_tokens", "text_width", "audio_channels"):
            _pos_int(f"data.{n}", getattr(self, n))
        _frac("data.caption_dropout", self.caption_dropout)
        if not self.buckets:
            raise ValueError("data.buckets must contain at least one bucket")
        _unique("data.buckets", tuple(b.name for b in self.buckets))
        if self.source == "latent_shards" and not self.root:
            raise ValueError("data.root must be set when data.source='latent_shards'")

    @property
    def has_audio(self) -> bool:
        return self.audio_frames > 0

    def bucket(self, name: str) -> BucketConfig:
        for b in self.buckets:
            if b.name == name:
                return b
        raise KeyError(f"no bucket named {name!r}; defined: {', '.join(b.name for b in self.buckets)}")

    def largest_bucket(self) -> BucketConfig:
        return max(self.buckets, key=lambda b: b.frames * b.height * b.width)


@dataclass(frozen=True, slots=True)
class TrainConfig:
    steps: int = 1000
    global_batch_size: int = 8
    micro_batch_size: int = -1
    optimizer: str = "adamw"
    lr: float = 1e-4
    weight_decay: float = 0.01
    beta1: float = 0.9
    beta2: float = 0.95
    eps: float = 1e-8
    max_grad_norm: float = 1.0
    schedule: str = "cosine"
    warmup_steps: int = 100
    decay_ratio: float = 0.1
    min_lr_ratio: float = 0.1
    objective: str = "flow_matching"
    timestep_sampler: str = "shifted_logit_normal"
    logit_normal_mean: float = 0.0
    logit_normal_std: float = 1.0
    base_shift: float = 0.5
    max_shift: float = 1.15
    base_seq_len: int = 256
    max_seq_len: int = 4096
    audio_loss_weight: float = 1.0
    ema_decay: float = 0.9999
    ema_warmup_steps: int = 0
    seed: int = 0
    log_every: int = 10
    eval_every: int = 0
    seed_deterministic: bool = False

    def __post_init__(self) -> None:
        _pos_int("train.steps", self.steps)
        _pos_int("train.global_batch_size", self.global_batch_size)
        if self.micro_batch_size != -1:
            _pos_int("train.micro_batch_size", self.micro_batch_size)
        _choice("train.optimizer", self.optimizer, OPTIMIZER_NAMES)
        _choice("train.schedule", self.schedule, SCHEDULE_NAMES)
        _choice("train.timestep_sampler", self.timestep_sampler, TIMESTEP_SAMPLERS)
        _pos("train.lr", self.lr)
        _pos("train.eps", self.eps)
        for n in ("weight_decay", "max_grad_norm", "audio_loss_weight"):
            _nonneg(f"train.{n}", getattr(self, n))
        for n in ("beta1", "beta2", "decay_ratio", "min_lr_ratio", "ema_decay"):
            _frac(f"train.{n}", getattr(self, n))
        for n in ("logit_normal_std", "base_shift", "max_shift"):
            _pos(f"train.{n}", getattr(self, n))
        for n in ("base_seq_len", "max_seq_len", "log_every"):
            _pos_int(f"train.{n}", getattr(self, n))
        for n in ("warmup_steps", "ema_warmup_steps", "eval_every", "seed"):
            _nonneg_int(f"train.{n}", getattr(self, n))
        if self.warmup_steps >= self.steps:
            raise ValueError(f"train.warmup_steps={self.warmup_steps} must be less than train.steps={self.steps}")
        if self.max_seq_len <= self.base_seq_len:
            raise ValueError("train.max_seq_len must exceed train.base_seq_len")
        if self.beta2 <= self.beta1:
            raise ValueError("train.beta2 must exceed train.beta1")

    @property
    def ema_enabled(self) -> bool:
        return self.ema_decay > 0.0

    @property
    def betas(self) -> tuple[float, float]:
        return (self.beta1, self.beta2)


@dataclass(frozen=True, slots=True)
class PrecisionSpec:
    param_dtype: str = "bfloat16"
    reduce_dtype: str = "float32"
    enable_float8: bool = False
    float8_min_features: int = 1024
    float8_recipe: str = "tensorwise"

    def __post_init__(self) -> None:
        _choice("parallel.precision.param_dtype", self.param_dtype, DTYPE_NAMES)
        _choice("parallel.precision.reduce_dtype", self.reduce_dtype, DTYPE_NAMES)
        _choice("parallel.precision.float8_recipe", self.float8_recipe, ("tensorwise", "rowwise"))
        _pos_int("parallel.precision.float8_min_features", self.float8_min_features)

    @property
    def param_dtype_bytes(self) -> int:
        return 4 if self.param_dtype == "float32" else 2


@dataclass(frozen=True, slots=True)
class ActivationSpec:
    # "fused": the sm_100a block's built-in recompute (saves x, O, lse); the others are the eager policies
    mode: str = "fused"
    layer_interval: int = 2
    save_op_frequency: int = 1

    def __post_init__(self) -> None:
        _choice("parallel.activation.mode", self.mode, AC_MODES)
        _pos_int("parallel.activation.layer_interval", self.layer_interval)
        _pos_int("parallel.activation.save_op_frequency", self.save_op_frequency)


@dataclass(frozen=True, slots=True)
class FSDPSpec:
    reshard_after_forward: bool = True
    cpu_offload: bool = False
    shard_last_block_after_forward: bool = False
    ignore_frozen_params: bool = False


@dataclass(frozen=True, slots=True)
class PipelineSpec:
    schedule: str = "1f1b"
    microbatches: int = 8
    stages_per_rank: int = 1

    def __post_init__(self) -> None:
        _choice("parallel.pipeline.schedule", self.schedule, PIPELINE_SCHEDULES)
        _pos_int("parallel.pipeline.microbatches", self.microbatches)
        _pos_int("parallel.pipeline.stages_per_rank", self.stages_per_rank)
        if self.stages_per_rank > 1 and self.schedule in ("gpipe", "1f1b"):
            raise ValueError(f"parallel.pipeline.schedule={self.schedule!r} is single-stage but stages_per_rank="
                             f"{self.stages_per_rank}")


@dataclass(frozen=True, slots=True)
class ParallelConfigSpec:
    dp_replicate: int = 1
    dp_shard: int = -1
    tensor: int = 1
    context: int = 1
    pipeline: int = 1
    enable_loss_parallel: bool = True
    sequence_parallel: bool = True
    compile_blocks: bool = False
    compile_mode: str = "default"
    gpus_per_node: int = 8
    precision: PrecisionSpec = field(default_factory=PrecisionSpec)
    activation: ActivationSpec = field(default_factory=ActivationSpec)
    fsdp: FSDPSpec = field(default_factory=FSDPSpec)
    pipeline_schedule: PipelineSpec = field(default_factory=PipelineSpec)

    def __post_init__(self) -> None:
        for n in ("dp_replicate", "tensor", "context", "pipeline", "gpus_per_node"):
            _pos_int(f"parallel.{n}", getattr(self, n))
        if self.dp_shard != -1:
            _pos_int("parallel.dp_shard", self.dp_shard)
        _choice("parallel.compile_mode", self.compile_mode,
                ("default", "reduce-overhead", "max-autotune", "max-autotune-no-cudagraphs"))
        if self.tensor > self.gpus_per_node:
            raise ValueError(f"parallel.tensor={self.tensor} exceeds parallel.gpus_per_node={self.gpus_per_node}: "
                             "tensor parallelism must stay inside one NVLink domain")

    @property
    def model_parallel_degree(self) -> int:
        return self.tensor * self.context * self.pipeline


@dataclass(frozen=True, slots=True)
class CheckpointConfig:
    dir: str = ""
    save_every: int = 1000
    keep_last_n: int = 3
    keep_every_n_steps: int = 0
    async_save: bool = True
    resume: str = ""
    load_model_only: bool = False
    export_dtype: str = ""
    save_config: bool = True

    def __post_init__(self) -> None:
        for n in ("save_every", "keep_last_n", "keep_every_n_steps"):
            _nonneg_int(f"checkpoint.{n}", getattr(self, n))
        if self.export_dtype:
            _choice("checkpoint.export_dtype", self.export_dtype, DTYPE_NAMES)


@dataclass(frozen=True, slots=True)
class TelemetryConfig:
    loggers: tuple[str, ...] = ("console", "jsonl")
    project: str = "avgen"
    run_name: str = ""
    log_every: int = 10
    jsonl_path: str = ""
    tensorboard_dir: str = ""
    profile_steps: int = 0
    profile_warmup: int = 5
    memory_report_every: int = 0
    report_mfu: bool = True

    def __post_init__(self) -> None:
        _unique("telemetry.loggers", self.loggers)
        for n in self.loggers:
            _choice("telemetry.loggers[]", n, LOGGER_NAMES)
        _pos_int("telemetry.log_every", self.log_every)
        for n in ("profile_steps", "profile_warmup", "memory_report_every"):
            _nonneg_int(f"telemetry.{n}", getattr(self, n))


@dataclass(frozen=True, slots=True)
class EvalConfig:
    metrics: tuple[str, ...] = ("temporal_consistency", "motion_magnitude", "flicker_index", "static_frames")
    prompts_file: str = ""
    num_prompts: int = 0
    batch_size: int = 1
    seed: int = 0
    steps: int = 30
    guidance: float = 5.0
    sampler: str = "euler"
    negative_prompt: str = ""
    frames: int = 16
    height: int = 32
    width: int = 32
    decode: bool = False
    output_dir: str = ""
    save_samples: bool = False
    baseline_report: str = ""

    def __post_init__(self) -> None:
        _unique("eval.metrics", self.metrics)
        if not self.metrics:
            raise ValueError("eval.metrics must name at least one metric")
        _choice("eval.sampler", self.sampler, SAMPLER_NAMES)
        for n in ("steps", "batch_size", "frames", "height", "width"):
            _pos_int(f"eval.{n}", getattr(self, n))
        _nonneg_int("eval.num_prompts", self.num_prompts)
        _nonneg_int("eval.seed", self.seed)
        _nonneg("eval.guidance", self.guidance)


@dataclass(frozen=True, slots=True)
class InferenceConfig:
    sampler: str = "euler"
    steps: int = 30
    guidance: float = 5.0
    guidance_rescale: float = 0.0
    negative_prompt: str = ""
    seed: int = -1
    frames: int = 16
    height: int = 32
    width: int = 32
    fps: float = 16.0
    batch_size: int = 1
    dtype: str = "bfloat16"
    output: str = "samples"

    def __post_init__(self) -> None:
        _choice("inference.sampler", self.sampler, SAMPLER_NAMES)
        _choice("inference.dtype", self.dtype, DTYPE_NAMES)
        for n in ("steps", "batch_size", "frames", "height", "width"):
            _pos_int(f"inference.{n}", getattr(self, n))
        _nonneg("inference.guidance", self.guidance)
        _frac("inference.guidance_rescale", self.guidance_rescale)
        _pos("inference.fps", self.fps)


@dataclass(frozen=True, slots=True)
class FinetuneConfig:
    mode: str = "lora"
    base_checkpoint: str = ""
    lora_rank: int = 32
    lora_alpha: float = 32.0
    lora_dropout: float = 0.0
    lora_targets: tuple[str, ...] = ("q_proj", "k_proj", "v_proj", "out_proj", "gate_proj", "up_proj", "down_proj")
    use_dora: bool = False
    freeze_patterns: tuple[str, ...] = ()
    control_channels: int = 3
    control_blocks: int = -1
    control_scale: float = 1.0
    train_norms: bool = True

    def __post_init__(self) -> None:
        _choice("finetune.mode", self.mode, FINETUNE_MODES)
        _pos_int("finetune.lora_rank", self.lora_rank)
        _pos("finetune.lora_alpha", self.lora_alpha)
        _frac("finetune.lora_dropout", self.lora_dropout)
        _pos_int("finetune.control_channels", self.control_channels)
        _nonneg("finetune.control_scale", self.control_scale)
        if self.control_blocks != -1:
            _pos_int("finetune.control_blocks", self.control_blocks)
        if self.mode == "lora" and not self.lora_targets:
            raise ValueError("finetune.lora_targets is empty")
        _unique("finetune.lora_targets", self.lora_targets)


@dataclass(frozen=True, slots=True)
class RLConfig:
    algorithm: str = "grpo"
    reference_checkpoint: str = ""
    group_size: int = 8
    sampler_steps: int = 16
    kl_coefficient: float = 0.04
    clip_range: float = 0.2
    advantage_normalize: bool = True
    mixgrpo_window: int = 0
    sde_noise_scale: float = 0.7
    prompts_file: str = ""
    dpo_beta: float = 0.1
    guidance: float = 1.0
    timestep_shift: bool = False
    rewards: tuple[str, ...] = ()
    reward_weights: tuple[float, ...] = ()

    def __post_init__(self) -> None:
        _choice("rl.algorithm", self.algorithm, RL_ALGORITHMS)
        _pos_int("rl.group_size", self.group_size)
        _pos_int("rl.sampler_steps", self.sampler_steps)
        _nonneg("rl.kl_coefficient", self.kl_coefficient)
        _pos("rl.clip_range", self.clip_range)
        _nonneg("rl.sde_noise_scale", self.sde_noise_scale)
        _pos("rl.dpo_beta", self.dpo_beta)
        _nonneg("rl.guidance", self.guidance)
        _nonneg_int("rl.mixgrpo_window", self.mixgrpo_window)
        _unique("rl.rewards", self.rewards)
        if self.reward_weights and len(self.reward_weights) != len(self.rewards):
            raise ValueError("rl.reward_weights must have one entry per rl.rewards entry")
        if self.algorithm == "grpo" and self.group_size < 2:
            raise ValueError("rl.group_size must be at least 2 for GRPO")


@dataclass(frozen=True, slots=True)
class RunConfig:
    schema_version: int = SCHEMA_VERSION
    run_name: str = ""
    output_dir: str = "runs/default"
    seed: int = 0
    model: ModelConfig = field(default_factory=ModelConfig)
    data: DataConfig = field(default_factory=DataConfig)
    train: TrainConfig = field(default_factory=TrainConfig)
    parallel: ParallelConfigSpec = field(default_factory=ParallelConfigSpec)
    checkpoint: CheckpointConfig = field(default_factory=CheckpointConfig)
    telemetry: TelemetryConfig = field(default_factory=TelemetryConfig)
    eval: EvalConfig = field(default_factory=EvalConfig)
    inference: InferenceConfig = field(default_factory=InferenceConfig)
    finetune: FinetuneConfig = field(default_factory=FinetuneConfig)
    rl: RLConfig = field(default_factory=RLConfig)
    notes: str = ""

    def __post_init__(self) -> None:
        _pos_int("schema_version", self.schema_version)
        if self.schema_version > SCHEMA_VERSION:
            raise ValueError(f"schema_version={self.schema_version} is newer than this version understands "
                             f"({SCHEMA_VERSION})")
        _nonneg_int("seed", self.seed)
        if self.model.has_audio and not self.data.has_audio:
            raise ValueError(f"model.audio_width={self.model.audio_width} declares an audio tower but "
                             "data.audio_frames=0")
        for b in self.data.buckets:
            b.tokens(self.model)
        shard = self.parallel.context * (self.parallel.tensor if self.parallel.sequence_parallel else 1)
        if shard > 1:
            for b in self.data.buckets:
                if b.tokens(self.model) % shard:
                    raise ValueError(f"data bucket {b.name!r} yields {b.tokens(self.model)} tokens, not divisible by "
                                     f"the sequence-shard factor {shard} (context x tensor when sequence parallel)")

    @property
    def sequence_length(self) -> int:
        return self.data.largest_bucket().tokens(self.model)

    @property
    def micro_batch_size(self) -> int:
        if self.train.micro_batch_size != -1:
            return self.train.micro_batch_size
        return self.data.largest_bucket().micro_batch_size

    def resolved_run_name(self) -> str:
        if self.run_name:
            return self.run_name
        return f"{self.model.name}-{self.model.estimated_parameters() / 1e9:.1f}b-d{self.model.depth}"
