"""Text-to-video(/audio) generation (avgen/infer/pipeline.py:263-892 API).

``GenerationPipeline(model, video_codec=..., text_encoder=...)(prompts)`` encodes
the prompts, draws latent noise from the ``sampler`` RNG stream, builds the
sigma schedule (with the shift resolved from the global token count), runs the
sampler loop and decodes.

B200 choices: with guidance on, the conditional and unconditional branches run
as ONE forward over a doubled batch (the GEMMs see twice the rows and the
attention kernel twice the heads, instead of two launches of every kernel),
and the loop never synchronises with the host between steps. Under context
parallelism each forward shards the token streams and gathers the outputs.
"""
from __future__ import annotations

import json
import math
from collections.abc import Callable, Mapping, Sequence
from dataclasses import asdict, dataclass, field, replace
from pathlib import Path
from typing import Any, cast

import torch

from avgen_b200.codecs.normalization import LatentStatistics, denormalize_latents, resolve_latent_normalization
from avgen_b200.core.model_input import ModelInput, ModelOutput
from avgen_b200.core.patchify import GridPatchifier, Patchifier, unpatchify_grid
from avgen_b200.core.rng import RNGStreams
from avgen_b200.core.tokens import TextContext, TokenStream
from avgen_b200.infer.conditioning import StreamState, build_model_input, default_audio_patchifier
from avgen_b200.infer.guidance import GuidanceConfig, apply_guidance
from avgen_b200.infer.sampler import EulerSampler, Sampler, SamplerConfig, build_sampler
from avgen_b200.infer.schedule import ScheduleConfig, SigmaSchedule, build_sigma_schedule

__all__ = ["GeneratedMedia", "GenerationConfig", "GenerationPipeline", "LatentCallback", "ProgressCallback"]

ProgressCallback = Callable[[int, int, float], None]
LatentCallback = Callable[[int, torch.Tensor], None]
_DTYPES = ("float32", "bfloat16", "float16")


@dataclass(frozen=True, slots=True)
class GenerationConfig:
    steps: int = 30
    seed: int = 0
    height: int = 256
    width: int = 256
    num_frames: int = 17
    fps: float = 24.0
    guidance: GuidanceConfig = field(default_factory=GuidanceConfig)
    sampler: SamplerConfig = field(default_factory=SamplerConfig)
    schedule: ScheduleConfig = field(default_factory=ScheduleConfig)
    negative_prompt: str | None = None
    generate_audio: bool = False
    audio_seconds: float | None = None
    dtype: str = "float32"

    def __post_init__(self) -> None:
        for name in ("steps", "height", "width", "num_frames"):
            v = getattr(self, name)
            if isinstance(v, bool) or v < 1:
                raise ValueError(f"{name} must be a positive integer; got {v!r}")
        if isinstance(self.seed, bool) or self.seed < 0:
            raise ValueError(f"seed must be a non-negative integer; got {self.seed!r}")
        if not (math.isfinite(self.fps) and self.fps > 0.0):
            raise ValueError(f"fps must be positive; got {self.fps!r}")
        if self.audio_seconds is not None and not self.audio_seconds > 0.0:
            raise ValueError(f"audio_seconds must be positive; got {self.audio_seconds!r}")
        if self.dtype not in _DTYPES:
            raise ValueError(f"dtype must be one of {_DTYPES}; got {self.dtype!r}")

    @property
    def duration_seconds(self) -> float:
        return self.num_frames / self.fps

    def to_dict(self) -> dict[str, Any]:
        out = asdict(self)
        out["guidance"], out["sampler"], out["schedule"] = (self.guidance.to_dict(), self.sampler.to_dict(),
                                                            self.schedule.to_dict())
        return out

    @classmethod
    def from_dict(cls, values: Mapping[str, Any]) -> GenerationConfig:
        v = dict(values)
        if isinstance(v.get("guidance"), Mapping):
            v["guidance"] = GuidanceConfig.from_dict(v["guidance"])
        if isinstance(v.get("sampler"), Mapping):
            v["sampler"] = SamplerConfig.from_dict(v["sampler"])
        if isinstance(v.get("schedule"), Mapping):
            v["schedule"] = ScheduleConfig.from_dict(v["schedule"])
        names = set(cls.__dataclass_fields__)  # type: ignore[attr-defined]
        return cls(**{k: val for k, val in v.items() if k in names})


@dataclass(frozen=True, slots=True)
class GeneratedMedia:
    video: torch.Tensor
    prompts: tuple[str, ...]
    fps: float
    config: Mapping[str, Any]
    audio: torch.Tensor | None = None
    sample_rate: int | None = None
    latents: torch.Tensor | None = None
    negative_prompts: tuple[str, ...] = ()

    @property
    def batch_size(self) -> int:
        return int(self.video.shape[0])

    def __len__(self) -> int:
        return self.batch_size

    @property
    def has_audio(self) -> bool:
        return self.audio is not None

    @property
    def duration_seconds(self) -> float:
        return int(self.video.shape[2]) / self.fps

    def metadata(self) -> dict[str, Any]:
        return {"prompts": list(self.prompts), "negative_prompts": list(self.negative_prompts), "fps": self.fps,
                "frames": int(self.video.shape[2]), "height": int(self.video.shape[3]),
                "width": int(self.video.shape[4]), "sample_rate": self.sample_rate, "has_audio": self.has_audio,
                "config": dict(self.config)}


def _cat_streams(a: TokenStream, b: TokenStream) -> TokenStream:
    lv = torch.cat((a.level_values, b.level_values)) if a.has_level_groups and b.has_level_groups else \
        torch.empty(0, device=a.tokens.device)
    li = torch.cat((a.level_index, b.level_index)) if a.has_level_groups and b.has_level_groups else \
        torch.empty(0, dtype=torch.int32, device=a.tokens.device)
    return TokenStream(tokens=torch.cat((a.tokens, b.tokens)), coords=torch.cat((a.coords, b.coords)),
                       mask=torch.cat((a.mask, b.mask)), noise_level=torch.cat((a.noise_level, b.noise_level)),
                       layout=a.layout, conditioned=torch.cat((a.conditioned, b.conditioned)), level_values=lv,
                       level_index=li)


def _doubled(inputs: ModelInput, other_text: TextContext) -> ModelInput:
    """``inputs`` followed by the same streams with ``other_text`` (one batched forward for CFG)."""
    text = TextContext(features=torch.cat((inputs.text.features, other_text.features)),
                       mask=torch.cat((inputs.text.mask, other_text.mask)))
    return ModelInput(video=_cat_streams(inputs.video, inputs.video), audio=_cat_streams(inputs.audio, inputs.audio),
                      text=text, condition_mode=torch.cat((inputs.condition_mode, inputs.condition_mode)))


class GenerationPipeline:
    __slots__ = ("audio_codec", "audio_patchifier", "batch_guidance", "config", "cp_mesh", "device",
                 "latent_statistics", "model", "patchifier", "text_encoder", "video_codec")

    def __init__(self, model: Any, *, video_codec: Any, text_encoder: Any = None, audio_codec: Any = None,
                 patchifier: Patchifier | None = None, audio_patchifier: Patchifier | None = None,
                 config: GenerationConfig | None = None, device: torch.device | str | None = None,
                 latent_statistics: LatentStatistics | None = None, cp_mesh: Any = None,
                 batch_guidance: bool = True) -> None:
        self.model = model
        self.video_codec = video_codec
        self.text_encoder = text_encoder
        self.audio_codec = audio_codec
        self.config = config or GenerationConfig()
        if self.config.generate_audio and audio_codec is None:
            raise ValueError("generate_audio needs an audio_codec to decode the audio latent")
        self.patchifier = patchifier or getattr(model, "patchifier", None) or GridPatchifier()
        self.audio_patchifier = audio_patchifier or default_audio_patchifier()
        self.device = torch.device(device) if device is not None else _model_device(model)
        self.latent_statistics = latent_statistics or resolve_latent_normalization(
            video_codec, channels=getattr(video_codec, "latent_channels", None))
        self.cp_mesh = cp_mesh
        self.batch_guidance = batch_guidance

    # ------------------------------------------------------------------ public API
    def __call__(self, prompts: Sequence[str] | str, *, steps: int | None = None,
                 guidance: GuidanceConfig | float | None = None, seed: int | None = None, height: int | None = None,
                 width: int | None = None, num_frames: int | None = None, fps: float | None = None,
                 negative_prompts: Sequence[str] | str | None = None, sampler: SamplerConfig | str | None = None,
                 schedule: ScheduleConfig | None = None, generate_audio: bool | None = None,
                 progress_callback: ProgressCallback | None = None, latent_callback: LatentCallback | None = None,
                 return_latents: bool = False) -> GeneratedMedia:
        plist = [prompts] if isinstance(prompts, str) else list(prompts)
        if not plist:
            raise ValueError("prompts must contain at least one entry")
        cfg = self._resolve(steps=steps, guidance=guidance, seed=seed, height=height, width=width,
                            num_frames=num_frames, fps=fps, sampler=sampler, schedule=schedule,
                            generate_audio=generate_audio, negative_prompts=negative_prompts)
        negatives = _negatives(negative_prompts, cfg, len(plist))
        if cfg.generate_audio and self.audio_codec is None:
            raise ValueError("audio generation was requested but the pipeline has no audio_codec")
        dtype = getattr(torch, cfg.dtype)
        rng = RNGStreams.from_seed(cfg.seed, device=self.device)
        text = self._encode(plist, dtype=dtype)
        null_text = self._encode(negatives, dtype=dtype) if any(negatives) else text.nullified()
        video, audio = self._initial_states(batch=len(plist), config=cfg, rng=rng, dtype=dtype)
        tokens = _sequence_length(video, audio, self.patchifier, self.audio_patchifier)
        sched = build_sigma_schedule(cfg.schedule, sequence_length=tokens, device=self.device)
        solver = build_sampler(cfg.sampler)
        solver.reset()
        video, audio = self._sample(video_state=video, audio_state=audio, text=text, null_text=null_text,
                                    schedule=sched, solver=solver, config=cfg, rng=rng,
                                    progress_callback=progress_callback, latent_callback=latent_callback)
        pinned = dict(cfg.to_dict())
        pinned.update(resolved_shift=sched.shift, sequence_length=tokens,
                      video_codec_id=getattr(self.video_codec, "fingerprint", None),
                      audio_codec_id=getattr(self.audio_codec, "fingerprint", None),
                      text_encoder_id=getattr(self.text_encoder, "fingerprint", None),
                      latent_statistics=self.latent_statistics.to_dict())
        out_audio = self._decode_audio(audio.latents) if audio is not None else None
        sr = int(getattr(self.audio_codec, "sample_rate", 0)) or None if out_audio is not None else None
        return GeneratedMedia(video=self._decode_video(video.latents), audio=out_audio, fps=cfg.fps, sample_rate=sr,
                              prompts=tuple(plist), negative_prompts=tuple(negatives), config=pinned,
                              latents=video.latents if return_latents else None)

    @classmethod
    def from_checkpoint(cls, path: str | Path, *, video_codec: Any, text_encoder: Any = None, audio_codec: Any = None,
                        config: GenerationConfig | None = None, device: torch.device | str | None = None,
                        model_name: str | None = None, model_config: Mapping[str, Any] | None = None,
                        **kwargs: Any) -> GenerationPipeline:
        """Build the model named in ``config.json`` next to the weights, load safetensors
        exports or a checkpoint directory, and wrap it."""
        from avgen_b200.models import build_model

        root = Path(path)
        if not root.exists():
            raise FileNotFoundError(f"checkpoint path does not exist: {root}")
        manifest = _manifest(root)
        name = model_name or manifest.get("model", {}).get("name")
        if name is None:
            raise RuntimeError(f"no model name under {root}; pass model_name= or add config.json with model.name")
        model = build_model(name, dict(model_config or manifest.get("model", {}).get("config", {})))
        _load_weights(root, model)
        model.eval()
        target = torch.device(device) if device is not None else _model_device(model)
        model.to(target)
        defaults = config if config is not None else (
            GenerationConfig.from_dict(manifest["generation"]) if "generation" in manifest else None)
        return cls(model, video_codec=video_codec, text_encoder=text_encoder, audio_codec=audio_codec,
                   config=defaults, device=target, **kwargs)

    # ------------------------------------------------------------------ internals
    def _resolve(self, *, steps: int | None, guidance: GuidanceConfig | float | None, seed: int | None,
                 height: int | None, width: int | None, num_frames: int | None, fps: float | None,
                 sampler: SamplerConfig | str | None, schedule: ScheduleConfig | None, generate_audio: bool | None,
                 negative_prompts: Sequence[str] | str | None) -> GenerationConfig:
        o: dict[str, Any] = {k: v for k, v in (("steps", steps), ("seed", seed), ("height", height),
                                               ("width", width), ("num_frames", num_frames), ("fps", fps),
                                               ("generate_audio", generate_audio), ("schedule", schedule))
                             if v is not None}
        if guidance is not None:
            o["guidance"] = GuidanceConfig(scale=float(guidance)) if isinstance(guidance, (int, float)) else guidance
        if sampler is not None:
            o["sampler"] = SamplerConfig(name=sampler) if isinstance(sampler, str) else sampler
        if isinstance(negative_prompts, str):
            o["negative_prompt"] = negative_prompts
        cfg = replace(self.config, **o)
        if cfg.schedule.steps != cfg.steps:
            cfg = replace(cfg, schedule=replace(cfg.schedule, steps=cfg.steps))
        return cfg

    def _encode(self, prompts: Sequence[str], *, dtype: torch.dtype) -> TextContext:
        if self.text_encoder is None:
            return TextContext.empty(len(prompts), 1, device=self.device, dtype=dtype)
        feats, mask = self.text_encoder.encode(list(prompts))
        ctx = TextContext(features=feats.to(device=self.device, dtype=dtype), mask=mask.to(device=self.device))
        ctx.validate()
        return ctx

    def _initial_states(self, *, batch: int, config: GenerationConfig, rng: RNGStreams,
                        dtype: torch.dtype) -> tuple[StreamState, StreamState | None]:
        pixels = (batch, int(getattr(self.video_codec, "channels", 3)), config.num_frames, config.height, config.width)
        shape = tuple(self.video_codec.latent_shape(pixels))
        latents = torch.randn(shape, generator=rng.sampler, device=self.device, dtype=dtype)
        video = StreamState(latents=latents, fps=config.fps / max(int(self.video_codec.temporal_compression), 1))
        if not config.generate_audio:
            return video, None
        seconds = config.audio_seconds or config.duration_seconds
        hop = int(getattr(self.audio_codec, "hop_length", 256))
        rate = int(getattr(self.audio_codec, "sample_rate", 24000))
        frames = max(round(seconds * rate / hop), 1)
        chans = int(getattr(self.audio_codec, "latent_channels", 1))
        audio = torch.randn((batch, chans, frames), generator=rng.sampler, device=self.device, dtype=dtype)
        return video, StreamState(latents=audio, fps=rate / hop)

    def _sample(self, *, video_state: StreamState, audio_state: StreamState | None, text: TextContext,
                null_text: TextContext, schedule: SigmaSchedule, solver: Sampler, config: GenerationConfig,
                rng: RNGStreams, progress_callback: ProgressCallback | None,
                latent_callback: LatentCallback | None) -> tuple[StreamState, StreamState | None]:
        total = schedule.num_steps
        audio_solver = build_sampler(config.sampler) if audio_state is not None else None
        if audio_solver is not None:
            audio_solver.reset()
        with torch.no_grad():
            for i, sigma, sigma_next in schedule:
                progress = i / max(total - 1, 1)
                video_state, audio_state = self._advance(video_state, audio_state, text, null_text, sigma,
                                                         sigma_next, progress, solver, audio_solver, config, rng)
                if progress_callback is not None:
                    progress_callback(i, total, sigma_next)
                if latent_callback is not None:
                    latent_callback(i, video_state.latents)
        return video_state, audio_state

    def _advance(self, video_state: StreamState, audio_state: StreamState | None, text: TextContext,
                 null_text: TextContext, sigma: float, sigma_next: float, progress: float, solver: Sampler,
                 audio_solver: Sampler | None, config: GenerationConfig,
                 rng: RNGStreams) -> tuple[StreamState, StreamState | None]:
        audio_lat = audio_state.latents if audio_state is not None else None
        if audio_state is None and self._fusable_euler(solver, config, video_state):
            return self._guided_euler(video_state, text, null_text, sigma, sigma_next, progress, config), None

        def velocity(v_lat: torch.Tensor, a_lat: torch.Tensor | None, at: float):  # noqa: ANN202
            a_st = audio_state.with_latents(a_lat) if audio_state is not None and a_lat is not None else None
            return self._velocity(video_state.with_latents(v_lat), a_st, text, null_text, at, config, progress)

        v_vel, a_vel = velocity(video_state.latents, audio_lat, sigma)
        nv = solver.step(v_vel, video_state.latents, sigma, sigma_next,
                         denoise=lambda probe, at: velocity(probe, audio_lat, at)[0], generator=rng.sampler)
        next_video = video_state.with_latents(nv)
        next_audio = audio_state
        if audio_state is not None and a_vel is not None and audio_solver is not None:
            next_audio = audio_state.with_latents(audio_solver.step(a_vel, audio_state.latents, sigma, sigma_next,
                                                                    generator=rng.sampler))
        return next_video, next_audio

    def _fusable_euler(self, solver: Sampler, config: GenerationConfig, video_state: StreamState) -> bool:
        """Plain Euler with plain CFG on a B200: the guidance combine and the
        update run as one fused kernel over the batched forward's two halves."""
        g = config.guidance
        return (isinstance(solver, EulerSampler) and video_state.latents.is_cuda and self.batch_guidance
                and g.is_enabled and g.rescale == 0.0 and not g.projection)

    def _guided_euler(self, video_state: StreamState, text: TextContext, null_text: TextContext, sigma: float,
                      sigma_next: float, progress: float, config: GenerationConfig) -> StreamState:
        from avgen_b200.ops import kernels as K

        inputs = build_model_input(video=video_state, sigma=sigma, text=text, patchifier=self.patchifier)
        both = self._forward(_doubled(inputs, null_text))
        b = inputs.batch_size
        cond = unpatchify_grid(both.video[:b], inputs.video.layout)
        uncond = unpatchify_grid(both.video[b:], inputs.video.layout)
        lat = video_state.latents
        s = torch.full((b,), sigma, device=lat.device, dtype=torch.float32)
        sn = torch.full((b,), sigma_next, device=lat.device, dtype=torch.float32)
        scale = config.guidance.modality_scale("text", progress)
        return video_state.with_latents(K.guided_euler(cond, uncond, lat, s, sn, scale=scale))

    def _velocity(self, video_state: StreamState, audio_state: StreamState | None, text: TextContext,
                  null_text: TextContext, sigma: float, config: GenerationConfig,
                  progress: float) -> tuple[torch.Tensor, torch.Tensor | None]:
        inputs = build_model_input(video=video_state, sigma=sigma, text=text, patchifier=self.patchifier,
                                   audio=audio_state, audio_patchifier=self.audio_patchifier)
        uncond: ModelOutput | None = None
        if config.guidance.is_enabled and self.batch_guidance:
            both = self._forward(_doubled(inputs, null_text))
            b = inputs.batch_size
            cond = ModelOutput(video=both.video[:b], audio=both.audio[:b])
            uncond = ModelOutput(video=both.video[b:], audio=both.audio[b:])
        else:
            cond = self._forward(inputs)
            if config.guidance.is_enabled:
                uncond = self._forward(replace(inputs, text=null_text))
        v = apply_guidance(cond.video.float(), uncond.video.float() if uncond is not None else None,
                           config=config.guidance, progress=progress, modality="text")
        v_grid = unpatchify_grid(v, inputs.video.layout).to(video_state.latents.dtype)
        a_grid = None
        if audio_state is not None and inputs.has_audio:
            a = apply_guidance(cond.audio.float(), uncond.audio.float() if uncond is not None else None,
                               config=config.guidance, progress=progress, modality="audio")
            a_grid = unpatchify_grid(a, inputs.audio.layout)[..., 0, 0].to(audio_state.latents.dtype)
        return v_grid, a_grid

    def _forward(self, inputs: ModelInput) -> ModelOutput:
        if self.cp_mesh is None or self.cp_mesh.size() == 1:
            return cast(ModelOutput, self.model(inputs))
        from avgen_b200.parallel.context import gather_tokens, shard_stream

        sharded = inputs.replace_streams(video=shard_stream(inputs.video, self.cp_mesh),
                                         audio=shard_stream(inputs.audio, self.cp_mesh) if inputs.has_audio
                                         else inputs.audio)
        out = self.model(sharded)
        return ModelOutput(video=gather_tokens(out.video, self.cp_mesh),
                           audio=gather_tokens(out.audio, self.cp_mesh) if inputs.has_audio else out.audio,
                           auxiliary=tuple(gather_tokens(t, self.cp_mesh) for t in out.auxiliary))

    def _decode_video(self, latents: torch.Tensor) -> torch.Tensor:
        return self.video_codec.decode(denormalize_latents(latents, self.latent_statistics))

    def _decode_audio(self, latents: torch.Tensor) -> torch.Tensor:
        stats = resolve_latent_normalization(self.audio_codec, channels=int(latents.shape[1]))
        return self.audio_codec.decode(denormalize_latents(latents, stats))


def _sequence_length(video: StreamState, audio: StreamState | None, patchifier: Patchifier,
                     audio_patchifier: Patchifier) -> int:
    n = patchifier.layout_for(tuple(video.grid().shape)).num_tokens
    if audio is not None:
        n += audio_patchifier.layout_for(tuple(audio.grid().shape)).num_tokens
    return n


def _negatives(negative_prompts: Sequence[str] | str | None, config: GenerationConfig, batch: int) -> list[str]:
    if negative_prompts is None:
        return [config.negative_prompt or ""] * batch
    if isinstance(negative_prompts, str):
        return [negative_prompts] * batch
    vals = list(negative_prompts)
    if len(vals) == 1:
        return vals * batch
    if len(vals) != batch:
        raise ValueError(f"negative_prompts must have 1 or {batch} entries; got {len(vals)}")
    return vals


def _model_device(model: Any) -> torch.device:
    params = getattr(model, "parameters", None)
    if callable(params):
        for p in params():
            return torch.device(p.device)
    return torch.device("cpu")


def _manifest(root: Path) -> dict[str, Any]:
    for cand in ((root / "config.json") if root.is_dir() else root.with_suffix(".json"), root.parent / "config.json"):
        if cand.is_file():
            return cast(dict[str, Any], json.loads(cand.read_text()))
    return {}


def _load_weights(root: Path, model: Any) -> None:
    files = [root] if root.is_file() and root.suffix == ".safetensors" else (
        sorted(root.glob("*.safetensors")) or sorted(root.glob("*/*.safetensors")) if root.is_dir() else [])
    if files:
        from safetensors.torch import load_file

        state: dict[str, torch.Tensor] = {}
        for f in files:
            state.update(load_file(str(f)))
        missing = list(getattr(model.load_state_dict(state, strict=False), "missing_keys", ()) or ())
        if missing:
            raise RuntimeError(f"{len(missing)} parameters missing from the weights under {root}; first: "
                               f"{missing[:5]}")
        return
    from avgen_b200.checkpoint import load_model

    load_model(root, model)
