"""Sampling: samplers, sigma schedules, guidance, conditioning and the
generation pipeline (avgen/infer/__init__.py)."""
from avgen_b200.infer.conditioning import (StreamState, build_model_input, condition_first_frame, condition_mask,
                                           condition_stream, condition_temporal_prefix, default_audio_patchifier,
                                           first_frame_mask, temporal_prefix_mask, unconditional_input)
from avgen_b200.infer.guidance import (GuidanceConfig, adaptive_projected_guidance, apply_guidance,
                                       apply_modality_guidance, classifier_free_guidance, rescale_guidance,
                                       unconditional_branch)
from avgen_b200.infer.pipeline import GeneratedMedia, GenerationConfig, GenerationPipeline
from avgen_b200.infer.sampler import (DPMSolverPlusPlus2M, EulerAncestralSampler, EulerSampler, HeunSampler,
                                      ResMultistepSampler, Sampler, SamplerConfig, build_sampler, list_samplers,
                                      register_sampler, to_epsilon, to_x0)
from avgen_b200.infer.schedule import (ScheduleConfig, SigmaSchedule, apply_shift, build_sigma_schedule,
                                       karras_sigmas, linear_quadratic_sigmas, linear_sigmas, list_sigma_schedules,
                                       register_sigma_schedule, resolution_shift)

__all__ = ["DPMSolverPlusPlus2M", "EulerAncestralSampler", "EulerSampler", "GeneratedMedia", "GenerationConfig",
           "GenerationPipeline", "GuidanceConfig", "HeunSampler", "ResMultistepSampler", "Sampler", "SamplerConfig",
           "ScheduleConfig", "SigmaSchedule", "StreamState", "adaptive_projected_guidance", "apply_guidance",
           "apply_modality_guidance", "apply_shift", "build_model_input", "build_sampler", "build_sigma_schedule",
           "classifier_free_guidance", "condition_first_frame", "condition_mask", "condition_stream",
           "condition_temporal_prefix", "default_audio_patchifier", "first_frame_mask", "karras_sigmas",
           "linear_quadratic_sigmas", "linear_sigmas", "list_samplers", "list_sigma_schedules", "register_sampler",
           "register_sigma_schedule", "rescale_guidance", "resolution_shift", "temporal_prefix_mask", "to_epsilon",
           "to_x0", "unconditional_branch", "unconditional_input"]
