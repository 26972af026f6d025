"""Models: VideoDiT / AVDiT, their blocks and layers, attention, RoPE, registry."""
from avgen_b200.models.attention import attention, device_arch, key_padding_mask
from avgen_b200.models.blocks import CrossModalFusion, DiTBlock, RopeInputs, TextRefinerBlock, temporal_neighbour_mask
from avgen_b200.models.dit import AVDiT, AVDiTConfig, VideoDiT, VideoDiTConfig, list_presets, preset
from avgen_b200.models.layers import (AdaLNModulation, CrossAttention, FusedRMSNorm, GeluMLP, SelfAttention, SwiGLU,
                                      TimestepEmbedding, modulate, sinusoidal_embedding)
from avgen_b200.models.registry import build_model, list_models, model_config_class, register_model
from avgen_b200.models.rope import RoPEScaling, RotaryEmbedding, RotaryTables, apply_rotary, build_rotary_tables

__all__ = [
    "AVDiT", "AVDiTConfig", "AdaLNModulation", "CrossAttention", "CrossModalFusion", "DiTBlock", "FusedRMSNorm",
    "GeluMLP", "RoPEScaling", "RopeInputs", "RotaryEmbedding", "RotaryTables", "SelfAttention", "SwiGLU",
    "TextRefinerBlock", "TimestepEmbedding", "VideoDiT", "VideoDiTConfig", "apply_rotary", "attention",
    "build_model", "build_rotary_tables", "device_arch", "key_padding_mask", "list_models", "list_presets",
    "model_config_class", "modulate", "preset", "register_model", "sinusoidal_embedding", "temporal_neighbour_mask",
]

# constants and helpers the reference also exports at this level
from avgen_b200.models.attention import attention_backends, sdpa_context  # noqa: E402
from avgen_b200.models.dit import FUSION_MODES  # noqa: E402
from avgen_b200.models.layers import MODULATION_CHUNKS, init_linear, init_norm, rms_norm  # noqa: E402
from avgen_b200.models.registry import MODEL_ENTRY_POINT_GROUP  # noqa: E402
from avgen_b200.models.rope import ROPE_SCALING_MODES, rope_axis_pairs  # noqa: E402

__all__ += ["FUSION_MODES", "MODEL_ENTRY_POINT_GROUP", "MODULATION_CHUNKS", "ROPE_SCALING_MODES", "attention_backends",
            "init_linear", "init_norm", "rms_norm", "rope_axis_pairs", "sdpa_context"]
