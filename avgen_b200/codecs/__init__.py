"""Codecs: protocols, dependency-free reference codecs, pretrained adapters,
latent normalisation and a mel frontend (avgen/codecs/__init__.py)."""
from avgen_b200.codecs.adapters import DiffusersVideoCodec, TilingConfig, TransformersTextEncoder, blend_tiles
from avgen_b200.codecs.mel import MelConfig, MelFrontend, hz_to_mel, mel_filterbank, mel_to_hz, stft_magnitude
from avgen_b200.codecs.normalization import (LatentStatistics, denormalize_latents, normalize_latents,
                                             resolve_latent_normalization)
from avgen_b200.codecs.protocols import AudioCodec, TextEncoder, VideoCodec, Vocoder, codec_fingerprint
from avgen_b200.codecs.reference import ReferenceAudioCodec, ReferenceTextEncoder, ReferenceVideoCodec

__all__ = ["AudioCodec", "DiffusersVideoCodec", "LatentStatistics", "MelConfig", "MelFrontend", "ReferenceAudioCodec",
           "ReferenceTextEncoder", "ReferenceVideoCodec", "TextEncoder", "TilingConfig", "TransformersTextEncoder",
           "VideoCodec", "Vocoder", "blend_tiles", "codec_fingerprint", "denormalize_latents", "hz_to_mel",
           "mel_filterbank", "mel_to_hz", "normalize_latents", "resolve_latent_normalization", "stft_magnitude"]
