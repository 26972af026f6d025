"""Codecs on CPU: the reference video / audio codecs are exact inverses at many
geometries, latent normalisation round-trips and resolves from every source
form, the mel front end against its closed forms (Slaney-style mel scale is
monotone and invertible, a pure tone lands in its mel band), the text encoder's
masking, and the tiling planner covers every index (reference test strategy:
tests/test_codecs*.py)."""
from __future__ import annotations

import math

import pytest
import torch

from avgen_b200.codecs.adapters import TilingConfig, blend_tiles
from avgen_b200.codecs.mel import MelConfig, MelFrontend, hz_to_mel, mel_filterbank, mel_to_hz, stft_magnitude
from avgen_b200.codecs.normalization import (LatentStatistics, denormalize_latents, normalize_latents,
                                             resolve_latent_normalization)
from avgen_b200.codecs.reference import ReferenceAudioCodec, ReferenceTextEncoder, ReferenceVideoCodec


@pytest.mark.parametrize("tc,sc,scale", [(1, 1, 1.0), (1, 2, 1.0), (2, 2, 0.5), (4, 4, 2.0)])
def test_reference_video_codec_is_an_exact_inverse(tc: int, sc: int, scale: float) -> None:
    codec = ReferenceVideoCodec(channels=3, temporal_compression=tc, spatial_compression=sc, scale=scale)
    pixels = torch.randn(2, 3, 4 * tc, 4 * sc, 8 * sc, dtype=torch.float64)
    z = codec.encode(pixels)
    assert tuple(z.shape) == codec.latent_shape(pixels.shape)
    assert z.shape[1] == 3 * tc * sc * sc
    torch.testing.assert_close(codec.decode(z), pixels)
    assert codec.pixel_shape(z.shape) == tuple(pixels.shape)


def test_reference_video_codec_errors_and_identity() -> None:
    codec = ReferenceVideoCodec(spatial_compression=2)
    with pytest.raises(ValueError):
        codec.latent_shape((1, 3, 4, 5, 8))  # height not divisible
    with pytest.raises(ValueError):
        codec.latent_shape((1, 4, 4, 4, 8))  # wrong channels
    with pytest.raises(ValueError):
        codec.pixel_shape((1, 5, 2, 2, 2))
    with pytest.raises(TypeError):
        codec.encode(torch.zeros(1, 3, 2, 2, 2, dtype=torch.int64))
    with pytest.raises(ValueError):
        ReferenceVideoCodec(channels=0)
    a, b = ReferenceVideoCodec(seed=0), ReferenceVideoCodec(seed=1)
    assert a.fingerprint != b.fingerprint and a.fingerprint == ReferenceVideoCodec(seed=0).fingerprint
    assert a.latent_statistics.channels == a.latent_channels


@pytest.mark.parametrize("channels,hop", [(1, 64), (2, 128), (1, 256)])
def test_reference_audio_codec_round_trip(channels: int, hop: int) -> None:
    codec = ReferenceAudioCodec(channels=channels, hop_length=hop, sample_rate=16000)
    wav = torch.randn(2, channels, hop * 5, dtype=torch.float64)
    z = codec.encode(wav)
    assert z.shape == (2, channels * hop, 5) and codec.latent_frames(hop * 5) == 5
    torch.testing.assert_close(codec.decode(z), wav)
    assert codec.num_samples(5) == hop * 5 and codec.latent_rate == 16000 / hop
    with pytest.raises(ValueError):
        codec.latent_frames(hop * 5 + 1)
    with pytest.raises(ValueError):
        codec.encode(torch.zeros(2, channels + 1, hop))


def test_reference_text_encoder_masks_and_determinism() -> None:
    enc = ReferenceTextEncoder(width=16, max_length=8)
    feats, mask = enc.encode(["hi", "hello world!", ""])
    assert feats.shape == (3, 8, 16) and mask.tolist()[0] == [True, True] + [False] * 6
    assert mask[1].all() and not mask[2].any()  # truncated to max_length; empty prompt has no tokens
    assert bool((feats[0, 2:] == 0).all()) and bool((feats[2] == 0).all())
    again, _ = enc.encode("hi")
    torch.testing.assert_close(again[0], feats[0])
    other, _ = ReferenceTextEncoder(width=16, max_length=8, seed=9).encode("hi")
    assert not torch.allclose(other[0, :2], feats[0, :2])


# ----------------------------------------------------------------------------- normalisation


@pytest.mark.parametrize("channel_dim", [1, -1])
def test_latent_normalisation_round_trip(channel_dim: int) -> None:
    stats = LatentStatistics((0.5, -1.0, 2.0), (2.0, 0.5, 1.0), channel_dim=channel_dim)
    shape = (2, 3, 4, 4) if channel_dim == 1 else (2, 4, 4, 3)
    x = torch.randn(shape, dtype=torch.float64)
    y = normalize_latents(x, stats)
    torch.testing.assert_close(denormalize_latents(y, stats), x)
    mean, std = stats.tensors(ndim=4, dtype=torch.float64)
    torch.testing.assert_close(y, (x - mean) / std)
    with pytest.raises(ValueError):
        normalize_latents(torch.zeros(2, 5, 4, 4) if channel_dim == 1 else torch.zeros(2, 4, 4, 5), stats)


def test_latent_statistics_from_latents_and_identity() -> None:
    g = torch.Generator().manual_seed(0)
    x = torch.randn(64, 2, 8, 8, generator=g, dtype=torch.float64) * torch.tensor([3.0, 0.5]).view(1, 2, 1, 1) + \
        torch.tensor([1.0, -2.0]).view(1, 2, 1, 1)
    stats = LatentStatistics.from_latents(x)
    assert stats.mean == pytest.approx((1.0, -2.0), abs=0.05) and stats.std == pytest.approx((3.0, 0.5), rel=0.03)
    normed = normalize_latents(x, stats)
    assert float(normed.mean()) == pytest.approx(0.0, abs=1e-6)
    ident = LatentStatistics.identity(4)
    assert ident.is_identity and normalize_latents(torch.ones(1, 4, 2), ident) is not None
    assert LatentStatistics.from_dict(stats.to_dict()) == stats
    for bad in (((), ()), ((0.0,), (0.0,)), ((float("nan"),), (1.0,)), ((0.0, 1.0), (1.0,))):
        with pytest.raises(ValueError):
            LatentStatistics(*bad)


def test_resolve_latent_normalisation_forms() -> None:
    assert resolve_latent_normalization(None, channels=3).is_identity
    with pytest.raises(ValueError):
        resolve_latent_normalization(None)
    s = resolve_latent_normalization({"mean": [0.1, 0.2], "std": [1.0, 2.0]})
    assert s.mean == (0.1, 0.2) and s.std == (1.0, 2.0)
    d = resolve_latent_normalization({"scaling_factor": 0.5, "shift_factor": 0.1}, channels=4)
    assert d.channels == 4 and d.std == (2.0,) * 4 and d.mean == (0.1,) * 4
    w = resolve_latent_normalization({"latents_mean": torch.tensor([1.0]), "latents_std": torch.tensor([2.0])},
                                     channels=2)
    assert w.mean == (1.0, 1.0)
    codec = ReferenceVideoCodec(scale=0.5)
    assert resolve_latent_normalization(codec) == codec.latent_statistics
    assert resolve_latent_normalization(s) is s
    with pytest.raises(KeyError):
        resolve_latent_normalization({"gain": 1.0})
    with pytest.raises(ValueError):
        resolve_latent_normalization({"mean": [0.0, 0.0], "std": [1.0, 1.0]}, channels=3)
    with pytest.raises(TypeError):
        resolve_latent_normalization(3.0)


# ----------------------------------------------------------------------------- mel front end


def test_mel_scale_is_monotone_and_invertible() -> None:
    f = torch.linspace(0.0, 12000.0, 500, dtype=torch.float64)
    m = hz_to_mel(f)
    assert bool((m[1:] > m[:-1]).all())
    torch.testing.assert_close(mel_to_hz(m), f, rtol=1e-9, atol=1e-6)


@pytest.mark.parametrize("n_fft,hop,n_mels", [(512, 128, 40), (1024, 256, 80)])
def test_filterbank_shape_and_triangles(n_fft: int, hop: int, n_mels: int) -> None:
    cfg = MelConfig(sample_rate=16000, n_fft=n_fft, hop_length=hop, n_mels=n_mels)
    bank = mel_filterbank(cfg)
    assert bank.shape == (n_fft // 2 + 1, n_mels) and bool((bank >= 0).all())
    peaks = bank.argmax(0)
    assert bool((peaks[1:] >= peaks[:-1]).all())  # band centres ascend


def test_pure_tone_lands_in_its_band_and_frames_count() -> None:
    cfg = MelConfig(sample_rate=16000, n_fft=1024, hop_length=256, n_mels=64)
    front = MelFrontend(cfg)
    t = torch.arange(16000, dtype=torch.float32) / 16000
    tone = torch.sin(2 * math.pi * 1000.0 * t)[None]
    mel = front(tone)
    assert mel.shape == (1, 64, cfg.frames_for(16000))
    band = int(mel[0].mean(1).argmax())
    bank = mel_filterbank(cfg)
    bin_1k = round(1000.0 * cfg.n_fft / cfg.sample_rate)
    assert bank[bin_1k, band] > 0  # the strongest band covers the tone's FFT bin
    logm = front.log_mel(torch.zeros(1, 4096))
    assert float(logm.max()) == pytest.approx(math.log(cfg.log_epsilon))
    mag = stft_magnitude(tone, cfg)
    assert mag.shape == (1, cfg.num_bins, cfg.frames_for(16000))


@pytest.mark.parametrize("kw", [{"sample_rate": 0}, {"n_fft": 0}, {"win_length": 2048}, {"f_min": 100.0, "f_max": 50.0},
                                {"f_max": 20000.0}, {"power": 0.0}, {"log_epsilon": 0.0}])
def test_mel_config_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        MelConfig(**kw)


def test_mel_frames_without_centering() -> None:
    cfg = MelConfig(center=False, n_fft=1024, hop_length=256)
    assert cfg.frames_for(1024) == 1 and cfg.frames_for(100) == 0 and cfg.frames_for(2048) == 5


# ----------------------------------------------------------------------------- tiling


@pytest.mark.parametrize("total,tile,overlap", [(10, 4, 1), (100, 32, 8), (7, 7, 2), (5, 8, 2), (33, 16, 0),
                                                (1, 1, 0)])
def test_blend_tiles_cover_every_index(total: int, tile: int, overlap: int) -> None:
    windows = blend_tiles(total, tile, overlap)
    covered = set()
    for a, b in windows:
        assert 0 <= a < b <= total and b - a <= max(tile, total if tile >= total else tile)
        covered.update(range(a, b))
    assert covered == set(range(total))
    assert windows[0][0] == 0 and windows[-1][1] == total
    assert blend_tiles(0, 4, 1) == []


@pytest.mark.parametrize("kw", [{"tile_size": -1}, {"enabled": True, "tile_size": 4, "tile_overlap": 4},
                                {"temporal_chunk": 4, "temporal_overlap": 4}])
def test_tiling_config_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        TilingConfig(**kw)


def test_tiled_application_of_an_identity_is_exact() -> None:
    from avgen_b200.codecs.adapters import _tiled

    x = torch.randn(1, 2, 6, 20, 28)
    tiling = TilingConfig(enabled=True, tile_size=8, tile_overlap=3, temporal_chunk=4, temporal_overlap=1)
    out = _tiled(x, lambda t: t * 2.0, tiling, 1.0, 1.0)
    torch.testing.assert_close(out, x * 2.0, rtol=1e-5, atol=1e-5)
