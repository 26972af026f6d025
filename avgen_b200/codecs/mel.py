"""Log-mel frontend (avgen/codecs/mel.py API): STFT magnitude -> Slaney mel
filterbank -> log. The Slaney scale (M. Slaney, Auditory Toolbox, 1998) is
linear below 1 kHz (200/3 Hz per mel) and logarithmic above (a factor of 6.4
per 27 mels); filters are area-normalised triangles."""
from __future__ import annotations

import math
from dataclasses import asdict, dataclass
from functools import lru_cache
from typing import Any

import torch

__all__ = ["MelConfig", "MelFrontend", "hz_to_mel", "mel_filterbank", "mel_to_hz", "stft_magnitude"]

_HZ_PER_MEL = 200.0 / 3.0
_BREAK_HZ = 1000.0
_BREAK_MEL = _BREAK_HZ / _HZ_PER_MEL
_LOG_STEP = math.log(6.4) / 27.0


@dataclass(frozen=True, slots=True)
class MelConfig:
    sample_rate: int = 24000
    n_fft: int = 1024
    hop_length: int = 256
    win_length: int | None = None
    n_mels: int = 80
    f_min: float = 0.0
    f_max: float | None = None
    power: float = 1.0
    center: bool = True
    normalized: bool = False
    log_epsilon: float = 1e-5

    def __post_init__(self) -> None:
        for name in ("sample_rate", "n_fft", "hop_length", "n_mels"):
            v = getattr(self, name)
            if isinstance(v, bool) or v < 1:
                raise ValueError(f"{name} must be a positive integer; got {v!r}")
        if self.win_length is not None and not 1 <= self.win_length <= self.n_fft:
            raise ValueError(f"win_length must be in [1, n_fft]; got {self.win_length!r}")
        if not 0.0 <= self.f_min < self.upper_hz <= self.nyquist:
            raise ValueError(f"need 0 <= f_min < f_max <= nyquist; got f_min={self.f_min}, f_max={self.f_max}")
        if self.power <= 0 or self.log_epsilon <= 0:
            raise ValueError("power and log_epsilon must be positive")

    @property
    def nyquist(self) -> float:
        return self.sample_rate / 2.0

    @property
    def window_length(self) -> int:
        return self.win_length or self.n_fft

    @property
    def upper_hz(self) -> float:
        return self.nyquist if self.f_max is None else float(self.f_max)

    @property
    def num_bins(self) -> int:
        return self.n_fft // 2 + 1

    def frames_for(self, samples: int) -> int:
        if self.center:
            return samples // self.hop_length + 1
        return max(0, (samples - self.n_fft) // self.hop_length + 1)

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


def hz_to_mel(frequency: torch.Tensor) -> torch.Tensor:
    f = frequency
    return torch.where(f < _BREAK_HZ, f / _HZ_PER_MEL,
                       _BREAK_MEL + torch.log(torch.clamp(f / _BREAK_HZ, min=1e-10)) / _LOG_STEP)


def mel_to_hz(mel: torch.Tensor) -> torch.Tensor:
    return torch.where(mel < _BREAK_MEL, mel * _HZ_PER_MEL, _BREAK_HZ * torch.exp(_LOG_STEP * (mel - _BREAK_MEL)))


@lru_cache(maxsize=16)
def _bank(num_bins: int, n_mels: int, sample_rate: int, f_min: float, f_max: float) -> torch.Tensor:
    freqs = torch.linspace(0.0, sample_rate / 2.0, num_bins, dtype=torch.float64)
    lo, hi = hz_to_mel(torch.tensor([f_min, f_max], dtype=torch.float64)).tolist()
    centres = mel_to_hz(torch.linspace(lo, hi, n_mels + 2, dtype=torch.float64))
    left, mid, right = centres[:-2], centres[1:-1], centres[2:]
    up = (freqs[:, None] - left[None]) / (mid - left)[None]
    down = (right[None] - freqs[:, None]) / (right - mid)[None]
    tri = torch.clamp(torch.minimum(up, down), min=0.0)
    return (tri * (2.0 / (right - left))[None]).float()  # [bins, mels], area-normalised


def mel_filterbank(config: MelConfig, *, device: torch.device | str = "cpu",
                   dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """``[num_bins, n_mels]`` filter matrix."""
    return _bank(config.num_bins, config.n_mels, config.sample_rate, float(config.f_min),
                 config.upper_hz).to(device=device, dtype=dtype)


@lru_cache(maxsize=16)
def _window(win: int, n_fft: int) -> torch.Tensor:
    w = torch.hann_window(win, periodic=True, dtype=torch.float64)
    pad = n_fft - win
    return torch.nn.functional.pad(w, (pad // 2, pad - pad // 2)).float()


def stft_magnitude(waveform: torch.Tensor, config: MelConfig) -> torch.Tensor:
    """``|STFT|^power`` of ``(..., samples)`` as ``(..., bins, frames)`` in fp32."""
    lead = waveform.shape[:-1]
    x = waveform.reshape(-1, waveform.shape[-1]).float()
    spec = torch.stft(x, n_fft=config.n_fft, hop_length=config.hop_length, win_length=config.n_fft,
                      window=_window(config.window_length, config.n_fft).to(x.device), center=config.center,
                      pad_mode="reflect", normalized=config.normalized, return_complex=True)
    mag = spec.abs()
    if config.power != 1.0:
        mag = mag.pow(config.power)
    return mag.reshape(*lead, *mag.shape[-2:])


class MelFrontend:
    """Waveform ``(..., samples)`` -> mel ``(..., n_mels, frames)``."""

    def __init__(self, config: MelConfig | None = None) -> None:
        self.config = config or MelConfig()

    @property
    def mel_bins(self) -> int:
        return self.config.n_mels

    @property
    def sample_rate(self) -> int:
        return self.config.sample_rate

    def filterbank(self, *, device: torch.device, dtype: torch.dtype) -> torch.Tensor:
        return mel_filterbank(self.config, device=device, dtype=dtype)

    def __call__(self, waveform: torch.Tensor) -> torch.Tensor:
        mag = stft_magnitude(waveform, self.config)
        bank = self.filterbank(device=mag.device, dtype=mag.dtype)
        return torch.einsum("...bf,bm->...mf", mag, bank)

    def log_mel(self, waveform: torch.Tensor) -> torch.Tensor:
        return torch.log(torch.clamp(self(waveform), min=self.config.log_epsilon))
