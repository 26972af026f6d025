"""Dense synthetic batches of a fixed shape (benchmarks, smoke tests).

Latents and text embeddings are i.i.d. N(0, 1), every token valid, frame
positions at ``fps``. :class:`avgen_b200.data.synthetic.SyntheticSource` is the
learnable, resumable procedural source; this helper only fixes shapes.
"""
from __future__ import annotations

import torch

from avgen_b200.core.batch import MediaBatch, MediaBatchSpec

__all__ = ["random_batch"]


def random_batch(*, batch: int, channels: int, frames: int, height: int, width: int, text_tokens: int,
                 text_width: int, fps: float = 24.0, generator: torch.Generator | None = None,
                 device: torch.device | str = "cpu", dtype: torch.dtype = torch.float32,
                 pin: bool = False, sample_offset: int = 0) -> MediaBatch:
    """A video-only batch with ``(batch, channels, frames, height, width)`` latents."""
    spec = MediaBatchSpec(schema_version=1, bucket_id=0, video_shape=(batch, channels, frames, height, width),
                          audio_shape=(batch, 1, 0), text_shape=(batch, text_tokens, text_width),
                          video_timebase_num=int(round(fps * 1000)), video_timebase_den=1000,
                          audio_timebase_num=1, audio_timebase_den=1, video_codec_id="synthetic",
                          audio_codec_id="none")
    g = generator
    dev = torch.device(device)

    def randn(*shape: int) -> torch.Tensor:
        return torch.randn(shape, generator=g, dtype=torch.float32).to(dtype)

    video = randn(batch, channels, frames, height, width)
    text = randn(batch, text_tokens, text_width)
    positions = (torch.arange(frames, dtype=torch.float32) / fps)[None].expand(batch, frames).contiguous()
    out = MediaBatch(video=video, audio=torch.zeros((batch, 1, 0), dtype=dtype), text=text,
                     video_mask=torch.ones((batch, frames, height, width), dtype=torch.bool),
                     audio_mask=torch.zeros((batch, 0), dtype=torch.bool), video_positions=positions,
                     audio_positions=torch.zeros((batch, 0), dtype=torch.float32),
                     sample_ids=torch.arange(sample_offset, sample_offset + batch, dtype=torch.int64), spec=spec,
                     text_mask=torch.ones((batch, text_tokens), dtype=torch.bool))
    if pin:
        out = out.pin_memory()
    if dev.type != "cpu":
        out = out.to(dev)
    return out
