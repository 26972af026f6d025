"""LoRA / DoRA semantics, adapter files, freezing, stages, control and IP adapters (CPU)."""
from __future__ import annotations

from dataclasses import asdict
from pathlib import Path

import pytest
import torch
from torch import nn

from avgen_b200.finetune import (ControlAdapter, ControlAdapterConfig, IPAdapter, IPAdapterConfig, LoRAConfig,
                                 LoRALinear, apply_lora, apply_stage, freeze_except, get_stage, list_stages,
                                 load_adapter, lora_parameters, mark_only_lora_trainable, merge_lora, save_adapter,
                                 trainable_summary, unmerge_lora)


def _model():  # noqa: ANN202
    from avgen_b200.models import build_model, preset

    torch.manual_seed(0)
    m = build_model("video_dit", {k: v for k, v in asdict(preset("tiny")).items() if k != "rope_scaling"})
    m.init_weights()
    with torch.no_grad():
        for p in m.parameters():
            p.add_(0.02 * torch.randn_like(p))
    return m


def _inputs(model):  # noqa: ANN001, ANN202
    from avgen_b200.core.tokens import TextContext
    from avgen_b200.infer.conditioning import StreamState, build_model_input

    g = torch.Generator().manual_seed(3)
    c = model.config
    lat = torch.randn(1, c.in_channels, 2, 8, 8, generator=g)
    text = TextContext(features=torch.randn(1, 5, c.text_width, generator=g), mask=torch.ones(1, 5, dtype=torch.bool))
    return build_model_input(video=StreamState(lat, fps=8.0), sigma=0.5, text=text, patchifier=model.patchifier)


@pytest.mark.parametrize("dora", [False, True])
def test_lora_starts_at_base_and_merges_exactly(dora: bool) -> None:
    torch.manual_seed(1)
    base = nn.Linear(16, 12)
    x = torch.randn(5, 16)
    lora = LoRALinear.from_linear(base, rank=4, alpha=8.0, use_dora=dora)
    torch.testing.assert_close(lora(x), base(x))
    with torch.no_grad():
        lora.lora_b.normal_()
    y = lora(x)
    w0 = lora.weight.detach().clone()
    lora.merge()
    torch.testing.assert_close(lora(x), y, rtol=1e-5, atol=1e-5)
    lora.unmerge()
    torch.testing.assert_close(lora.weight, w0, rtol=1e-5, atol=1e-6)
    y.sum().backward()
    assert lora.lora_a.grad is not None and lora.lora_b.grad is not None


def test_apply_lora_keeps_checkpoint_keys_and_roundtrips_adapter(tmp_path: Path) -> None:
    model = _model()
    keys = set(model.state_dict())
    inputs = _inputs(model)
    before = model(inputs).video.detach()
    apply_lora(model, LoRAConfig(rank=4, alpha=8.0))
    assert keys <= set(model.state_dict())
    torch.testing.assert_close(model(inputs).video, before)  # B = 0: identical at start
    n = mark_only_lora_trainable(model)
    assert n == sum(p.numel() for p in lora_parameters(model))
    with torch.no_grad():
        for p in lora_parameters(model):
            p.normal_(std=0.05)
    adapted = model(inputs).video.detach()
    path = save_adapter(tmp_path / "a.safetensors", model, config=LoRAConfig(rank=4, alpha=8.0))
    other = _model()
    apply_lora(other, LoRAConfig(rank=4, alpha=8.0))
    meta = load_adapter(path, other)
    assert meta["lora_config"]["rank"] == 4
    torch.testing.assert_close(other(inputs).video, adapted)
    merge_lora(other, strip=True)
    assert not any(isinstance(m, LoRALinear) for m in other.modules())
    torch.testing.assert_close(other(inputs).video, adapted, rtol=1e-4, atol=1e-5)


def test_freeze_and_stages() -> None:
    model = _model()
    s = freeze_except(model, ["q_proj", "final_proj"])
    assert 0 < s.trainable < s.total and "trainable" in s.describe()
    assert {"full", "lora", "control", "resolution_adaptation", "duration_extension", "distillation"} <= set(
        list_stages())
    m2 = _model()
    apply_stage(m2, get_stage("lora"))
    assert any(isinstance(m, LoRALinear) for m in m2.modules())
    assert trainable_summary(m2).trainable == sum(p.numel() for p in lora_parameters(m2))
    with pytest.raises(KeyError):
        get_stage("nope")


def test_control_adapter_starts_as_identity() -> None:
    model = _model()
    inputs = _inputs(model)
    ref = model(inputs).video.detach()
    adapter = ControlAdapter(model, ControlAdapterConfig(control_width=model.config.width, num_blocks=1))
    n = inputs.video.length
    control = torch.randn(1, n, model.config.width)
    with adapter.attach(model, control):
        out = model(inputs).video
    torch.testing.assert_close(out, ref)  # zero injections
    out.sum().backward()
    assert adapter.injections[0].weight.grad is not None


def test_ip_adapter_starts_as_identity() -> None:
    model = _model()
    inputs = _inputs(model)
    ref = model(inputs).video.detach()
    ip = IPAdapter(model, IPAdapterConfig(image_width=32, num_tokens=2))
    with ip.attach(model, torch.randn(1, 32)):
        out = model(inputs).video
    torch.testing.assert_close(out, ref)
    out.sum().backward()
    assert ip.to_out[0].weight.grad is not None
