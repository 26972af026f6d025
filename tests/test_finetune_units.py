"""Fine-tuning units on CPU against closed forms: LoRA's delta and scaling, the
effective weight with and without DoRA, merge / unmerge as exact inverses,
dropout-path equivalence, rank / alpha patterns, adapter save / load, freezing
helpers and the trainable summary (reference test strategy:
tests/test_finetune*.py)."""
from __future__ import annotations

from pathlib import Path

import pytest
import torch
import torch.nn.functional as F
from torch import nn

from avgen_b200.finetune.freeze import freeze_all, freeze_except, freeze_matching, trainable_summary
from avgen_b200.finetune.lora import (LoRAConfig, LoRALinear, adapter_state_dict, apply_lora, load_adapter,
                                      lora_modules, lora_parameters, mark_only_lora_trainable, merge_lora,
                                      save_adapter, unmerge_lora)


def _layer(rank: int = 4, alpha: float = 8.0, dora: bool = False, seed: int = 0) -> LoRALinear:
    torch.manual_seed(seed)
    base = nn.Linear(12, 10)
    layer = LoRALinear.from_linear(base, rank=rank, alpha=alpha, use_dora=dora)
    with torch.no_grad():
        layer.lora_b.normal_(0, 0.1)
    return layer


@pytest.mark.parametrize("rank,alpha", [(1, 1.0), (4, 8.0), (8, 4.0)])
def test_lora_delta_and_forward(rank: int, alpha: float) -> None:
    layer = _layer(rank, alpha)
    assert layer.scaling == alpha / rank
    delta = layer.lora_b @ layer.lora_a * (alpha / rank)
    torch.testing.assert_close(layer.lora_delta(), delta)
    x = torch.randn(3, 12)
    torch.testing.assert_close(layer(x), F.linear(x, layer.weight + delta, layer.bias))


def test_lora_starts_at_the_base_layer() -> None:
    torch.manual_seed(0)
    base = nn.Linear(12, 10)
    layer = LoRALinear.from_linear(base, rank=4, alpha=8.0)
    x = torch.randn(5, 12)
    torch.testing.assert_close(layer(x), base(x))  # B starts at zero
    assert layer.weight is base.weight


@pytest.mark.parametrize("init", ["kaiming", "gaussian", "zeros"])
def test_lora_init_modes(init: str) -> None:
    layer = LoRALinear.from_linear(nn.Linear(12, 10), rank=4, alpha=4.0, init=init)
    assert bool((layer.lora_b == 0).all())
    if init == "zeros":
        assert bool((layer.lora_a == 0).all())
    else:
        assert float(layer.lora_a.detach().abs().max()) > 0
    with pytest.raises(ValueError):
        layer.reset_lora_parameters("orthogonal")


def test_dora_effective_weight_has_the_magnitude_row_norms() -> None:
    layer = _layer(dora=True)
    w = layer.adapted_weight()
    torch.testing.assert_close(w.norm(dim=1), layer.lora_magnitude.detach(), rtol=1e-5, atol=1e-6)
    # at initialisation the magnitude equals the base rows' norms
    fresh = LoRALinear.from_linear(nn.Linear(12, 10), rank=2, alpha=2.0, use_dora=True)
    torch.testing.assert_close(fresh.lora_magnitude.detach(), fresh.weight.norm(dim=1))
    torch.testing.assert_close(fresh.adapted_weight(), fresh.weight)
    with pytest.raises(RuntimeError):
        _layer().reset_dora_magnitude()


@pytest.mark.parametrize("dora", [False, True])
def test_merge_unmerge_are_inverse(dora: bool) -> None:
    layer = _layer(dora=dora)
    x = torch.randn(4, 12)
    before = layer(x).detach()
    w0 = layer.weight.detach().clone()
    layer.merge()
    assert layer.merged
    torch.testing.assert_close(layer(x), before, rtol=1e-5, atol=1e-6)
    with pytest.raises(RuntimeError):
        layer.merge()
    layer.unmerge()
    torch.testing.assert_close(layer.weight, w0, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(layer(x), before, rtol=1e-5, atol=1e-6)
    with pytest.raises(RuntimeError):
        layer.unmerge()


def test_dropout_path_matches_effective_weight_in_eval() -> None:
    torch.manual_seed(1)
    layer = LoRALinear.from_linear(nn.Linear(12, 10), rank=4, alpha=8.0, dropout=0.5)
    with torch.no_grad():
        layer.lora_b.normal_(0, 0.1)
    layer.eval()
    x = torch.randn(3, 12)
    torch.testing.assert_close(layer(x), F.linear(x, layer.adapted_weight(), layer.bias), rtol=1e-5, atol=1e-6)
    layer.train()
    torch.manual_seed(2)
    y1 = layer(x)
    torch.manual_seed(3)
    y2 = layer(x)
    assert not torch.allclose(y1, y2)  # the adapter path sees fresh dropout masks


@pytest.mark.parametrize("kw", [{"rank": 0}, {"alpha": 0.0}, {"dropout": 1.0}, {"init_lora_weights": "xavier"},
                                {"target_modules": ()}, {"rank_pattern": (("q_proj", 0),)}])
def test_lora_config_rejects(kw: dict) -> None:
    with pytest.raises(ValueError):
        LoRAConfig(**kw)


def test_lora_config_patterns_and_metadata() -> None:
    cfg = LoRAConfig(rank=8, alpha=16.0, target_modules=("q_proj", "v_proj"), exclude_modules=("blocks.1.*",),
                     rank_pattern=(("*.v_proj", 2),), alpha_pattern=(("*.v_proj", 4.0),))
    assert cfg.rank_for("blocks.0.attention.q_proj") == 8 and cfg.rank_for("blocks.0.attention.v_proj") == 2
    assert cfg.alpha_for("blocks.0.attention.v_proj") == 4.0 and cfg.alpha_for("x.q_proj") == 16.0
    assert cfg.selects("blocks.0.attention.q_proj") and not cfg.selects("blocks.0.attention.k_proj")
    assert "lora_config" in cfg.to_metadata()


class _Tiny(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.q_proj = nn.Linear(8, 8)
        self.v_proj = nn.Linear(8, 8)
        self.other = nn.Linear(8, 8)
        self.norm = nn.LayerNorm(8)


def test_apply_lora_selects_modules_and_trains_only_adapters() -> None:
    model = _Tiny()
    apply_lora(model, LoRAConfig(rank=2, alpha=4.0, target_modules=("q_proj", "v_proj")))
    names = [n for n, _ in lora_modules(model)]
    assert names == ["q_proj", "v_proj"] and isinstance(model.q_proj, LoRALinear)
    assert not isinstance(model.other, LoRALinear)
    mark_only_lora_trainable(model)
    trainable = {n for n, p in model.named_parameters() if p.requires_grad}
    assert trainable == {"q_proj.lora_a", "q_proj.lora_b", "v_proj.lora_a", "v_proj.lora_b"}
    assert len(lora_parameters(model)) == 4
    s = trainable_summary(model)
    assert s.trainable == 4 * 2 * 8 and s.percentage < 50 and "trainable" in s.describe()


def test_merge_lora_strip_and_adapter_round_trip(tmp_path: Path) -> None:
    torch.manual_seed(0)
    model = _Tiny()
    apply_lora(model, LoRAConfig(rank=2, alpha=4.0, target_modules=("q_proj",)))
    with torch.no_grad():
        model.q_proj.lora_b.normal_(0, 0.1)
    x = torch.randn(2, 8)
    want = model.q_proj(x).detach()
    state = adapter_state_dict(model)
    assert set(state) == {"q_proj.lora_a", "q_proj.lora_b"}
    save_adapter(tmp_path / "adapter", model)
    other = _Tiny()
    other.load_state_dict({k: v for k, v in model.state_dict().items() if "lora" not in k}, strict=False)
    apply_lora(other, LoRAConfig(rank=2, alpha=4.0, target_modules=("q_proj",)))
    load_adapter(tmp_path / "adapter", other)
    torch.testing.assert_close(other.q_proj(x), want)
    merge_lora(model)
    torch.testing.assert_close(model.q_proj(x), want, rtol=1e-5, atol=1e-6)
    unmerge_lora(model)
    torch.testing.assert_close(model.q_proj(x), want, rtol=1e-5, atol=1e-6)
    stripped = merge_lora(model, strip=True)
    assert not any(isinstance(m, LoRALinear) for m in stripped.modules())
    torch.testing.assert_close(stripped.q_proj(x), want, rtol=1e-5, atol=1e-6)


# ----------------------------------------------------------------------------- freezing


def test_freeze_helpers() -> None:
    model = _Tiny()
    total = sum(p.numel() for p in model.parameters())
    assert freeze_all(model) == total and trainable_summary(model).trainable == 0
    s = freeze_except(model, ["q_proj.*"])
    assert s.trainable == 8 * 8 + 8 and s.trainable_tensors == 2
    with pytest.raises(ValueError):
        freeze_except(model, [])
    with pytest.raises(ValueError):
        freeze_except(model, ["nothing_matches"])
    for p in model.parameters():
        p.requires_grad_(True)
    s = freeze_matching(model, ["norm.*", "other.*"])
    assert s.frozen == 2 * 8 + 8 * 8 + 8 and s.total == total
    assert trainable_summary(model).optimizer_state_bytes == 12 * s.trainable


def test_stage_overrides_copy_and_plain_description() -> None:
    import json

    from avgen_b200.finetune.stages import get_stage, list_stages

    for name in list_stages():
        stage = get_stage(name)
        described = stage.to_dict()
        json.dumps(described)  # JSON-safe all the way down
        assert described["name"] == name and abs(sum(described["conditioning_mix"].values()) - 1.0) < 1e-9
        assert described["uses_adapter"] == stage.uses_adapter
    base = get_stage(list_stages()[0])
    changed = base.with_overrides(learning_rate=3e-6, notes="borrowed")
    assert changed.learning_rate == 3e-6 and changed.notes == "borrowed"
    assert base.learning_rate != 3e-6 and get_stage(base.name) == base  # the registered recipe is untouched
    with pytest.raises(ValueError):
        base.with_overrides(learning_rate=0.0)  # validation runs on the copy
