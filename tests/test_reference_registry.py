"""The drop-in through the reference's own plugin registry: the reference's ``prismyra.kernels`` module (its
``register`` / ``find`` / ``apply`` and its ``AdapterError``), with this repository's adapter inserted ahead of the
reference's own, the way INTEGRATION.md tells a maintainer to bind it, on transformers' own Qwen3.5-MoE blocks.

Runs where the reference checkout is available (``PRISMYRA_REFERENCE_DIR``, else a ``reference`` checkout beside this
repository) and no GPU is visible: on a host without CUDA the adapter must decline through the registry's
fail-closed rules (``required=True`` raises the reference's AdapterError; otherwise the skip is reported)."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch
from torch import nn

from prismyra_b200 import synth


def _reference_root() -> Path | None:
    for cand in (os.environ.get("PRISMYRA_REFERENCE_DIR"), Path(__file__).resolve().parents[2] / "reference"):
        if cand and (Path(cand) / "prismyra" / "kernels" / "__init__.py").exists():
            return Path(cand)
    return None


ROOT = _reference_root()
pytestmark = [pytest.mark.skipif(ROOT is None, reason="the reference checkout is not available here"),
              pytest.mark.skipif(torch.cuda.is_available(), reason="checks the registry's no-device path")]


@pytest.fixture(scope="module")
def ref_kernels():
    sys.path.insert(0, str(ROOT))
    try:
        import prismyra.kernels as rk
    except Exception as e:  # pragma: no cover - the reference's optional dependencies are missing
        pytest.skip(f"the reference's kernels package does not import here: {e}")
    from prismyra_b200.kernels.qwen3_moe import Qwen3MoeAdapter as B200MoeAdapter

    adapter = B200MoeAdapter()
    rk._ADAPTERS.insert(0, adapter)
    yield rk, adapter
    rk._ADAPTERS.remove(adapter)
    sys.path.remove(str(ROOT))


def _config(**kw):
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig

    cfg = Qwen3_5MoeTextConfig(hidden_size=256, moe_intermediate_size=128, num_experts=8, num_experts_per_tok=4,
                               num_hidden_layers=2, shared_expert_intermediate_size=128, num_attention_heads=2,
                               num_key_value_heads=1, head_dim=64, vocab_size=128,
                               layer_types=["full_attention", "full_attention"], **kw)
    cfg.architectures = ["Qwen3_5MoeForCausalLM"]
    return cfg


def _blocks(cfg, fp8: bool) -> nn.Module:
    """Two of transformers' own Qwen3_5MoeSparseMoeBlock, their expert stacks as 128x128 block-FP8 (the attribute
    names the reference's FusedExperts reads) when fp8."""
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeSparseMoeBlock

    model = nn.ModuleList([Qwen3_5MoeSparseMoeBlock(cfg) for _ in range(cfg.num_hidden_layers)])
    if fp8:
        for i, blk in enumerate(model):
            g = torch.Generator().manual_seed(i)
            w1, s1 = synth.quantize_fp8_blocks(torch.randn(8, 256, 256, generator=g) * 0.02)
            w2, s2 = synth.quantize_fp8_blocks(torch.randn(8, 256, 128, generator=g) * 0.02)
            blk.experts.gate_up_proj = nn.Parameter(w1, requires_grad=False)
            blk.experts.down_proj = nn.Parameter(w2, requires_grad=False)
            blk.experts.gate_up_proj_scale_inv = nn.Parameter(s1, requires_grad=False)
            blk.experts.down_proj_scale_inv = nn.Parameter(s2, requires_grad=False)
    return model


def test_the_reference_registry_finds_the_b200_adapter_first(ref_kernels):
    rk, adapter = ref_kernels
    assert rk.find(_config()) is adapter
    assert rk._ADAPTERS[0] is adapter and len(rk._ADAPTERS) >= 2  # the reference's own adapter is still registered


def test_without_a_device_the_reference_apply_reports_the_skip(ref_kernels):
    rk, _ = ref_kernels
    cfg = _config()
    model = _blocks(cfg, fp8=True)
    applied = rk.apply(model, cfg)
    assert applied.adapter == "qwen3-moe-b200"
    assert applied.skipped == ["no CUDA device: the B200 kernels need one"]
    assert applied.as_dict()["complete"] is False
    assert all(type(m).__name__ == "Qwen3_5MoeSparseMoeBlock" for m in model)  # nothing half-replaced


def test_required_kernels_fail_closed_with_the_reference_error(ref_kernels):
    rk, _ = ref_kernels
    cfg = _config()
    with pytest.raises(rk.AdapterError, match="could not apply every kernel"):
        rk.apply(_blocks(cfg, fp8=True), cfg, required=True)


def test_bf16_experts_are_declined_through_the_reference_registry(ref_kernels):
    rk, _ = ref_kernels
    cfg = _config()
    applied = rk.apply(_blocks(cfg, fp8=False), cfg)
    assert applied.skipped == ["routed experts are not 128x128 block-FP8 (the B200 FP8 kernels need them)"]
    with pytest.raises(rk.AdapterError):
        rk.apply(_blocks(cfg, fp8=False), cfg, required=True)
