"""The adapter contract (the reference's tests/test_kernels_registry.py behaviours), no device needed."""

from __future__ import annotations

from dataclasses import dataclass

import pytest
import torch
from torch import nn

from prismyra_b200 import kernels
from prismyra_b200.kernels import AdapterError, Applied, Swap


@dataclass
class FakeConfig:
    architectures: list
    num_hidden_layers: int = 0
    num_experts: int = 0
    num_experts_per_tok: int = 0
    hidden_size: int = 0
    moe_intermediate_size: int = 0


QWEN = dict(num_experts=128, num_experts_per_tok=8, hidden_size=2048, moe_intermediate_size=768)


def test_an_unknown_architecture_runs_without_the_kernels_by_default():
    applied = kernels.apply(nn.Linear(2, 2), FakeConfig(architectures=["SomethingElse"]))
    assert applied.adapter == "none" and applied.skipped


def test_an_unknown_architecture_can_be_made_fatal():
    with pytest.raises(AdapterError, match="no adapter"):
        kernels.apply(nn.Linear(2, 2), FakeConfig(architectures=["SomethingElse"]), required=True)


def test_a_wrong_count_fails_closed():
    class Miscounting:
        name = "miscounting"

        def supports(self, config):
            return True

        def replace(self, model, config):
            return Applied(adapter=self.name, swaps=[Swap("thing", replaced=3, expected=40)])

    kernels._ADAPTERS.insert(0, Miscounting())
    try:
        with pytest.raises(AdapterError, match="replaced 3 of an expected 40"):
            kernels.apply(nn.Linear(2, 2), FakeConfig(architectures=["Whatever"]))
    finally:
        kernels._ADAPTERS.pop(0)


def test_required_means_required_even_when_every_module_was_found():
    class Partial:
        name = "partial"

        def supports(self, config):
            return True

        def replace(self, model, config):
            return Applied(adapter=self.name, swaps=[Swap("norm", 4, 4)], skipped=["not built"])

    kernels._ADAPTERS.insert(0, Partial())
    try:
        assert kernels.apply(nn.Identity(), FakeConfig(architectures=["P"])).skipped
        with pytest.raises(AdapterError, match="could not apply every kernel"):
            kernels.apply(nn.Identity(), FakeConfig(architectures=["P"]), required=True)
    finally:
        kernels._ADAPTERS.pop(0)


def test_applied_reports_as_data():
    a = Applied(adapter="x", swaps=[Swap("a", 2, 2), Swap("b", 1, None, verified="self-check")], skipped=["c"])
    d = a.as_dict()
    assert d["complete"] is False and d["applied"] == {"a": 2, "b": 1} and d["verified"] == {"b": "self-check"}
    assert a.ok and "a=2" in a.summary() and "skipped=c" in a.summary()
    assert not hasattr(a, "ms")


def test_the_qwen_adapter_claims_only_shapes_the_kernels_accept():
    ok = FakeConfig(architectures=["Qwen3_5MoeForConditionalGeneration"], num_hidden_layers=36, **QWEN)
    assert kernels.find(ok).name == "qwen3-moe-b200"
    assert kernels.find(FakeConfig(architectures=["LlamaForCausalLM"], num_hidden_layers=36, **QWEN)) is None
    for bad in (dict(QWEN, num_experts=512), dict(QWEN, hidden_size=2000), dict(QWEN, moe_intermediate_size=700),
                dict(QWEN, num_experts_per_tok=32)):
        assert kernels.find(FakeConfig(architectures=["Qwen3_5MoeForCausalLM"], num_hidden_layers=36, **bad)) is None
    # the reference's own checkpoint shape (256 experts, I=512) is accepted too
    ref = dict(QWEN, num_experts=256, moe_intermediate_size=512)
    assert kernels.find(FakeConfig(architectures=["Qwen3_5MoeForCausalLM"], num_hidden_layers=40, **ref))


class Qwen3_5MoeSparseMoeBlock(nn.Module):  # matched by class name, like the framework's block
    def __init__(self, fp8=True):
        super().__init__()
        self.gate = nn.Linear(256, 8, bias=False)
        self.shared_expert = nn.Identity()
        self.shared_expert_gate = nn.Linear(256, 1, bias=False)
        self.experts = nn.Module()
        dt = torch.float8_e4m3fn if fp8 else torch.bfloat16
        self.experts.gate_up_proj = nn.Parameter(torch.zeros(8, 256, 256).to(dt), requires_grad=False)
        self.experts.down_proj = nn.Parameter(torch.zeros(8, 256, 128).to(dt), requires_grad=False)
        if fp8:
            self.experts.gate_up_proj_scale_inv = nn.Parameter(torch.ones(8, 2, 2), requires_grad=False)
            self.experts.down_proj_scale_inv = nn.Parameter(torch.ones(8, 2, 1), requires_grad=False)


def test_non_fp8_experts_are_skipped_not_half_replaced():
    model = nn.Sequential(Qwen3_5MoeSparseMoeBlock(fp8=False), Qwen3_5MoeSparseMoeBlock(fp8=False))
    cfg = FakeConfig(architectures=["Qwen3_5MoeForCausalLM"], num_hidden_layers=2, num_experts=8,
                     num_experts_per_tok=4, hidden_size=256, moe_intermediate_size=128)
    applied = kernels.apply(model, cfg)
    assert applied.skipped and all(type(m).__name__ == "Qwen3_5MoeSparseMoeBlock" for m in model)
    with pytest.raises(AdapterError):
        kernels.apply(model, cfg, required=True)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device branch")
def test_fp8_model_without_a_device_is_skipped():
    model = nn.Sequential(Qwen3_5MoeSparseMoeBlock(), Qwen3_5MoeSparseMoeBlock())
    cfg = FakeConfig(architectures=["Qwen3_5MoeForCausalLM"], num_hidden_layers=2, num_experts=8,
                     num_experts_per_tok=4, hidden_size=256, moe_intermediate_size=128)
    applied = kernels.apply(model, cfg)
    assert applied.skipped == ["no CUDA device: the B200 kernels need one"]
