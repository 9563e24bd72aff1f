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


def _fp8_linear_module(out_f, in_f, scale_shape=None):
    from transformers.integrations.finegrained_fp8 import FP8Linear

    m = FP8Linear(in_f, out_f, block_size=(128, 128))
    m.weight = nn.Parameter(torch.zeros(out_f, in_f).to(torch.float8_e4m3fn), requires_grad=False)
    m.weight_scale_inv = nn.Parameter(torch.ones(scale_shape or (out_f // 128, in_f // 128)), requires_grad=False)
    return m


class _SharedMLP(nn.Module):
    def __init__(self, H, Is, fp8=True):
        super().__init__()
        from transformers.activations import ACT2FN

        if fp8:
            self.gate_proj, self.up_proj = _fp8_linear_module(Is, H), _fp8_linear_module(Is, H)
            self.down_proj = _fp8_linear_module(H, Is)
        else:
            self.gate_proj, self.up_proj = nn.Linear(H, Is, bias=False), nn.Linear(H, Is, bias=False)
            self.down_proj = nn.Linear(Is, H, bias=False)
        self.act_fn = ACT2FN["silu"]


def _block_with_shared(fp8_shared=True, Is=128):
    blk = Qwen3_5MoeSparseMoeBlock()
    blk.shared_expert = _SharedMLP(256, Is, fp8_shared)
    blk.shared_expert_gate = nn.Linear(256, 1, bias=False).to(torch.bfloat16)
    return blk


def test_fused_experts_runs_a_block_fp8_shared_expert_in_the_library_and_keeps_others():
    """FusedExperts takes the shared expert into the library call only when its projections are bias-free
    block-FP8 with a bf16 one-row gate; anything else stays the framework's module (built on CPU: construction
    touches no device)."""
    from prismyra_b200.kernels.qwen3_moe import FusedExperts

    mod = FusedExperts(_block_with_shared(), 4)
    assert mod.shared_fp8 is not None
    w_sg, w13, s13, w2, s2 = mod.shared_fp8
    assert w_sg.shape == (256,) and w13.shape == (256, 256) and s13.shape == (2, 2)
    assert w2.shape == (256, 128) and s2.shape == (2, 1) and s13.dtype == torch.float32
    assert FusedExperts(_block_with_shared(fp8_shared=False), 4).shared_fp8 is None
    odd = _block_with_shared()
    odd.shared_expert.act_fn = nn.GELU()
    assert FusedExperts(odd, 4).shared_fp8 is None
    biased = _block_with_shared()
    biased.shared_expert.down_proj.bias = nn.Parameter(torch.zeros(256))
    assert FusedExperts(biased, 4).shared_fp8 is None


def test_dense_projection_modules_check_their_shapes():
    from prismyra_b200.kernels.qwen3_moe import Fp8Linear, FusedDenseProjection

    lin = Fp8Linear(_fp8_linear_module(512, 256))
    assert (lin.out_features, lin.in_features) == (512, 256) and lin.scale.dtype == torch.float32
    with pytest.raises(AdapterError):
        Fp8Linear(_fp8_linear_module(384, 256))  # output width not a multiple of 256
    with pytest.raises(AdapterError):
        Fp8Linear(nn.Linear(256, 256, bias=False))  # not FP8
    with pytest.raises(AdapterError):
        Fp8Linear(_fp8_linear_module(256, 256, scale_shape=(1, 1)))  # per-tensor scale
    fused = FusedDenseProjection([lin, Fp8Linear(_fp8_linear_module(256, 256))])
    assert fused.sizes == [512, 256] and fused.weight.shape == (768, 256) and fused.scale.shape == (6, 2)
    with pytest.raises(AdapterError):
        FusedDenseProjection([lin, Fp8Linear(_fp8_linear_module(256, 512))])  # different input widths


class FusedExperts(nn.Module):  # matched by class name, like the adapter's installed module
    """A stand-in for the installed routed-expert module whose repeat behaviour the test chooses."""

    def __init__(self, behaviour: str):
        super().__init__()
        self.hidden = 256
        self.w1 = torch.zeros(1)
        self.behaviour = behaviour
        self.calls = 0

    def forward(self, x):
        self.calls += 1
        if self.behaviour == "oom":
            raise torch.OutOfMemoryError("CUDA out of memory. Tried to allocate 2.00 GiB")
        if self.behaviour == "error":
            raise RuntimeError("launch failed")
        out = x * 2
        if self.behaviour == "flaky" and self.calls == 5:
            out = out + 1e-2
        return out


def test_fp8_determinism_probe_accepts_a_kernel_that_repeats_itself():
    from prismyra_b200.kernels import qwen3_moe as q

    m = FusedExperts("stable")
    applied = Applied(adapter="t")
    q._check_fp8_determinism(applied, nn.Sequential(m))
    assert m.calls == q.FP8_DETERMINISM_PROBES == 8
    assert any("agreed bit for bit" in n for n in applied.notes) and not applied.skipped


def test_fp8_determinism_probe_refuses_a_device_that_does_not():
    from prismyra_b200.kernels import qwen3_moe as q

    with pytest.raises(AdapterError, match="differently in 1 of 7"):
        q._check_fp8_determinism(Applied(adapter="t"), nn.Sequential(FusedExperts("flaky")))


def test_fp8_determinism_probe_out_of_memory_is_an_adapter_error_not_a_fallback():
    from prismyra_b200.kernels import qwen3_moe as q

    with pytest.raises(AdapterError, match="ran out of GPU memory"):
        q._check_fp8_determinism(Applied(adapter="t"), nn.Sequential(FusedExperts("oom")))


def test_fp8_determinism_probe_that_cannot_run_is_recorded_as_a_skip():
    from prismyra_b200.kernels import qwen3_moe as q

    applied = Applied(adapter="t")
    q._check_fp8_determinism(applied, nn.Sequential(FusedExperts("error")))
    assert applied.skipped == ["fp8_determinism: the probe raised RuntimeError: launch failed -- not checked"]
    applied = Applied(adapter="t")
    q._check_fp8_determinism(applied, nn.Sequential(nn.Identity()))
    assert applied.notes == ["fp8_determinism: nothing matched (no FusedExperts installed)"]


def test_the_probe_can_be_withheld_like_the_reference(monkeypatch):
    from prismyra_b200.kernels import qwen3_moe as q

    monkeypatch.setenv("PRISMYRA_WITHOUT", "dense_fusion, fp8_determinism")
    assert q._withheld() == {"dense_fusion", "fp8_determinism"}
    monkeypatch.delenv("PRISMYRA_WITHOUT")
    assert q._withheld() == set()


def test_fused_experts_act_scale_option(monkeypatch):
    from prismyra_b200.kernels.qwen3_moe import FusedExperts as FE

    blk = Qwen3_5MoeSparseMoeBlock()
    assert FE(blk, 4).act_scale == "fp32"
    assert FE(Qwen3_5MoeSparseMoeBlock(), 4, act_scale="ue8m0").act_scale == "ue8m0"
    monkeypatch.setenv("PRISMYRA_B200_ACT_SCALE", "ue8m0")
    assert FE(Qwen3_5MoeSparseMoeBlock(), 4).act_scale == "ue8m0"
    monkeypatch.setenv("PRISMYRA_B200_ACT_SCALE", "fp16")
    with pytest.raises(AdapterError, match="act_scale"):
        FE(Qwen3_5MoeSparseMoeBlock(), 4)
