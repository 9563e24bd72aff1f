"""The adapter on a GPU, on transformers' own Qwen3.5-MoE blocks with 128x128 block-FP8 expert stacks: apply swaps
every block for FusedExperts, runs the reference's 8-call self-repeat probe (it must agree bit for bit), and the
installed module's routed output matches the oracle; its forward is routed + the framework's shared expert."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from torch import nn

from oracle import oracle as O
from tests.conftest import cuda_ok

pytestmark = pytest.mark.gpu

if cuda_ok():
    from prismyra_b200 import kernels, synth

DEV = "cuda:0"


def _bits(t):
    t = t.detach().cpu().contiguous()
    return t.view(torch.uint16).numpy() if t.dtype == torch.bfloat16 else t.view(torch.uint8).numpy()


def test_apply_installs_fused_experts_that_repeat_themselves_and_match_the_oracle():
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeSparseMoeBlock

    H, I, E, k = 256, 128, 8, 4
    cfg = Qwen3_5MoeTextConfig(hidden_size=H, moe_intermediate_size=I, num_experts=E, num_experts_per_tok=k,
                               num_hidden_layers=2, shared_expert_intermediate_size=128, num_attention_heads=2,
                               num_key_value_heads=1, head_dim=64, vocab_size=128,
                               layer_types=["full_attention", "full_attention"])
    cfg.architectures = ["Qwen3_5MoeForCausalLM"]
    torch.manual_seed(0)
    model = nn.ModuleList([Qwen3_5MoeSparseMoeBlock(cfg) for _ in range(2)]).to(torch.bfloat16)
    fp8 = []
    for i, blk in enumerate(model):
        g = torch.Generator().manual_seed(i)
        w1, s1 = synth.quantize_fp8_blocks(torch.randn(E, 2 * I, H, generator=g) * 0.02)
        w2, s2 = synth.quantize_fp8_blocks(torch.randn(E, H, I, generator=g) * 0.02)
        blk.gate.weight.data = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
        blk.experts.gate_up_proj = nn.Parameter(w1, requires_grad=False)
        blk.experts.down_proj = nn.Parameter(w2, requires_grad=False)
        blk.experts.gate_up_proj_scale_inv = nn.Parameter(s1, requires_grad=False)
        blk.experts.down_proj_scale_inv = nn.Parameter(s2, requires_grad=False)
        fp8.append((w1, s1, w2, s2))
    model = model.to(DEV)
    applied = kernels.apply(model, cfg, required=True)
    assert applied.ok and applied.as_dict()["applied"] == {"routed_experts": 2}
    assert "fp8_determinism: 8 calls to the installed FP8 experts agreed bit for bit" in applied.notes
    assert all(type(m).__name__ == "FusedExperts" for m in model)
    x = (torch.randn(48, H, generator=torch.Generator().manual_seed(5))).to(torch.bfloat16).to(DEV)
    for mod, (w1, s1, w2, s2) in zip(model, fp8):
        routed = mod.routed(x)
        logits = mod._route(x)
        ref = O.moe_forward_fp8(_bits(x), _bits(logits), _bits(w1), s1.numpy(), _bits(w2), s2.numpy(), k)["out"]
        got = O.bf16_to_f32(_bits(routed)).astype(np.float64)
        want = O.bf16_to_f32(ref).astype(np.float64)
        assert np.linalg.norm(got - want) / np.linalg.norm(want) < 1e-2
        shared = torch.sigmoid(nn.functional.linear(x, mod.shared_expert_gate.weight)) * mod.shared_expert(x)
        assert torch.equal(mod(x.view(2, 24, H)).view(48, H), routed + shared)
    # idempotent: a second apply counts the installed modules and does not probe again
    again = kernels.apply(model, cfg, required=True)
    assert again.ok and again.as_dict()["applied"] == {"routed_experts": 2}
