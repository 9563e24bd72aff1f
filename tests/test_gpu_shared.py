"""The shared expert and the whole MoE block (routed + shared) on the B200 kernels against the CPU oracle, through
the C ABI.

Tolerances: layer outputs relative L2 <= 1e-2 and max <= 1e-2 * max|ref| (the north-star bf16 tolerance); the
gate within one bf16 ulp of the exactly-rounded sigmoid; the block equal, bit for bit, to the bf16 sum of the
routed call and the shared call; row-count invariance and determinism bit-exact.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from torch import nn

from oracle import oracle as O
from tests.conftest import cuda_ok

pytestmark = pytest.mark.gpu

if cuda_ok():
    from prismyra_b200 import ops, synth

DEV = "cuda:0"
H, I, IS, E, K = 2048, 768, 512, 32, 8


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.uint16).numpy()
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    return t.numpy()


def rel_err(got_bits, ref_bits):
    g = O.bf16_to_f32(got_bits).astype(np.float64)
    r = O.bf16_to_f32(ref_bits).astype(np.float64)
    return np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30), np.abs(g - r).max() / max(np.abs(r).max(), 1e-30)


@pytest.fixture(scope="module")
def block():
    L = synth.make_fp8_layer(T=300, H=H, I=I, E=E, seed=3, device="cpu")
    g = torch.Generator().manual_seed(17)
    w13, s13 = synth.quantize_fp8_blocks(torch.randn(2 * IS, H, generator=g) * 0.02)
    w2, s2 = synth.quantize_fp8_blocks(torch.randn(H, IS, generator=g) * 0.02)
    w_sg = (torch.randn(H, generator=g) * 0.02).to(torch.bfloat16)
    L.update(sw13=w13, sw13_s=s13, sw2=w2, sw2_s=s2, w_sg=w_sg)
    return L, {k: v.to(DEV) for k, v in L.items()}


def _shared(gpu, x):
    return ops.shared_fp8(x, gpu["w_sg"], gpu["sw13"], gpu["sw13_s"], gpu["sw2"], gpu["sw2_s"])


def _block(gpu, x):
    return ops.block_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, gpu["w_sg"], gpu["sw13"],
                         gpu["sw13_s"], gpu["sw2"], gpu["sw2_s"], router_w=gpu["router_w"])


@pytest.mark.parametrize("T", [1, 37, 300])
def test_shared_expert_matches_oracle(block, T):
    """Relative L2 <= 1e-2; the maximum error may add one bf16 ulp (2^-7 relative) on top of 1e-2: every row is
    scaled by its bf16 gate, which is allowed to differ from the oracle's exactly rounded sigmoid by one ulp (pinned
    on its own by test_shared_gate_within_one_ulp)."""
    L, gpu = block
    out = _shared(gpu, gpu["x"][:T].contiguous())
    ref = O.shared_expert_fp8(bits(L["x"][:T]), bits(L["w_sg"]), bits(L["sw13"]), bits(L["sw13_s"]),
                              bits(L["sw2"]), bits(L["sw2_s"]))
    l2, mx = rel_err(bits(out), ref)
    assert l2 < 1e-2 and mx < 1e-2 + 2.0 ** -7, (l2, mx)


def test_shared_gate_within_one_ulp(block):
    """The library's gate, read back as shared(x) / mlp(x): with a zero gate weight the gate is sigmoid(0) = 0.5
    exactly, so that call returns bf16(mlp)/2 exactly and gives mlp(x).  Then shared / mlp = g up to the bf16
    rounding of the product (2^-8 relative), and g is within one bf16 ulp (2^-7 relative) of the oracle's
    exactly rounded sigmoid."""
    L, gpu = block
    T = 300
    x = gpu["x"][:T].contiguous()
    ref = O.shared_gate(bits(L["x"][:T]), bits(L["w_sg"]))
    half = ops.shared_fp8(x, torch.zeros_like(gpu["w_sg"]), gpu["sw13"], gpu["sw13_s"], gpu["sw2"],
                          gpu["sw2_s"]).float()
    mlp = 2.0 * half
    full = _shared(gpu, x).float()
    mask = mlp.abs() > 1e-2
    ratio = (full[mask] / mlp[mask]).cpu().numpy()
    expect = ref[mask.nonzero()[:, 0].cpu().numpy()]
    assert mask.sum() > 1000
    assert np.all(np.abs(ratio - expect) <= expect * (2.0 ** -7 + 2.0 ** -8))


def test_block_is_routed_plus_shared_bit_for_bit(block):
    L, gpu = block
    for T in (1, 129, 300):
        x = gpu["x"][:T].contiguous()
        out = _block(gpu, x)
        routed = ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, router_w=gpu["router_w"])
        shared = _shared(gpu, x)
        assert torch.equal(out, routed + shared), T


def test_block_matches_oracle(block):
    L, gpu = block
    T = 300
    x = gpu["x"][:T].contiguous()
    logits, _, _ = ops.router_topk(x, gpu["router_w"], K)
    out = _block(gpu, x)
    routed = O.moe_forward_fp8(bits(L["x"][:T]), bits(logits), bits(L["w1"]), bits(L["w1_s"]), bits(L["w2"]),
                               bits(L["w2_s"]), K)["out"]
    shared = O.shared_expert_fp8(bits(L["x"][:T]), bits(L["w_sg"]), bits(L["sw13"]), bits(L["sw13_s"]),
                                 bits(L["sw2"]), bits(L["sw2_s"]))
    l2, mx = rel_err(bits(out), O.add_bf16(routed, shared))
    assert l2 < 1e-2 and mx < 1e-2 + 2.0 ** -7, (l2, mx)  # the shared part's gate: one bf16 ulp, as above


def test_block_row_count_invariant_and_deterministic(block):
    _, gpu = block
    full = _block(gpu, gpu["x"].contiguous())
    again = _block(gpu, gpu["x"].contiguous())
    assert torch.equal(full, again)
    for T in (1, 5, 128, 131):
        assert torch.equal(_block(gpu, gpu["x"][:T].contiguous()), full[:T]), T


def test_fused_experts_runs_an_fp8_shared_expert_in_the_library(block):
    """A block whose shared expert holds transformers FP8Linear projections: FusedExperts.forward is the
    library's block call, bit for bit."""
    from transformers.activations import ACT2FN
    from transformers.integrations.finegrained_fp8 import FP8Linear

    from prismyra_b200.kernels.qwen3_moe import FusedExperts

    L, gpu = block

    def fp8_linear(w, s):
        m = FP8Linear(w.shape[1], w.shape[0], block_size=(128, 128))
        m.weight = nn.Parameter(w.clone(), requires_grad=False)
        m.weight_scale_inv = nn.Parameter(s.clone(), requires_grad=False)
        return m.to(DEV)

    class MLP(nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_proj = fp8_linear(gpu["sw13"][:IS], gpu["sw13_s"][: IS // 128])
            self.up_proj = fp8_linear(gpu["sw13"][IS:], gpu["sw13_s"][IS // 128:])
            self.down_proj = fp8_linear(gpu["sw2"], gpu["sw2_s"])
            self.act_fn = ACT2FN["silu"]

    class Experts(nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_up_proj = nn.Parameter(gpu["w1"], requires_grad=False)
            self.down_proj = nn.Parameter(gpu["w2"], requires_grad=False)
            self.gate_up_proj_scale_inv = nn.Parameter(gpu["w1_s"], requires_grad=False)
            self.down_proj_scale_inv = nn.Parameter(gpu["w2_s"], requires_grad=False)

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.gate = nn.Linear(H, E, bias=False).to(DEV, torch.bfloat16)
            self.gate.weight.data.copy_(gpu["router_w"])
            self.experts = Experts()
            self.shared_expert = MLP()
            self.shared_expert_gate = nn.Linear(H, 1, bias=False).to(DEV, torch.bfloat16)
            self.shared_expert_gate.weight.data.copy_(gpu["w_sg"].reshape(1, H))

    mod = FusedExperts(Block(), K)
    assert mod.shared_fp8 is not None
    x = gpu["x"][:77].contiguous()
    y = mod(x.reshape(7, 11, H))
    assert y.shape == (7, 11, H)
    assert torch.equal(y.reshape(77, H), _block(gpu, x))
