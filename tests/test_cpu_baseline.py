"""The reference's CPU fallback (transformers block) that bench.py times as its CPU baseline runs here and agrees
with the oracle up to the FP8 activation quantisation the fallback does not do."""

from __future__ import annotations

import numpy as np
import torch

from oracle import oracle as O
from oracle import torch_fallback
from prismyra_b200 import synth


def test_fallback_runs_and_agrees_with_the_oracle():
    L = synth.make_fp8_layer(48, 256, 128, 8, seed=3)
    w1 = synth.dequantize_fp8_blocks(L["w1"], L["w1_s"])
    w2 = synth.dequantize_fp8_blocks(L["w2"], L["w2_s"])
    router, experts = torch_fallback.build_block(L["router_w"].float(), w1, w2, 4)
    y = torch_fallback.routed(router, experts, L["x"].float())
    logits = O.router_logits(L["x"].view(torch.uint16).numpy(), L["router_w"].view(torch.uint16).numpy())
    ref = O.moe_forward_fp8(L["x"].view(torch.uint16).numpy(), logits, L["w1"].view(torch.uint8).numpy(),
                            L["w1_s"].numpy(), L["w2"].view(torch.uint8).numpy(), L["w2_s"].numpy(), 4)["out"]
    r = O.bf16_to_f32(ref).astype(np.float64)
    rel = np.linalg.norm(y.double().numpy() - r) / np.linalg.norm(r)
    assert rel < 8e-2  # FP8 activation quantisation (e4m3, 3 mantissa bits) is the only difference
    t = torch_fallback.time_routed(router, experts, L["x"].float(), max_seconds=0.05, max_calls=6)
    assert t["tokens_per_s"] > 0 and 5 <= t["calls"] <= 6 and t["warmup"] == 2
    assert t["tokens_per_s"] == L["x"].shape[0] / t["median_s"] and t["cpu_model"]
    rb, eb = torch_fallback.build_block(L["router_w"].float(), w1, w2, 4, dtype=torch.bfloat16)
    tb = torch_fallback.time_routed(rb, eb, L["x"], max_seconds=0.05)
    assert tb["dtype"] == "bfloat16" and tb["tokens_per_s"] > 0
