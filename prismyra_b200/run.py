"""Run the routed-expert layer on synthetic data a fixed number of times (for profilers and quick checks).

    python -m prismyra_b200.run --tokens 5120 --iters 3 [--format fp8|nvfp4|block|prepare]

Builds the seeded synthetic layer (H=2048, I=768, E=128, top-8 by default; NVFP4 weights derived from the FP8
ones) on the current GPU, runs the forward ``--iters`` times on the current stream and prints the output checksum
and the device status.  ``block`` runs routed + shared expert (a synthetic block-FP8 shared expert of
``--shared-inter`` columns) in one call; ``prepare`` runs the NVFP4 weight preparation of both expert stacks.
"""

from __future__ import annotations

import argparse

import torch

from . import ops, synth


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=5120)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--inter", type=int, default=768)
    ap.add_argument("--experts", type=int, default=128)
    ap.add_argument("--top-k", type=int, default=8)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--format", choices=["fp8", "nvfp4", "block", "prepare"], default="fp8")
    ap.add_argument("--shared-inter", type=int, default=512)
    a = ap.parse_args()
    dev = torch.device("cuda", torch.cuda.current_device())
    L = synth.make_fp8_layer(a.tokens, a.hidden, a.inter, a.experts, seed=a.seed, device=dev, gen_device="cuda")
    if a.format == "nvfp4":
        nw = synth.nvfp4_device_layer(L, dev)

        def step():
            return ops.forward_nvfp4(L["x"], nw["w1"], nw["w1_sf"], nw["al1"], nw["a1"], nw["w2"], nw["w2_sf"],
                                     nw["al2"], nw["a2"], a.top_k, router_w=L["router_w"])
    elif a.format == "block":
        g = torch.Generator("cuda").manual_seed(a.seed + 77)
        Is = a.shared_inter
        sw13, sw13_s = synth.quantize_fp8_blocks(torch.randn(2 * Is, a.hidden, generator=g, device=dev) * 0.02)
        sw2, sw2_s = synth.quantize_fp8_blocks(torch.randn(a.hidden, Is, generator=g, device=dev) * 0.02)
        w_sg = (torch.randn(a.hidden, generator=g, device=dev) * 0.02).to(torch.bfloat16)

        def step():
            return ops.block_fp8(L["x"], L["w1"], L["w1_s"], L["w2"], L["w2_s"], a.top_k, w_sg, sw13, sw13_s, sw2,
                                 sw2_s, router_w=L["router_w"])
    elif a.format == "prepare":
        def step():
            ops.nvfp4_prepare(L["w1"], L["w1_s"])
            return ops.nvfp4_prepare(L["w2"], L["w2_s"])[2]
    else:
        def step():
            return ops.forward_fp8(L["x"], L["w1"], L["w1_s"], L["w2"], L["w2_s"], a.top_k, router_w=L["router_w"])
    torch.cuda.synchronize()
    out = None
    for _ in range(a.iters):
        out = step()
    if a.format in ("fp8", "nvfp4"):
        ws, _ = ops.workspace_for(L["x"], a.tokens, a.hidden, a.inter, a.experts, a.top_k, int(a.format == "nvfp4"))
        ops.read_status(ws)
    torch.cuda.synchronize()
    print(f"format={a.format} tokens={a.tokens} iters={a.iters} checksum={out.float().abs().sum().item():.6e} status=ok")


if __name__ == "__main__":
    main()
