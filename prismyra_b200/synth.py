"""Seeded synthetic inputs for the routed-expert layer (no checkpoint or dataset is involved).

One ``torch.Generator`` seeded with ``seed`` draws, in order: x ~ N(0,1) [T, H]; the router weight ~ N(0, 0.02)
[E, H]; then, expert by expert, the gate_up weight ~ N(0, 0.02) [2I, H] and afterwards, expert by expert, the
down weight ~ N(0, 0.02) [H, I].  Expert weights are quantised to e4m3 per 128x128 block with scale = block
amax / 448 (the multiplier a stored value is restored with), the recipe of the reference's own FP8 test
synthesiser (tests/test_nvfp4.py:32-39).  x and the router weight are bf16.
"""

from __future__ import annotations

import math

import torch

FP8 = torch.float8_e4m3fn


def quantize_fp8_blocks(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[..., R, C] float -> e4m3 [..., R, C] and fp32 scales [..., R/128, C/128] (scale = amax / 448)."""
    *lead, r, c = w.shape
    v = w.reshape(-1, r // 128, 128, c // 128, 128).float()
    s = v.abs().amax((2, 4)) / 448.0
    q = (v / s[:, :, None, :, None].clamp(min=1e-12)).clamp(-448, 448).to(FP8)
    return q.reshape(*lead, r, c), s.reshape(*lead, r // 128, c // 128).contiguous()


def dequantize_fp8_blocks(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    *lead, r, c = q.shape
    v = q.float().reshape(-1, r // 128, 128, c // 128, 128) * s.reshape(-1, r // 128, 1, c // 128, 1)
    return v.reshape(*lead, r, c)


def make_fp8_layer(T: int, H: int = 2048, I: int = 768, E: int = 128, seed: int = 0, device="cpu",
                   gen_device: str = "cpu") -> dict:
    """The BASELINE layer (defaults: H=2048, I=768, E=128) with T tokens.  ``gen_device='cuda'`` draws on the
    GPU (a different, equally seeded stream) to keep the bench's set-up short."""
    g = torch.Generator(gen_device).manual_seed(seed)
    kw = dict(generator=g, device=gen_device)
    x = torch.randn(T, H, **kw).to(torch.bfloat16)
    router_w = (torch.randn(E, H, **kw) * 0.02).to(torch.bfloat16)
    w1 = torch.empty(E, 2 * I, H, dtype=FP8, device=gen_device)
    s1 = torch.empty(E, 2 * I // 128, H // 128, dtype=torch.float32, device=gen_device)
    for e in range(E):
        w1[e], s1[e] = quantize_fp8_blocks(torch.randn(2 * I, H, **kw) * 0.02)
    w2 = torch.empty(E, H, I, dtype=FP8, device=gen_device)
    s2 = torch.empty(E, H // 128, I // 128, dtype=torch.float32, device=gen_device)
    for e in range(E):
        w2[e], s2[e] = quantize_fp8_blocks(torch.randn(H, I, **kw) * 0.02)
    out = dict(x=x, router_w=router_w, w1=w1, w1_s=s1, w2=w2, w2_s=s2)
    return {k: v.to(device) for k, v in out.items()}


def zipf_bias(E: int, s: float = 1.1, seed: int = 0) -> torch.Tensor:
    """Per-expert logit bias b_e = ln(E * p_e), p_e proportional to rank_e^-s over a seeded permutation of the
    experts: added to the router logits it skews the expert load like a Zipf(s) law."""
    g = torch.Generator().manual_seed(10_000 + seed)
    perm = torch.randperm(E, generator=g)
    ranks = torch.empty(E)
    ranks[perm] = torch.arange(1, E + 1, dtype=torch.float32)
    p = ranks.pow(-s)
    p = p / p.sum()
    return torch.log(E * p)


def layer_flops(T: int, H: int = 2048, I: int = 768, k: int = 8) -> dict:
    """Algorithmic FLOPs of the routed layer (router excluded): 2*k*(2I*H + H*I) per token."""
    g1 = 2 * k * (2 * I * H) * T
    g2 = 2 * k * (H * I) * T
    return {"gemm1": g1, "gemm2": g2, "total": g1 + g2, "router": 2 * H * 128 * T}


def layer_bytes(T: int, experts_hit: int, H: int = 2048, I: int = 768, E: int = 128) -> int:
    """Algorithmic HBM bytes of one FP8 layer call: every expert matrix with at least one routed token (weights
    + fp32 block scales), x and out in bf16, and the router weight."""
    per_expert = 2 * I * H + H * I + ((2 * I // 128) * (H // 128) + (H // 128) * (I // 128)) * 4
    return experts_hit * per_expert + 2 * T * H * 2 + E * H * 2


def expected_experts_hit(T: int, E: int = 128, k: int = 8) -> float:
    """Expected number of experts with >= 1 token under uniform routing of T tokens, k distinct experts each."""
    return E * (1.0 - math.pow(1.0 - k / E, T))


def make_nvfp4_layer(fp8: dict, calib_tokens: int = 256, top_k: int = 8) -> dict:
    """NVFP4 weights from an FP8 synthetic layer (the reference's prepare_layer recipe) plus a synthetic activation
    calibration: w13_in_amax = max|x|, w2_in_amax = max|silu(gate)*up| over the first ``calib_tokens`` tokens routed
    by the layer's own router, computed in fp32 from the dequantised FP8 weights (no calibration file exists for
    synthetic data)."""
    from .kernels import nvfp4

    dev = fp8["w1"].device
    prep = nvfp4.prepare_layer(fp8["w1"], fp8["w1_s"], fp8["w2"], fp8["w2_s"], dev)
    x = fp8["x"][:calib_tokens].float()
    logits = (x @ fp8["router_w"].float().t()).to(torch.bfloat16).float()
    ids = torch.topk(torch.softmax(logits, -1), top_k, dim=-1).indices
    amax2 = 0.0
    I = fp8["w1"].shape[1] // 2
    for e in ids.unique().tolist():
        rows = (ids == e).any(-1)
        w = dequantize_fp8_blocks(fp8["w1"][e], fp8["w1_s"][e])
        h = x[rows] @ w.t()
        a = torch.nn.functional.silu(h[:, :I]) * h[:, I:]
        amax2 = max(amax2, float(a.abs().max()))
    act = {"w13_in_amax": float(fp8["x"].float().abs().max()), "w2_in_amax": [amax2]}
    return {"prepared": prep, "act": act}


def nvfp4_device_layer(fp8: dict, dev) -> dict:
    """The NVFP4 operands of :func:`make_nvfp4_layer` on ``dev`` in the kernels' layouts: FP4 weights, blocked
    e4m3 scale tiles, per-expert alphas 1/(g_w * g_a) and the two activation global scales 448*6/(1.25*amax)."""
    from .kernels import nvfp4

    nv = make_nvfp4_layer(fp8)
    prep, act = nv["prepared"], nv["act"]
    a1 = float(448.0 * 6.0 / (1.25 * act["w13_in_amax"]))
    a2 = float(448.0 * 6.0 / (1.25 * max(act["w2_in_amax"])))
    return {"w1": prep["w1"].to(dev), "w2": prep["w2"].to(dev), "w1_sf": nvfp4.block_scales(prep["s1"]).to(dev),
            "w2_sf": nvfp4.block_scales(prep["s2"]).to(dev), "al1": (1.0 / (prep["g1"] * a1)).float().to(dev),
            "al2": (1.0 / (prep["g2"] * a2)).float().to(dev), "a1": a1, "a2": a2}
