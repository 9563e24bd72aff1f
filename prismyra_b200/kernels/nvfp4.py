"""Routed experts in NVFP4 on the B200 kernels: weight preparation and the drop-in ``FusedExpertsFp4``.

Mirrors the reference's ``prismyra/kernels/nvfp4.py``:

* :func:`quantize` / :func:`prepare_layer` produce exactly the reference's tensors (nvfp4.py:41-51, 97-100,
  315-331; checked bit for bit against the reference by the golden tests): FP8 128x128 blocks are restored to
  fp32, every expert matrix gets a global scale g = 448*6/amax, each 16-element group an e4m3 scale
  e4m3(min(amax/6*g, 448)), and each value the nearest e2m1 code (ties to the smaller magnitude, the first
  arg-min of the reference), two codes per byte with the even column in the low nibble.
* :class:`FusedExpertsFp4` takes the same constructor arguments as the reference's module (the framework block,
  top_k, the prepared tensors, the per-layer activation calibration, the device) and computes the activation
  global scales a1 = 448*6/(1.25*w13_in_amax), a2 = 448*6/(1.25*max(w2_in_amax)) and the per-expert
  alphas 1/(g*a) the same way (nvfp4.py:115-145).  The scales are rearranged once into the blocked layout the
  tensor core reads (:func:`block_scales`); gate and up rows keep their order (the reference reorders them only
  because FlashInfer wants up before gate).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from .. import ops

FP8 = torch.float8_e4m3fn
HEADROOM = 1.25
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def quantize(w: torch.Tensor, global_scale) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 [rows, cols] and a global scale -> packed uint8 [rows, cols/2] and e4m3 scales [rows, cols/16]."""
    rows, cols = w.shape
    groups = w.reshape(rows, cols // 16, 16)
    g = torch.as_tensor(global_scale, dtype=torch.float32, device=w.device)
    scale = (groups.abs().amax(-1) / 6.0 * g).clamp(max=448.0).to(FP8)
    step = (scale.float() / g).unsqueeze(-1)
    x = torch.where(step > 0, groups / step, torch.zeros_like(groups)).clamp(-6, 6)
    grid = torch.tensor(E2M1_VALUES, device=w.device)
    code = (x.abs().unsqueeze(-1) - grid).abs().argmin(-1)  # first nearest: ties keep the smaller magnitude
    code = (code | ((x < 0).long() << 3)).to(torch.uint8).reshape(rows, cols)
    return (code[:, 0::2] | (code[:, 1::2] << 4)).contiguous(), scale.contiguous()


def dequant_fp8(w: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """128x128 block FP8 -> fp32 (the stored value times its block's multiplier)."""
    o, i = w.shape
    return (w.float().reshape(o // 128, 128, i // 128, 128) * s.float().reshape(o // 128, 1, i // 128, 1)).reshape(o, i)


def prepare_layer(w13, s13, w2, s2, device) -> dict:
    """One layer's FP8 experts -> NVFP4 tensors (row-major scales) and one global scale per expert matrix."""
    out = {k: [] for k in ("w1", "s1", "g1", "w2", "s2", "g2")}
    for e in range(w13.shape[0]):
        for w, s, tag in ((w13, s13, "1"), (w2, s2, "2")):
            d = dequant_fp8(w[e].to(device), s[e].to(device))
            g = 448.0 * 6.0 / d.abs().amax().clamp_min(1e-12)
            packed, scale = quantize(d, g)
            out["w" + tag].append(packed)
            out["s" + tag].append(scale)
            out["g" + tag].append(g.float())
    return {k: torch.stack(v).cpu() for k, v in out.items()}


def block_scales(sf: torch.Tensor) -> torch.Tensor:
    """Row-major e4m3 scales [..., R, K/16] -> the blocked layout [..., R/128, K/64, 512] (bytes) in which row r of a
    128-row block keeps the four scales of a 64-column chunk as one 32-bit word at byte (r%32)*16 + (r/32)*4."""
    *lead, R, G = sf.shape
    b = sf.contiguous().view(torch.uint8).reshape(*lead, R // 128, 4, 32, G // 4, 4)
    n = len(lead)
    perm = list(range(n)) + [n, n + 3, n + 2, n + 1, n + 4]
    return b.permute(*perm).contiguous().reshape(*lead, R // 128, G // 4, 512)


def unblock_scales(blocked: torch.Tensor, R: int, G: int) -> torch.Tensor:
    """Inverse of :func:`block_scales` for one matrix: [R/128, G/4, 512] -> [R, G] uint8."""
    b = blocked.reshape(R // 128, G // 4, 32, 4, 4)
    return b.permute(0, 3, 2, 1, 4).contiguous().reshape(R, G)


class FusedExpertsFp4(nn.Module):
    """The routed path in NVFP4 on the B200 kernels; router and shared expert as in the framework block."""

    def __init__(self, block: nn.Module, top_k: int, prepared: dict, act: dict, device):
        super().__init__()
        self.gate = block.gate
        self.shared_expert = block.shared_expert
        self.shared_expert_gate = block.shared_expert_gate
        self.top_k = int(top_k)
        t = {k: v.to(device) for k, v in prepared.items()}
        e = t["w1"].shape[0]
        self.a1_gscale = float(448.0 * 6.0 / (HEADROOM * float(act["w13_in_amax"])))
        self.a2_gscale = float(448.0 * 6.0 / (HEADROOM * float(max(act["w2_in_amax"]))))
        self.w1, self.w2 = t["w1"].contiguous(), t["w2"].contiguous()
        self.w1_scale = block_scales(t["s1"])
        self.w2_scale = block_scales(t["s2"])
        self.g1_alphas = (1.0 / (t["g1"].float() * self.a1_gscale)).contiguous()
        self.g2_alphas = (1.0 / (t["g2"].float() * self.a2_gscale)).contiguous()
        self.n, self.k, self.e = t["w2"].shape[2] * 2, t["w1"].shape[2] * 2, e
        if hasattr(block, "experts"):
            del block.experts

    def routed(self, x: torch.Tensor, logits: torch.Tensor | None = None) -> torch.Tensor:
        return ops.forward_nvfp4(x.contiguous(), self.w1, self.w1_scale, self.g1_alphas, self.a1_gscale, self.w2,
                                 self.w2_scale, self.g2_alphas, self.a2_gscale, self.top_k,
                                 router_w=None if logits is not None else self.gate.weight.contiguous(),
                                 logits=logits)

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        out = self.routed(x)
        shared = torch.sigmoid(F.linear(x, self.shared_expert_gate.weight)) * self.shared_expert(x)
        return (out + shared).reshape(shape)
