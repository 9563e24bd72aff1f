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


def _group_scales(amax: torch.Tensor, g: torch.Tensor, frac: float = 1.0) -> torch.Tensor:
    """e4m3(min(amax/6 * g * frac, 448)) per 16-group, rounded step by step in fp32 (frac 1.0 multiplies exactly)."""
    return (amax / 6.0 * g * frac).clamp(max=448.0).to(FP8)


def _encode(groups: torch.Tensor, scale: torch.Tensor, g: torch.Tensor):
    """Nearest e2m1 magnitude index (the first of equals, i.e. the smaller magnitude), sign and step of each value
    of groups [..., G, 16] under e4m3 group scales [..., G] and global scales g broadcastable to [..., G]."""
    step = (scale.float() / g).unsqueeze(-1)
    x = torch.where(step > 0, groups / step, torch.zeros_like(groups)).clamp(-6, 6)
    grid = torch.tensor(E2M1_VALUES, device=groups.device)
    mag = (x.abs().unsqueeze(-1) - grid).abs().argmin(-1)
    return mag, x < 0, step


def _pack(mag: torch.Tensor, neg: torch.Tensor) -> torch.Tensor:
    """Codes [..., G, 16] -> bytes [..., G*8]: two codes per byte, the even column in the low nibble."""
    code = (mag | (neg.long() << 3)).to(torch.uint8).flatten(-2)
    return (code[..., 0::2] | (code[..., 1::2] << 4)).contiguous()


SEARCH = (1.0, 0.95, 0.9, 0.85, 0.8, 0.75, 0.7)


def _quantize_groups(groups: torch.Tensor, g: torch.Tensor, imp: torch.Tensor | None = None, search: bool = False):
    """groups [..., G, 16] fp32 under global scales g (broadcastable to [..., G]) -> (packed bytes, e4m3 scales).

    Without ``search`` every 16-group gets the plain scale e4m3(min(amax/6*g, 448)).  With it, the scale is chosen
    among SEARCH fractions of the plain one: the fraction whose decoded group has the smallest importance-weighted
    squared error (imp broadcastable to groups; None weighs every value 1), the earliest fraction among equals."""
    amax = groups.abs().amax(-1)
    if not search:
        scale = _group_scales(amax, g)
    else:
        w = imp if imp is not None else torch.ones((), device=groups.device)
        grid = torch.tensor(E2M1_VALUES, device=groups.device)
        cand, errs = [], []
        for frac in SEARCH:
            sc = _group_scales(amax, g, frac)
            mag, neg, step = _encode(groups, sc, g)
            back = grid[mag] * torch.where(neg, -1.0, 1.0) * step
            errs.append((w * (back - groups) ** 2).sum(-1))
            cand.append(sc.view(torch.uint8))
        pick = torch.stack(errs).argmin(0, keepdim=True)
        scale = torch.stack(cand).gather(0, pick)[0].view(FP8)
    mag, neg, _ = _encode(groups, scale, g)
    return _pack(mag, neg), scale.contiguous()


def quantize(w: torch.Tensor, global_scale) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 [rows, cols] and a global scale -> packed uint8 [rows, cols/2] and e4m3 scales [rows, cols/16]."""
    rows, cols = w.shape
    g = torch.as_tensor(global_scale, dtype=torch.float32, device=w.device)
    return _quantize_groups(w.reshape(rows, cols // 16, 16), g)


def quantize_search(w: torch.Tensor, global_scale, importance: torch.Tensor | None):
    """:func:`quantize` with each 16-group's scale searched among SEARCH fractions of its plain scale (the
    reference's nvfp4.py:57-94).  importance is per input column; None weighs every column 1."""
    rows, cols = w.shape
    g = torch.as_tensor(global_scale, dtype=torch.float32, device=w.device)
    imp = importance.float().reshape(cols // 16, 16) if importance is not None else None
    return _quantize_groups(w.reshape(rows, cols // 16, 16), g, imp, search=True)


def dequant_fp8(w: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """128x128 block FP8 [..., R, C] -> fp32 (each stored value times its block's multiplier)."""
    *lead, o, i = w.shape
    v = w.float().reshape(-1, o // 128, 128, i // 128, 128) * s.float().reshape(-1, o // 128, 1, i // 128, 1)
    return v.reshape(*lead, o, i)


def _prepare_stack(w: torch.Tensor, s: torch.Tensor, device, imp: torch.Tensor | None, chunk: int = 4):
    """An FP8 expert stack [E, R, C] -> (packed [E, R, C/2], scales [E, R, C/16], g [E]), ``chunk`` experts at a
    time: every matrix is restored to fp32, g = 448*6/max(amax, 1e-12) per matrix (torch evaluates the quotient as
    reciprocal(amax) * 2688), then its groups are quantised (searched when ``imp`` [E, C] is given)."""
    E, R, C = w.shape
    packed, scales, gs = [], [], []
    for e0 in range(0, E, chunk):
        d = dequant_fp8(w[e0:e0 + chunk].to(device), s[e0:e0 + chunk].to(device))
        n = d.shape[0]
        g = 448.0 * 6.0 / d.abs().amax((1, 2)).clamp_min(1e-12)
        im = imp[e0:e0 + n].to(device).float().reshape(n, 1, C // 16, 16) if imp is not None else None
        p, sc = _quantize_groups(d.reshape(n, R, C // 16, 16), g.view(n, 1, 1), im, search=imp is not None)
        packed.append(p.cpu())
        scales.append(sc.cpu())
        gs.append(g.float().cpu())
    return torch.cat(packed), torch.cat(scales), torch.cat(gs)


def prepare_layer(w13, s13, w2, s2, device, imp_in=None, imp_mid=None, tok=None) -> dict:
    """One layer's FP8 experts -> NVFP4 tensors (row-major scales) and one global scale per expert matrix
    (the reference's nvfp4.py:315-331, same arguments and results).

    On a CUDA device the whole stack goes through the library's preparation kernels
    (:func:`prismyra_b200.ops.nvfp4_prepare`, bit-identical to the torch arithmetic of :func:`_prepare_stack`);
    with importance weights (imp_in for w13's input columns, imp_mid for w2's) each 16-group's scale is searched,
    experts whose token count ``tok`` is 0 weighing every column 1."""
    dev = torch.device(device)
    def importance(imp):
        if imp is None:
            return None
        imp = imp.float().clone()
        if tok is not None:
            imp[torch.as_tensor(tok) <= 0] = 1.0  # experts without tokens: plain squared error
        return imp

    out = {}
    if dev.type == "cuda":
        for w, s, imp, tag in ((w13, s13, imp_in, "1"), (w2, s2, imp_mid, "2")):
            imp = importance(imp)
            packed, scale, g = ops.nvfp4_prepare(w.to(dev).contiguous(), s.to(dev, torch.float32).contiguous(),
                                                 importance=imp.to(dev).contiguous() if imp is not None else None,
                                                 search=imp_in is not None)
            out["w" + tag], out["s" + tag], out["g" + tag] = packed, scale, g
        return {k: v.cpu() for k, v in out.items()}
    for w, s, imp, tag in ((w13, s13, imp_in, "1"), (w2, s2, imp_mid, "2")):
        out["w" + tag], out["s" + tag], out["g" + tag] = _prepare_stack(w, s, dev, importance(imp))
    return out


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
