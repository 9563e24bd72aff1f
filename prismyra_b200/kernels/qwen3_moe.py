"""The routed-expert layer of Qwen3.5/3.6-MoE checkpoints on B200 kernels, and its adapter.

``FusedExperts`` is a drop-in for the reference's module of the same name (prismyra/kernels/qwen3_moe.py:
142-199): it is built from the framework's ``Qwen3_5MoeSparseMoeBlock`` and ``top_k``, exposes ``gate``,
``shared_expert``, ``shared_expert_gate``, ``top_k``, ``w1`` and ``w2``, and its ``forward`` maps bf16
``[..., H]`` to bf16 of the same shape.  The routed path (router projection, softmax / top-k, expert alignment,
both grouped FP8 GEMMs with silu-and-mul between them, and the weighted top-k sum) runs in
``libprismyra_moe.so``.  When the block's shared expert holds 128x128 block-FP8 projections (transformers'
``FP8Linear`` or the reference's ``Fp8Linear``) the shared expert, its sigmoid gate and the final ``routed +
shared`` run in the same library call (``pm_moe_block_fp8``) with the reference's arithmetic; otherwise they stay
the framework's own modules, as in the reference.
"""

from __future__ import annotations

import os

import torch
import torch.nn.functional as F
from torch import nn

from .. import ops
from . import AdapterError, Applied, Swap, register

BLOCK = (128, 128)

#: Shapes the B200 kernels accept (include/prismyra_moe.h).
LIMITS = {"max_experts": 256, "max_top_k": 16, "hidden_multiple": 256, "intermediate_multiple": 128}


def _fp8_expert_tensors(experts: nn.Module):
    """(w1, w1_scale, w2, w2_scale) from a framework experts module holding 128x128 block-FP8 weights, or None.
    ``*_scale_inv`` is the multiplier that restores a stored value (reference qwen3_moe.py:158-161)."""
    w1 = getattr(experts, "gate_up_proj", None)
    w2 = getattr(experts, "down_proj", None)
    s1 = getattr(experts, "gate_up_proj_scale_inv", None)
    s2 = getattr(experts, "down_proj_scale_inv", None)
    if any(t is None for t in (w1, w2, s1, s2)):
        return None
    if w1.dtype != torch.float8_e4m3fn or w2.dtype != torch.float8_e4m3fn:
        return None
    return w1, s1, w2, s2


def _fp8_linear(m: nn.Module | None):
    """(weight e4m3 [out, in], block multipliers f32 [out/128, in/128]) of a bias-free block-FP8 projection with
    dynamic activation quantisation, or None."""
    if m is None:
        return None
    w = getattr(m, "weight", None)
    s = getattr(m, "weight_scale_inv", None)
    if s is None:
        s = getattr(m, "scale", None)
    if w is None or s is None or w.dtype != torch.float8_e4m3fn or getattr(m, "bias", None) is not None:
        return None
    if getattr(m, "activation_scheme", "dynamic") != "dynamic":
        return None
    o, i = w.shape
    if o % 128 or i % 128 or tuple(s.shape) != (o // 128, i // 128):
        return None
    return w, s


def _fp8_shared_tensors(block: nn.Module, hidden: int):
    """(w_sg bf16 [H], w13 e4m3 [2 Is, H], w13_s, w2 e4m3 [H, Is], w2_s) of a silu-gated block-FP8 shared expert
    with a bf16 one-row gate, or None."""
    se = getattr(block, "shared_expert", None)
    gate = getattr(block, "shared_expert_gate", None)
    if se is None or gate is None:
        return None
    parts = [_fp8_linear(getattr(se, n, None)) for n in ("gate_proj", "up_proj", "down_proj")]
    if any(p is None for p in parts):
        return None
    act = type(getattr(se, "act_fn", None)).__name__
    w_sg = getattr(gate, "weight", None)
    if act not in ("SiLU", "SiLUActivation") or w_sg is None or w_sg.dtype != torch.bfloat16:
        return None
    (wg, sg), (wu, su), (wd, sd) = parts
    Is = wg.shape[0]
    if (tuple(w_sg.shape) != (1, hidden) or tuple(wg.shape) != (Is, hidden) or wu.shape != wg.shape
            or tuple(wd.shape) != (hidden, Is)):
        return None
    w13 = torch.cat([wg.detach(), wu.detach()], 0).contiguous()
    s13 = torch.cat([sg.detach(), su.detach()], 0).to(torch.float32).contiguous()
    return (w_sg.detach().reshape(hidden).contiguous(), w13, s13, wd.detach().contiguous(),
            sd.detach().to(torch.float32).contiguous())


class FusedExperts(nn.Module):
    """Routed experts through the B200 kernels; router and shared expert kept as in the framework block.

    ``act_scale`` (default: the PRISMYRA_B200_ACT_SCALE environment variable, else "fp32") picks how activations are
    quantised: "fp32" scales max(amax, 1e-10)/448, the reference's arithmetic (vLLM's per_token_group_quant_fp8); or
    "ue8m0", those scales rounded up to powers of two, which is what the reference's vLLM call computes on a host
    where vLLM runs DeepGEMM with E8M0 scales (VLLM_USE_DEEP_GEMM_E8M0, on by default wherever DeepGEMM is
    installed).  In the "ue8m0" mode a block-FP8 shared expert stays the framework's module."""

    def __init__(self, block: nn.Module, top_k: int, act_scale: str | None = None):
        super().__init__()
        self.act_scale = act_scale or os.environ.get("PRISMYRA_B200_ACT_SCALE", "fp32")
        if self.act_scale not in ops.ACT_SCALES:
            raise AdapterError(f"act_scale must be one of {sorted(ops.ACT_SCALES)}, got {self.act_scale!r}")
        tensors = _fp8_expert_tensors(block.experts)
        if tensors is None:
            raise AdapterError("FusedExperts needs 128x128 block-FP8 expert weights (gate_up_proj[_scale_inv], "
                               "down_proj[_scale_inv])")
        w1, s1, w2, s2 = tensors
        self.gate = block.gate
        self.shared_expert = block.shared_expert
        self.shared_expert_gate = block.shared_expert_gate
        self.top_k = int(top_k)
        self.w1 = w1.detach().contiguous()
        self.w2 = w2.detach().contiguous()
        self.w1_scale = s1.detach().to(torch.float32).contiguous()
        self.w2_scale = s2.detach().to(torch.float32).contiguous()
        E, I2, H = self.w1.shape
        self.num_experts, self.hidden, self.inter = E, H, I2 // 2
        if (E > LIMITS["max_experts"] or self.top_k > min(LIMITS["max_top_k"], E)
                or H % LIMITS["hidden_multiple"] or self.inter % LIMITS["intermediate_multiple"]):
            raise AdapterError(f"shape outside the kernel's range: E={E} k={self.top_k} H={H} I={self.inter}")
        #: (w_sg, w13, w13_s, w2, w2_s) when the shared expert runs in the library, else None
        self.shared_fp8 = _fp8_shared_tensors(block, H) if self.act_scale == "fp32" else None

    def _route(self, x: torch.Tensor) -> torch.Tensor:
        """Router logits (bf16 [T, E]), row-count invariant: each logit is reduced over H in a fixed order."""
        logits, _, _ = ops.router_topk(x.contiguous(), self.gate.weight.contiguous(), self.top_k)
        return logits

    def routed(self, x: torch.Tensor, logits: torch.Tensor | None = None) -> torch.Tensor:
        """The routed-expert output for x [T, H] (no shared expert)."""
        return ops.forward_fp8(x.contiguous(), self.w1, self.w1_scale, self.w2, self.w2_scale, self.top_k,
                               router_w=None if logits is not None else self.gate.weight.contiguous(),
                               logits=logits, act_scale=self.act_scale)

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1]).contiguous()
        if self.shared_fp8 is not None:
            w_sg, w13, s13, w2, s2 = self.shared_fp8
            out = ops.block_fp8(x, self.w1, self.w1_scale, self.w2, self.w2_scale, self.top_k, w_sg, w13, s13, w2,
                                s2, router_w=self.gate.weight.contiguous())
            return out.reshape(shape)
        routed = self.routed(x)
        shared = torch.sigmoid(F.linear(x, self.shared_expert_gate.weight)) * self.shared_expert(x)
        return (routed + shared).reshape(shape)


class Fp8Linear(nn.Module):
    """A block-quantised projection on the library's kernel, wrapping the original module's weights (the reference's
    Fp8Linear, prismyra/kernels/qwen3_moe.py:211-230): per-token-group FP8 quantisation of the input and the
    block-scaled matmul, bf16 out.  The weight stays (out, in); its scale_inv widens to fp32."""

    def __init__(self, inner: nn.Module):
        super().__init__()
        t = _fp8_linear(inner)
        if t is None:
            raise AdapterError("Fp8Linear needs a bias-free e4m3 weight with 128x128 fp32 block scales")
        self.inner = inner
        self.weight = inner.weight
        self.register_buffer("scale", t[1].detach().to(torch.float32).contiguous(), persistent=False)
        self.out_features, self.in_features = inner.weight.shape
        if self.out_features % 256 or self.in_features % 128:
            raise AdapterError(f"Fp8Linear on the B200 kernel needs out % 256 == 0 and in % 128 == 0, got "
                               f"{self.out_features} x {self.in_features}")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.fp8_linear(x.contiguous(), self.weight.detach(), self.scale)


class FusedDenseProjection(nn.Module):
    """One block-FP8 matmul for several sibling projections of the same input, split back into their own widths (the
    reference's _FusedDenseProjection, qwen3_moe.py:233-262).  Every sibling's width is a multiple of 128, so no
    weight block straddles a seam and each output keeps its own per-row reduction: the split outputs equal the
    separate calls bit for bit."""

    def __init__(self, parts: list):
        super().__init__()
        if not parts or any(not isinstance(p, Fp8Linear) for p in parts):
            raise AdapterError("FusedDenseProjection needs Fp8Linear parts")
        if any(p.in_features != parts[0].in_features or p.out_features % 128 for p in parts):
            raise AdapterError("FusedDenseProjection needs one input width and output widths that are multiples "
                               "of 128")
        self.sizes = [p.out_features for p in parts]
        self.in_features = parts[0].in_features
        self.out_features = sum(self.sizes)
        if self.out_features % 256:
            raise AdapterError("FusedDenseProjection needs a combined output width that is a multiple of 256")
        self.register_buffer("weight", torch.cat([p.weight.detach() for p in parts], 0).contiguous(),
                             persistent=False)
        self.register_buffer("scale", torch.cat([p.scale for p in parts], 0).contiguous(), persistent=False)

    def forward(self, x: torch.Tensor) -> tuple:
        out = ops.fp8_linear(x.contiguous(), self.weight, self.scale)
        return torch.split(out, self.sizes, dim=-1)


#: How many times the construction-time self-check calls one installed FusedExperts on the same input (the
#: reference's FP8 determinism probe, prismyra/kernels/qwen3_moe.py:1677-1683).
FP8_DETERMINISM_PROBES = 8


def _withheld() -> set[str]:
    """Checks a caller switched off with PRISMYRA_WITHOUT (a comma-separated list), as in the reference."""
    return {w.strip() for w in os.environ.get("PRISMYRA_WITHOUT", "").split(",") if w.strip()}


def _raise_if_out_of_resources(e: Exception, context: str) -> None:
    """A self-check that could not run because the device ran out of memory says nothing about the kernel; it is
    raised as AdapterError instead of silently choosing a slower path (the reference's qwen3_moe.py:29-65, whose
    other resource case, a Triton shared-memory limit, has no counterpart here: these kernels' shared memory is
    fixed at build time)."""
    if isinstance(e, torch.OutOfMemoryError):
        raise AdapterError(
            f"{context}: ran out of GPU memory while self-checking the installed kernel ({type(e).__name__}: {e}); "
            "retry with more free memory on this device") from e


def _check_fp8_determinism(applied: Applied, root: nn.Module) -> None:
    """Call one installed FusedExperts on a fixed input FP8_DETERMINISM_PROBES times and refuse to start when the
    bits ever differ (the reference's _check_fp8_determinism, qwen3_moe.py:1683-1761, pointed at the FP8 module this
    adapter installs).  The kernels have no atomics in any reduction, so a difference is a device fault; there is
    nothing to retry.  Running out of memory raises AdapterError; any other failure to run the probe is recorded as a
    skip of this check."""
    probe = next((m for m in root.modules() if type(m).__name__ == "FusedExperts"), None)
    if probe is None:
        applied.notes.append("fp8_determinism: nothing matched (no FusedExperts installed)")
        return
    width = probe.hidden
    g = torch.Generator(device="cpu").manual_seed(width)
    x = (torch.randn(64, width, generator=g) * 0.1).to(device=probe.w1.device, dtype=torch.bfloat16)
    try:
        with torch.inference_mode():
            first = probe(x).clone()
            repeats = [probe(x).clone() for _ in range(FP8_DETERMINISM_PROBES - 1)]
    except Exception as e:  # noqa: BLE001 - a probe that cannot run is a resource question, not a finding
        _raise_if_out_of_resources(e, "fp8_determinism")
        applied.skipped.append(f"fp8_determinism: the probe raised {type(e).__name__}: {e} -- not checked")
        return
    bad = [i for i, r in enumerate(repeats) if not torch.equal(first, r)]
    if bad:
        moved = max((first.float() - repeats[i].float()).abs().max().item() for i in bad)
        raise AdapterError(
            f"fp8_determinism: the installed FP8 experts answered the same input differently in {len(bad)} of "
            f"{FP8_DETERMINISM_PROBES - 1} repeated calls (max difference {moved:.3e}); this device does not give "
            "the same bits back twice -- move to another GPU, or set PRISMYRA_WITHOUT=fp8_determinism to serve "
            "from it anyway")
    applied.notes.append(f"fp8_determinism: {FP8_DETERMINISM_PROBES} calls to the installed FP8 experts agreed "
                         "bit for bit")


def _swap_children(root: nn.Module, class_name: str, make) -> int:
    count = 0
    for parent in list(root.modules()):
        for name, child in list(parent.named_children()):
            if type(child).__name__ == class_name:
                setattr(parent, name, make(child))
                count += 1
    return count


class Qwen3MoeAdapter:
    """Installs ``FusedExperts`` into Qwen3.5/3.6-MoE models whose per-layer shape the kernels accept."""

    name = "qwen3-moe-b200"

    def supports(self, config) -> bool:
        names = getattr(config, "architectures", None) or []
        if not any("Qwen3_5Moe" in n for n in names):
            return False
        d = getattr(config, "text_config", config)
        E = getattr(d, "num_experts", 0) or 0
        k = getattr(d, "num_experts_per_tok", 0) or 0
        H = getattr(d, "hidden_size", 0) or 0
        I = getattr(d, "moe_intermediate_size", 0) or 0
        return (0 < k <= min(E, LIMITS["max_top_k"]) and E <= LIMITS["max_experts"] and H > 0
                and H % LIMITS["hidden_multiple"] == 0 and I > 0 and I % LIMITS["intermediate_multiple"] == 0)

    def replace(self, model: nn.Module, config) -> Applied:
        d = getattr(config, "text_config", config)
        applied = Applied(adapter=self.name)
        text = getattr(model, "language_model", model)
        if text is not model:
            applied.notes.append("replacements were applied to the text decoder; the vision tower is untouched")
        already = sum(1 for m in text.modules() if type(m).__name__ in ("FusedExperts", "FusedExpertsFp4"))
        if already:
            applied.swaps.append(Swap("routed_experts", already, d.num_hidden_layers))
            return applied
        blocks = [m for m in text.modules() if type(m).__name__ == "Qwen3_5MoeSparseMoeBlock"]
        if blocks and _fp8_expert_tensors(blocks[0].experts) is None:
            applied.skipped.append("routed experts are not 128x128 block-FP8 (the B200 FP8 kernels need them)")
            return applied
        if not torch.cuda.is_available():
            applied.skipped.append("no CUDA device: the B200 kernels need one")
            return applied
        n = _swap_children(text, "Qwen3_5MoeSparseMoeBlock", lambda m: FusedExperts(m, d.num_experts_per_tok))
        applied.swaps.append(Swap("routed_experts", n, d.num_hidden_layers))
        applied.notes.append("only the routed experts are replaced; attention, norms and dense projections keep "
                             "the framework's modules")
        if "fp8_determinism" not in _withheld():
            _check_fp8_determinism(applied, text)
        return applied


register(Qwen3MoeAdapter())
