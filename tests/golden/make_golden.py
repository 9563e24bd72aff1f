"""Generate the golden fixtures that pin the CPU oracle to the reference's own arithmetic.

Run once in a container that has the reference checkout and its dependencies (vLLM 0.22, transformers 5.5):

    PYTHONPATH=<reference checkout> python tests/golden/make_golden.py

The reference (Prismyra) delegates the routed-expert arithmetic to vLLM / FlashInfer, so the fixtures come from
the code that actually defines it, run on the CPU:

* ``fp8_layer.npz`` -- vLLM's Triton kernels ``_per_token_group_quant_fp8`` and ``fused_moe_kernel``
  (``vllm/model_executor/layers/quantization/utils/fp8_utils.py``, ``vllm/model_executor/layers/fused_moe/
  fused_moe.py:295-557``) executed by the Triton CPU interpreter (``TRITON_INTERPRET=1``), chained exactly as
  ``fused_experts_impl`` chains them (``fused_moe.py:1664-1869``); the silu-and-mul step is vLLM's own
  ``SiluAndMul.forward_native`` and the top-k sum is ``torch.sum`` over the top-k axis (the fallback
  ``moe_sum`` takes for top_k > 4).  The compiled ``moe_align_block_size`` cannot run here; its documented
  semantics are restated below (``_align``) and pinned separately by ``align_kat.npz``.
* ``fp8_layer_ue8m0.npz`` -- the same layer with both activation quantisations in vLLM's power-of-two (UE8M0)
  scale mode, ``use_ue8m0=True`` (``fp8_utils.py:145``), which vLLM takes when it runs DeepGEMM with E8M0 scales
  (``VLLM_USE_DEEP_GEMM_E8M0``, on by default where DeepGEMM is installed, as on the B200 hosts of this build);
  ``act_quant.npz`` holds the edge rows in both modes.
* ``align_kat.npz`` -- the worked example of the ``moe_align_block_size`` docstring
  (``vllm/model_executor/layers/fused_moe/moe_align_block_size.py:60-69``).  The docstring numbers its experts
  1..4, so the fixture uses ``num_experts=5`` with expert 0 empty.
* ``router.npz`` -- transformers ``Qwen3_5MoeTopKRouter`` (the reference's CPU fallback router) on seeded inputs,
  plus the logits it computed.
* ``nvfp4.npz`` -- the reference's own ``prismyra.kernels.nvfp4.quantize`` / ``_dequant_fp8`` / ``prepare_layer``
  and vLLM's Triton ``_nvfp4_quant_dequant_kernel`` (the activation quantisation of its NVFP4 emulation path),
  interpreted on the CPU.
* ``nvfp4_search.npz`` -- the reference's ``quantize_search`` (with and without importance weights),
  ``prepare_layer`` with importance weights (one expert with no tokens), and the global scale ``448.0 * 6.0 / t``
  over many maxima (torch evaluates it as ``t.reciprocal() * 2688``, which a true division misses about one time
  in four).
* ``nvfp4_layer.npz`` -- the whole NVFP4 routed layer as vLLM's NVFP4 emulation MoE computes it
  (``vllm/model_executor/layers/fused_moe/experts/nvfp4_emulation_moe.py:83-160``): weights prepared by the
  reference's own ``prepare_layer`` and dequantised by vLLM's ``dequantize_to_dtype`` (times 1/g per expert, bf16),
  activations quantise-dequantised by vLLM's Triton ``_nvfp4_quant_dequant_kernel`` (global scales
  448*6/(1.25*amax), the reference's nvfp4.py:125-126), then vLLM's ``fused_moe_kernel`` in bf16 for both GEMMs,
  ``SiluAndMul.forward_native`` between them and the top-k sum.  The reference itself runs FlashInfer's closed
  CUTLASS MoE here; this chain is the readable restatement of the same quantised arithmetic (it rounds the
  dequantised operands to bf16, which the real FP4 GEMM does not, so it pins the layer within the bf16 tolerance).
"""

from __future__ import annotations

import os

os.environ["TRITON_INTERPRET"] = "1"

import sys  # noqa: E402
from pathlib import Path  # noqa: E402
from types import SimpleNamespace  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402

OUT = Path(__file__).resolve().parent
FP8 = torch.float8_e4m3fn


def _patch_interpreter_rounding() -> None:
    """The Triton CPU interpreter's own float-narrowing helper (triton/runtime/interpreter.py `_convert_float`)
    truncates fp32->bf16 and rounds fp32->fp8 half-up without carrying into the exponent (31.99 becomes 16),
    whereas compiled Triton narrows with round-to-nearest-even (cvt.rn[.satfinite]).  Narrowing conversions to
    bf16 / fp16 / e4m3 are therefore routed through torch's RNE conversion; widening ones are exact and keep the
    interpreter's path.  This corrects the tool, not the kernels being interpreted."""
    import triton.language as tl
    from triton.runtime import interpreter as itp

    orig = itp._convert_float
    narrow = {tl.bfloat16: (torch.bfloat16, torch.uint16), tl.float16: (torch.float16, torch.uint16),
              tl.float8e4nv: (FP8, torch.uint8)}

    def convert(input, input_dtype, output_dtype, rounding_mode):
        if input_dtype == tl.float32 and output_dtype in narrow:
            to, view = narrow[output_dtype]
            t = torch.from_numpy(np.frombuffer(input.tobytes(), dtype=np.float32).copy())
            return t.to(to).view(view).numpy().reshape(input.shape)
        return orig(input, input_dtype, output_dtype, rounding_mode)

    itp._convert_float = convert


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.uint16).numpy().copy()
    if t.dtype == FP8:
        return t.contiguous().view(torch.uint8).numpy().copy()
    return t.contiguous().numpy().copy()


def _fp8_blocks(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """128x128 block FP8 with scale = amax/448, the recipe of the reference's tests/test_nvfp4.py:32-39."""
    e, r, c = w.shape
    v = w.view(e, r // 128, 128, c // 128, 128)
    s = v.abs().amax((2, 4)) / 448.0
    q = (v / s.view(e, r // 128, 1, c // 128, 1).clamp(min=1e-12)).clamp(-448, 448).to(FP8)
    return q.view(e, r, c), s.float().contiguous()


def _align(flat_ids: torch.Tensor, num_experts: int, bm: int):
    """moe_align_block_size's documented result: ascending flat indices per expert, padded with numel."""
    n = flat_ids.numel()
    sorted_ids, expert_ids = [], []
    for e in range(num_experts):
        idx = (flat_ids == e).nonzero().flatten().tolist()
        pad = (-len(idx)) % bm
        sorted_ids += idx + [n] * pad
        expert_ids += [e] * ((len(idx) + pad) // bm)
    return (
        torch.tensor(sorted_ids, dtype=torch.int32),
        torch.tensor(expert_ids, dtype=torch.int32),
        torch.tensor([len(sorted_ids)], dtype=torch.int32),
    )


def _triton_group_quant(x: torch.Tensor, ue8m0: bool = False):
    from vllm.model_executor.layers.quantization.utils import fp8_utils

    rows, cols = x.shape
    q = torch.empty(rows, cols, dtype=FP8)
    s = torch.empty(rows, cols // 128, dtype=torch.float32)
    fp8_utils._per_token_group_quant_fp8[(rows * cols // 128,)](
        x, q, s, 128, cols, cols, 1e-10, -448.0, 448.0, ue8m0, BLOCK=128
    )
    return q, s


def _triton_gemm(a, a_s, w, w_s, c, weights, sorted_ids, expert_ids, npp, top_k, mul_routed_weight, bm):
    import triton
    import triton.language as tl
    from vllm.model_executor.layers.fused_moe import fused_moe as fm

    E, N, K = w.shape
    em = sorted_ids.numel()
    bn = 64
    grid = (triton.cdiv(em, bm) * triton.cdiv(N, bn),)
    fm.fused_moe_kernel[grid](
        a, w, c, None, a_s, w_s, weights, sorted_ids, expert_ids, npp,
        N, K, em, weights.numel(),
        a.stride(0), a.stride(1), w.stride(0), w.stride(2), w.stride(1), c.stride(-2), c.stride(-1),
        a_s.stride(0), a_s.stride(1), w_s.stride(0), w_s.stride(2), w_s.stride(1), 0, 0,
        group_n=128, group_k=128, naive_block_assignment=False,
        BLOCK_SIZE_M=bm, BLOCK_SIZE_N=bn, BLOCK_SIZE_K=128, GROUP_SIZE_M=1, SPLIT_K=1,
        MUL_ROUTED_WEIGHT=mul_routed_weight, top_k=top_k, compute_type=tl.bfloat16, use_fp8_w8a8=True,
        use_int8_w8a8=False, use_int8_w8a16=False, per_channel_quant=False, HAS_BIAS=False,
    )


def make_fp8_layer(seed: int = 7, T: int = 24, H: int = 256, I: int = 128, E: int = 8, k: int = 4,
                   ue8m0: bool = False):
    """With ue8m0 both activation quantisations take power-of-two scales (vLLM's DeepGEMM-E8M0 mode, the default
    where DeepGEMM is installed) and the fixture is fp8_layer_ue8m0.npz."""
    from vllm.model_executor.layers.activation import SiluAndMul

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    x[3] = 0.0  # an all-zero token: every group takes the 1e-10 floor scale
    x[5, :128] *= 200.0  # a token with a large group
    logits = torch.randn(T, E, generator=g)
    logits[:, E - 1] -= 40.0  # the last expert receives no token (a zero-block expert)
    logits = logits.to(torch.bfloat16)
    w1, w1_s = _fp8_blocks(torch.randn(E, 2 * I, H, generator=g) * 0.02)
    w2, w2_s = _fp8_blocks(torch.randn(E, H, I, generator=g) * 0.02)

    probs = torch.softmax(logits.float(), dim=-1)
    top_w, top_i = torch.topk(probs, k, dim=-1)
    top_w = top_w / top_w.sum(-1, keepdim=True)
    top_i = top_i.to(torch.int32)

    bm = 16
    sorted_ids, expert_ids, npp = _align(top_i.flatten(), E, bm)
    xq, xs = _triton_group_quant(x, ue8m0)
    c1 = torch.zeros(T, k, 2 * I, dtype=torch.bfloat16)
    _triton_gemm(xq, xs, w1, w1_s, c1, top_w.flatten().contiguous(), sorted_ids, expert_ids, npp, k, False, bm)
    c2 = SiluAndMul.forward_native(c1.view(-1, 2 * I))
    c2q, c2s = _triton_group_quant(c2.contiguous(), ue8m0)
    c3 = torch.zeros(T * k, H, dtype=torch.bfloat16)
    _triton_gemm(c2q, c2s, w2, w2_s, c3, top_w.flatten().contiguous(), sorted_ids, expert_ids, npp, 1, True, bm)
    out = c3.view(T, k, H).sum(dim=1)

    np.savez_compressed(
        OUT / ("fp8_layer_ue8m0.npz" if ue8m0 else "fp8_layer.npz"),
        x=_bits(x), logits=_bits(logits), w1=_bits(w1), w1_s=_bits(w1_s), w2=_bits(w2), w2_s=_bits(w2_s),
        top_w=_bits(top_w.float()), top_i=_bits(top_i), sorted_ids=_bits(sorted_ids), expert_ids=_bits(expert_ids),
        x_q=_bits(xq), x_s=_bits(xs), c1=_bits(c1), c2=_bits(c2), c2q=_bits(c2q), c2s=_bits(c2s), c3=_bits(c3),
        out=_bits(out), k=np.int32(k), block_m=np.int32(bm),
    )


def make_quant_edges():
    """Extra rows for the activation quantiser: zeros, a single spike, tiny values, exact-tie magnitudes."""
    g = torch.Generator().manual_seed(3)
    rows = [torch.randn(2048, generator=g) for _ in range(6)]
    rows.append(torch.zeros(2048))
    spike = torch.zeros(2048)
    spike[17] = 3.0e4
    rows.append(spike)
    rows.append(torch.randn(2048, generator=g) * 1e-30)
    ties = torch.arange(2048, dtype=torch.float32) % 129 - 64.0
    rows.append(ties)
    x = torch.stack(rows).to(torch.bfloat16)
    q, s = _triton_group_quant(x)
    qe, se = _triton_group_quant(x, ue8m0=True)
    np.savez_compressed(OUT / "act_quant.npz", x=_bits(x), q=_bits(q), s=_bits(s), q_ue8m0=_bits(qe),
                        s_ue8m0=_bits(se))


def make_align_kat():
    ids = torch.tensor([[2, 3, 4], [1, 2, 4], [1, 3, 4], [1, 2, 3]], dtype=torch.int32)
    sorted_ids = np.array([3, 6, 9, 12, 0, 4, 10, 12, 1, 7, 11, 12, 2, 5, 8, 12], np.int32)
    expert_ids = np.array([1, 2, 3, 4], np.int32)
    np.savez_compressed(
        OUT / "align_kat.npz", ids=_bits(ids), num_experts=np.int32(5), block_m=np.int32(4),
        sorted_ids=sorted_ids, expert_ids=expert_ids, num_post_pad=np.int32(16),
    )


def make_router(seed: int = 11, T: int = 96, H: int = 2048, E: int = 128, k: int = 8):
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeTopKRouter

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    router = Qwen3_5MoeTopKRouter(SimpleNamespace(num_experts_per_tok=k, num_experts=E, hidden_size=H))
    with torch.no_grad():
        router.weight.copy_((torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16))
        router = router.to(torch.bfloat16)
        logits = torch.nn.functional.linear(x, router.weight)
        probs, scores, idx = router(x)
    assert torch.equal(probs, torch.softmax(logits, dtype=torch.float, dim=-1))
    srt = torch.sort(logits.float(), dim=-1, descending=True).values
    ties_at_cut = int((srt[:, k - 1] == srt[:, k]).sum())
    np.savez_compressed(
        OUT / "router.npz", x=_bits(x), weight=_bits(router.weight.detach()), logits=_bits(logits),
        scores=_bits(scores.float()), ids=_bits(idx.to(torch.int32)), k=np.int32(k), ties_at_cut=np.int32(ties_at_cut),
    )


def make_nvfp4():
    from prismyra.kernels.nvfp4 import _dequant_fp8, prepare_layer, quantize
    from vllm.model_executor.layers.quantization.utils.nvfp4_emulation_utils import _triton_nvfp4_quant_dequant

    g = torch.Generator().manual_seed(5)
    w = torch.randn(64, 256, generator=g) * 0.05
    w[0] = 0.0  # an all-zero row: every scale 0, every code 0
    w[1, :16] = torch.tensor([0.75, -0.75, 0.25, -0.25, 1.25, 2.5, 5.0, 3.5, 1.75, -1.75, 6.0, -6.0, 0.0, 0.1, -0.1, 4.0])
    gs = float(448.0 * 6.0 / w.abs().amax())
    packed, scale = quantize(w, torch.tensor(gs))

    wq, ws = _fp8_blocks(torch.randn(2, 256, 256, generator=g) * 0.02)
    wq2, ws2 = _fp8_blocks(torch.randn(2, 256, 128, generator=g) * 0.02)
    deq = _dequant_fp8(wq[0], ws[0])
    prep = prepare_layer(wq, ws, wq2, ws2, "cpu")

    xa = (torch.randn(8, 256, generator=g) * 2.0).to(torch.bfloat16)
    xa[2] = 0.0
    a_gs = torch.tensor([448.0 * 6.0 / float(xa.float().abs().amax())], dtype=torch.float32)
    xdq = _triton_nvfp4_quant_dequant(xa.float(), a_gs, 16)

    np.savez_compressed(
        OUT / "nvfp4.npz", w=_bits(w), gs=np.float32(gs), packed=_bits(packed), scale=_bits(scale),
        fp8_w=_bits(wq), fp8_s=_bits(ws), fp8_w2=_bits(wq2), fp8_s2=_bits(ws2), dequant0=_bits(deq),
        prep_w1=_bits(prep["w1"]), prep_s1=_bits(prep["s1"]), prep_g1=_bits(prep["g1"]),
        prep_w2=_bits(prep["w2"]), prep_s2=_bits(prep["s2"]), prep_g2=_bits(prep["g2"]),
        act_x=_bits(xa), act_gs=_bits(a_gs), act_dequant=_bits(xdq),
    )


def make_nvfp4_search():
    from prismyra.kernels.nvfp4 import prepare_layer, quantize_search

    g = torch.Generator().manual_seed(9)
    w = torch.randn(96, 256, generator=g) * 0.04
    w[3] = 0.0
    imp = torch.rand(256, generator=g) * 2.0
    gs = 448.0 * 6.0 / w.abs().amax()
    p_imp, s_imp = quantize_search(w, gs, imp)
    p_one, s_one = quantize_search(w, gs, None)
    wq, ws = _fp8_blocks(torch.randn(3, 256, 256, generator=g) * 0.02)
    wq2, ws2 = _fp8_blocks(torch.randn(3, 256, 128, generator=g) * 0.02)
    imp_in = torch.rand(3, 256, generator=g)
    imp_mid = torch.rand(3, 128, generator=g)
    tok = torch.tensor([5, 0, 2])
    prep = prepare_layer(wq, ws, wq2, ws2, "cpu", imp_in=imp_in, imp_mid=imp_mid, tok=tok)
    amax = torch.rand(4096, generator=g) * 0.5 + 1e-4
    np.savez_compressed(
        OUT / "nvfp4_search.npz", w=_bits(w), imp=_bits(imp), gs=_bits(gs.reshape(1)),
        p_imp=_bits(p_imp), s_imp=_bits(s_imp), p_one=_bits(p_one), s_one=_bits(s_one),
        fp8_w=_bits(wq), fp8_s=_bits(ws), fp8_w2=_bits(wq2), fp8_s2=_bits(ws2), imp_in=_bits(imp_in),
        imp_mid=_bits(imp_mid), tok=tok.numpy(),
        prep_w1=_bits(prep["w1"]), prep_s1=_bits(prep["s1"]), prep_g1=_bits(prep["g1"]),
        prep_w2=_bits(prep["w2"]), prep_s2=_bits(prep["s2"]), prep_g2=_bits(prep["g2"]),
        amax=_bits(amax), gscale=_bits(448.0 * 6.0 / amax),
    )


def _triton_gemm_bf16(a, w, c, weights, sorted_ids, expert_ids, npp, top_k, mul_routed_weight, bm):
    """vLLM's fused_moe_kernel with bf16 operands (no quantisation), as TritonExperts runs it after the NVFP4
    emulation has dequantised the weights.  The Triton CPU interpreter's dot multiplies bf16 operands as their raw
    16-bit patterns, so the operands are handed over as fp32 copies of the same bf16 values: every product of two
    bf16 values is exact in fp32 and the sum is an fp32 accumulation, which is what the compiled kernel's bf16
    tensor-core dot computes.  This corrects the tool, not the kernel being interpreted."""
    import triton
    import triton.language as tl
    from vllm.model_executor.layers.fused_moe import fused_moe as fm

    E, N, K = w.shape
    a, w = a.float().contiguous(), w.float().contiguous()
    em = sorted_ids.numel()
    bn = 64
    grid = (triton.cdiv(em, bm) * triton.cdiv(N, bn),)
    fm.fused_moe_kernel[grid](
        a, w, c, None, None, None, weights, sorted_ids, expert_ids, npp,
        N, K, em, weights.numel(),
        a.stride(0), a.stride(1), w.stride(0), w.stride(2), w.stride(1), c.stride(-2), c.stride(-1),
        0, 0, 0, 0, 0, 0, 0,
        group_n=0, group_k=0, naive_block_assignment=False,
        BLOCK_SIZE_M=bm, BLOCK_SIZE_N=bn, BLOCK_SIZE_K=64, GROUP_SIZE_M=1, SPLIT_K=1,
        MUL_ROUTED_WEIGHT=mul_routed_weight, top_k=top_k, compute_type=tl.bfloat16, use_fp8_w8a8=False,
        use_int8_w8a8=False, use_int8_w8a16=False, per_channel_quant=False, HAS_BIAS=False,
    )


def make_nvfp4_layer(seed: int = 13, T: int = 24, H: int = 256, I: int = 256, E: int = 8, k: int = 4):
    from prismyra.kernels.nvfp4 import prepare_layer
    from vllm.model_executor.layers.activation import SiluAndMul
    from vllm.model_executor.layers.quantization.utils.nvfp4_emulation_utils import (
        _triton_nvfp4_quant_dequant, dequantize_to_dtype)

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    x[4] = 0.0  # an all-zero token: every group scale is 0
    logits = torch.randn(T, E, generator=g)
    logits[:, 2] -= 40.0  # expert 2 receives no token
    logits = logits.to(torch.bfloat16)
    w13, s13 = _fp8_blocks(torch.randn(E, 2 * I, H, generator=g) * 0.02)
    w2f, s2f = _fp8_blocks(torch.randn(E, H, I, generator=g) * 0.02)
    prep = prepare_layer(w13, s13, w2f, s2f, "cpu")

    probs = torch.softmax(logits.float(), dim=-1)
    top_w, top_i = torch.topk(probs, k, dim=-1)
    top_w = top_w / top_w.sum(-1, keepdim=True)
    top_i = top_i.to(torch.int32)

    # synthetic calibration: the activation maxima the reference reads from its calibration file
    a1_amax = float(x.float().abs().max())
    w1d = _fp8_deq(w13, s13)
    h = torch.einsum("th,tkih->tki", x.float(), w1d[top_i.long()])
    a2_amax = float((torch.nn.functional.silu(h[..., :I]) * h[..., I:]).abs().max())
    a1_gs = torch.tensor([448.0 * 6.0 / (1.25 * a1_amax)], dtype=torch.float32)
    a2_gs = torch.tensor([448.0 * 6.0 / (1.25 * a2_amax)], dtype=torch.float32)

    w1_dq = dequantize_to_dtype(prep["w1"], prep["s1"].view(torch.uint8), 1.0 / prep["g1"], torch.bfloat16,
                                16, swizzle=False)
    w2_dq = dequantize_to_dtype(prep["w2"], prep["s2"].view(torch.uint8), 1.0 / prep["g2"], torch.bfloat16,
                                16, swizzle=False)
    bm = 16
    sorted_ids, expert_ids, npp = _align(top_i.flatten(), E, bm)
    x_dq = _triton_nvfp4_quant_dequant(x, a1_gs, 16)
    c1 = torch.zeros(T, k, 2 * I, dtype=torch.bfloat16)
    _triton_gemm_bf16(x_dq, w1_dq, c1, top_w.flatten().contiguous(), sorted_ids, expert_ids, npp, k, False, bm)
    c2 = SiluAndMul.forward_native(c1.view(-1, 2 * I))
    c2_dq = _triton_nvfp4_quant_dequant(c2.contiguous(), a2_gs, 16)
    c3 = torch.zeros(T * k, H, dtype=torch.bfloat16)
    _triton_gemm_bf16(c2_dq, w2_dq, c3, top_w.flatten().contiguous(), sorted_ids, expert_ids, npp, 1, True, bm)
    out = c3.view(T, k, H).sum(dim=1)

    np.savez_compressed(
        OUT / "nvfp4_layer.npz",
        x=_bits(x), logits=_bits(logits), w1=_bits(prep["w1"]), s1=_bits(prep["s1"]), g1=_bits(prep["g1"]),
        w2=_bits(prep["w2"]), s2=_bits(prep["s2"]), g2=_bits(prep["g2"]), a1_gs=_bits(a1_gs), a2_gs=_bits(a2_gs),
        top_w=_bits(top_w.float()), top_i=_bits(top_i), x_dq=_bits(x_dq), c1=_bits(c1), c2=_bits(c2),
        c2_dq=_bits(c2_dq), c3=_bits(c3), out=_bits(out), k=np.int32(k),
    )


def _fp8_deq(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    e, r, c = q.shape
    return (q.float().view(e, r // 128, 128, c // 128, 128) * s.view(e, r // 128, 1, c // 128, 1)).view(e, r, c)


if __name__ == "__main__":
    if not any("reference" in p for p in sys.path):
        print("note: PYTHONPATH should hold the reference checkout for the NVFP4 fixtures", file=sys.stderr)
    if sys.argv[1:] == ["nvfp4_search"]:
        make_nvfp4_search()
        sys.exit(0)
    _patch_interpreter_rounding()
    if sys.argv[1:] == ["nvfp4_layer"]:
        make_nvfp4_layer()
        sys.exit(0)
    if sys.argv[1:] == ["ue8m0"]:
        make_quant_edges()
        make_fp8_layer(ue8m0=True)
        sys.exit(0)
    make_align_kat()
    make_router()
    make_quant_edges()
    make_fp8_layer()
    make_fp8_layer(ue8m0=True)
    make_nvfp4()
    make_nvfp4_search()
    make_nvfp4_layer()
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)
