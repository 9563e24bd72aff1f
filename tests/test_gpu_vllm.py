"""This repository's layer against the kernels the reference itself runs on a GPU (prismyra/kernels/qwen3_moe.py:
184-197: vLLM's fused_topk and fused_experts, FP8 w8a8 with 128x128 block scales), on the same seeded tensors and the
same router logits.  Routing ids bit-exact against vLLM's topk_softmax; layer output within the north-star
tolerance (relative L2 <= 1e-2, max <= 1e-2 * max|ref|).  Skipped, with the reason, when vLLM does not import.

On a GPU vLLM quantises activations with its compiled quantiser: scales max(amax, 1e-10)/448 correctly rounded (the
library's default rule), or, when it runs DeepGEMM with E8M0 scales (``VLLM_USE_DEEP_GEMM_E8M0``, on by default
where DeepGEMM is installed), those scales rounded up to powers of two (the library's "ue8m0" rule).  Both settings
are compared, each with its own rule."""

from __future__ import annotations

import pytest
import torch

from tests.conftest import cuda_ok

pytestmark = pytest.mark.gpu

if cuda_ok():
    from prismyra_b200 import ops, synth

DEV = "cuda:0"
K = 8


def _vllm():
    try:
        from vllm.model_executor.layers.fused_moe import fused_experts, fused_topk
        from vllm.model_executor.layers.fused_moe.config import FusedMoEQuantConfig
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"vllm does not import here: {type(e).__name__}: {e}")
    return fused_experts, fused_topk, FusedMoEQuantConfig


@pytest.fixture(scope="module")
def layer():
    L = synth.make_fp8_layer(T=5120, seed=0, device="cpu")
    return {k: v.to(DEV) for k, v in L.items()}


@pytest.mark.parametrize("T", [128, 512, 5120])
def test_routed_layer_matches_vllm_fused_experts(layer, T, monkeypatch):
    monkeypatch.setenv("VLLM_USE_DEEP_GEMM_E8M0", "0")
    fused_experts, fused_topk, QC = _vllm()
    x = layer["x"][:T].contiguous()
    logits, w, ids = ops.router_topk(x, layer["router_w"], K)
    vw, vids = fused_topk(x, logits, K, renormalize=True)[:2]
    assert torch.equal(ids, vids.to(torch.int32))
    torch.testing.assert_close(w, vw, rtol=1e-6, atol=0)
    quant = QC.make(quant_dtype=torch.float8_e4m3fn, block_shape=[128, 128], w1_scale=layer["w1_s"],
                    w2_scale=layer["w2_s"])
    ref = fused_experts(x, layer["w1"], layer["w2"], vw, vids, quant_config=quant).float()
    out = ops.forward_fp8(x, layer["w1"], layer["w1_s"], layer["w2"], layer["w2_s"], K, logits=logits).float()
    l2 = float((out - ref).norm() / ref.norm())
    mx = float((out - ref).abs().max() / ref.abs().max())
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)


@pytest.mark.parametrize("T", [128, 5120])
def test_ue8m0_mode_matches_vllm_default_with_deepgemm_e8m0(layer, T, monkeypatch):
    """vLLM's default where DeepGEMM runs with E8M0 scales (VLLM_USE_DEEP_GEMM_E8M0=1): both activation
    quantisations take power-of-two scales.  The layer's act_scale="ue8m0" mode is that arithmetic."""
    monkeypatch.setenv("VLLM_USE_DEEP_GEMM_E8M0", "1")
    fused_experts, fused_topk, QC = _vllm()
    from vllm.utils import deep_gemm

    if not deep_gemm.is_deep_gemm_e8m0_used():
        pytest.skip("vLLM does not run DeepGEMM with E8M0 scales on this host")
    x = layer["x"][:T].contiguous()
    logits, w, ids = ops.router_topk(x, layer["router_w"], K)
    vw, vids = fused_topk(x, logits, K, renormalize=True)[:2]
    quant = QC.make(quant_dtype=torch.float8_e4m3fn, block_shape=[128, 128], w1_scale=layer["w1_s"],
                    w2_scale=layer["w2_s"])
    ref = fused_experts(x, layer["w1"], layer["w2"], vw, vids, quant_config=quant).float()
    out = ops.forward_fp8(x, layer["w1"], layer["w1_s"], layer["w2"], layer["w2_s"], K, logits=logits,
                          act_scale="ue8m0").float()
    l2 = float((out - ref).norm() / ref.norm())
    mx = float((out - ref).abs().max() / ref.abs().max())
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)
    # and the fp32-scale mode is what differs from vLLM's E8M0 default by an e4m3 quantisation step
    out32 = ops.forward_fp8(x, layer["w1"], layer["w1_s"], layer["w2"], layer["w2_s"], K, logits=logits).float()
    assert float((out32 - ref).norm() / ref.norm()) > 5 * l2


@pytest.mark.parametrize("ue8m0", [False, True])
def test_activation_quantisation_matches_vllm_cuda_op(layer, ue8m0):
    """vLLM's compiled per_token_group_quant_fp8 (the op its fused_experts runs on a GPU) against the library's
    quantisation kernel: scales bit-exact; codes bit-exact (power-of-two scales make the quotient exact, and with
    fp32 scales both round the IEEE quotient to nearest even)."""
    _vllm()
    from vllm.model_executor.layers.quantization.utils import fp8_utils

    x = layer["x"]
    qv, sv = fp8_utils.per_token_group_quant_fp8(x, 128, use_ue8m0=ue8m0)
    q, s = ops.quant_fp8(x, act_scale="ue8m0" if ue8m0 else "fp32")
    assert torch.equal(s, sv)
    assert torch.equal(q.view(torch.uint8), qv.view(torch.uint8))
