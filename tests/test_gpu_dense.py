"""Dense block-FP8 projections (the reference's Fp8Linear and _FusedDenseProjection) on the B200 kernel against
the CPU oracle, through the C ABI.

Tolerances: outputs relative L2 <= 1e-2 and max <= 1e-2 * max|ref| against the oracle's per-K-block exact product
sums (the north-star bf16 tolerance); the fused projection equal, bit for bit, to the separate ones; row-count
invariance and determinism bit-exact.
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


def _weights(N, K, seed):
    g = torch.Generator().manual_seed(seed)
    return synth.quantize_fp8_blocks(torch.randn(N, K, generator=g) * 0.02)


def _oracle(x_cpu, w, s):
    q, qs = O.quant_fp8_groups(bits(x_cpu))
    acc = O.gemm_fp8_rows(q, qs, np.zeros(q.shape[0], np.int32), bits(w)[None], bits(s)[None])
    return O.f32_to_bf16(acc)


@pytest.mark.parametrize("T,K,N", [(1, 2048, 2048), (37, 2048, 4096), (300, 512, 2048), (1000, 2048, 768 * 2)])
def test_fp8_linear_matches_oracle(T, K, N):
    w, s = _weights(N, K, T + N)
    x = torch.randn(T, K, generator=torch.Generator().manual_seed(T)).to(torch.bfloat16)
    out = ops.fp8_linear(x.to(DEV), w.to(DEV), s.to(DEV))
    l2, mx = rel_err(bits(out), _oracle(x, w, s))
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)


def test_fp8_linear_row_invariant_deterministic_and_shaped():
    w, s = _weights(4096, 2048, 5)
    w, s = w.to(DEV), s.to(DEV)
    x = torch.randn(6, 100, 2048, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16).to(DEV)
    full = ops.fp8_linear(x, w, s)
    assert full.shape == (6, 100, 4096)
    assert torch.equal(full, ops.fp8_linear(x, w, s))
    flat = x.reshape(-1, 2048)
    for T in (1, 7, 128, 129, 600):
        assert torch.equal(ops.fp8_linear(flat[:T].contiguous(), w, s), full.reshape(-1, 4096)[:T]), T


def test_fused_projection_equals_separate_projections():
    """Three siblings of one input (widths 1024, 512, 512) through one matmul equal their three separate calls."""
    from transformers.integrations.finegrained_fp8 import FP8Linear

    from prismyra_b200.kernels.qwen3_moe import Fp8Linear, FusedDenseProjection

    def fp8_module(N, K, seed):
        w, s = _weights(N, K, seed)
        m = FP8Linear(K, N, block_size=(128, 128))
        m.weight = nn.Parameter(w, requires_grad=False)
        m.weight_scale_inv = nn.Parameter(s, requires_grad=False)
        return m.to(DEV)

    parts = [Fp8Linear(fp8_module(n, 2048, 40 + i)) for i, n in enumerate((1024, 512, 512))]
    fused = FusedDenseProjection(parts)
    x = torch.randn(333, 2048, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(DEV)
    outs = fused(x)
    assert [o.shape[-1] for o in outs] == [1024, 512, 512]
    for p, o in zip(parts, outs):
        assert torch.equal(o, p(x))
