"""Whole-layer parity with the CPU oracle at the benchmarked configurations (all calls through the C ABI).

The benchmark's token counts take the large-tile persistent GEMMs (T*k > 32*E): many tiles per CTA, the tile-to-tile
hand-off of the two TMEM accumulators, the next tile's scale / flat-index prefetch, and experts spanning several
128-row blocks.  Here those paths are compared with the oracle, not only with themselves:

* the FP8 layer at T=5120, seed 0, every token against the oracle;
* the same layer with one hot expert taking 2,000 tokens (16 blocks), other experts on random logits;
* T=513 (the smallest token count on the large-tile GEMMs at E=128, k=8) and T=2049;
* the NVFP4 layer at T=5120 (weights from the FP8 layer by the reference's prepare_layer
  recipe, on the GPU), a spread 1,024-token subset against the oracle.

Tolerances as in the stage tests: routing ids and the expert permutation bit-exact; layer outputs relative L2
<= 1e-2 and max <= 1e-2 * max|ref| for FP8 (2e-2 max for NVFP4, whose intermediate requantisation to e2m1 moves a
code by a whole step when the two sides' fp32 sums straddle a rounding boundary).  A token's output depends only on
its own row, its logits and the expert weights, so the oracle may be evaluated on a subset of the tokens the GPU
computed together.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.conftest import cuda_ok

pytestmark = pytest.mark.gpu

if cuda_ok():
    from prismyra_b200 import _lib, ops, synth

DEV = "cuda:0"
H, I, E, K = 2048, 768, 128, 8


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
def layer():
    """T=5120, H=2048, I=768, E=128, seed 0 (drawn on the CPU, as bench.py does)."""
    L = synth.make_fp8_layer(T=5120, H=H, I=I, E=E, seed=0, device="cpu")
    gpu = {k: v.to(DEV) for k, v in L.items()}
    cpu = {k: bits(v) for k, v in L.items()}
    return cpu, gpu


def _fp8_oracle(cpu, x_bits, logits_bits):
    return O.moe_forward_fp8(x_bits, logits_bits, cpu["w1"], cpu["w1_s"], cpu["w2"], cpu["w2_s"], K)["out"]


def _check_routing_and_permutation(gpu, x, T):
    """The forward's own router output and expert alignment, read back from its workspace, against the oracle."""
    ws, _ = ops.workspace_for(x, T, H, I, E, K)
    ops.read_status(ws)
    reg = lambda name, dt, shape: ops.region(ws, T, H, I, E, K, 0, name, dt, shape)
    logits = reg("logits", torch.bfloat16, (T, E)).clone()
    ids = reg("topk_ids", torch.int32, (T, K))
    rw, rids = O.route_topk(bits(logits), K)
    assert np.array_equal(bits(ids), rids)
    np.testing.assert_allclose(bits(reg("topk_w", torch.float32, (T, K))), rw, rtol=1e-6)
    ms = _lib.max_slots(T, E, K)
    rs, re, rn = O.align(rids, E, 128)
    npp = int(bits(reg("num_post_pad", torch.int32, (1,)))[0])
    assert npp == rn
    assert np.array_equal(bits(reg("sorted", torch.int32, (ms,)))[:rn], rs)
    assert np.array_equal(bits(reg("expert_ids", torch.int32, (ms // 128,)))[: rn // 128], re)
    return logits, rids


def test_fp8_t5120_matches_oracle_on_every_token(layer):
    cpu, gpu = layer
    T = 5120
    x = gpu["x"]
    out = ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, router_w=gpu["router_w"]).clone()
    logits, rids = _check_routing_and_permutation(gpu, x, T)
    counts = np.bincount(rids.reshape(-1), minlength=E)
    assert (counts > 128).sum() > 100  # most experts span several 128-row blocks at this size
    ref = _fp8_oracle(cpu, cpu["x"], bits(logits))
    l2, mx = rel_err(bits(out), ref)
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)


def test_fp8_t5120_with_a_hot_expert(layer):
    """Expert 5 is in the top-k of tokens 0..1999 (16 blocks of one expert in a row, spread over many CTAs); the
    other slots follow random logits.  Oracle on every third token (each token's output is its own)."""
    cpu, gpu = layer
    T = 5120
    g = torch.Generator().manual_seed(11)
    logits = torch.randn(T, E, generator=g) * 0.5
    logits[:2000, 5] = 6.0
    logits = logits.to(torch.bfloat16)
    out = ops.forward_fp8(gpu["x"], gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, logits=logits.to(DEV))
    ws, _ = ops.workspace_for(gpu["x"], T, H, I, E, K)
    ops.read_status(ws)
    _, rids = O.route_topk(bits(logits), K)
    got_ids = ops.region(ws, T, H, I, E, K, 0, "topk_ids", torch.int32, (T, K))
    assert np.array_equal(bits(got_ids), rids)
    assert np.bincount(rids.reshape(-1), minlength=E)[5] >= 2000  # 16+ blocks of one expert
    sub = np.arange(0, T, 3)
    ref = _fp8_oracle(cpu, cpu["x"][sub], bits(logits)[sub])
    l2, mx = rel_err(bits(out)[sub], ref)
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)


@pytest.mark.parametrize("T", [513, 2049])
def test_fp8_large_tile_thresholds_match_oracle(layer, T):
    cpu, gpu = layer
    x = gpu["x"][:T].contiguous()
    assert T * K > 32 * E  # the large-tile GEMMs
    out = ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, router_w=gpu["router_w"]).clone()
    logits, _ = _check_routing_and_permutation(gpu, x, T)
    ref = _fp8_oracle(cpu, cpu["x"][:T], bits(logits))
    l2, mx = rel_err(bits(out), ref)
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)


def test_fp8_t5120_ue8m0_mode_matches_oracle(layer):
    """The power-of-two activation-scale mode (vLLM's DeepGEMM-E8M0 arithmetic) at BASELINE configs[1]: routing and
    permutation as in the fp32 mode, output against the oracle in the same mode on a spread 1,024-token subset."""
    cpu, gpu = layer
    x = gpu["x"]
    out = ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, router_w=gpu["router_w"],
                          act_scale="ue8m0").clone()
    logits, _ = _check_routing_and_permutation(gpu, x, 5120)
    sub = np.linspace(0, 5119, 1024).astype(np.int64)
    ref = O.moe_forward_fp8(cpu["x"][sub], bits(logits)[sub], cpu["w1"], cpu["w1_s"], cpu["w2"], cpu["w2_s"], K,
                            scale="ue8m0")["out"]
    l2, mx = rel_err(bits(out)[sub], ref)
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)


def test_golden_fp8_layer_ue8m0_through_gpu(golden):
    """vLLM's Triton chain in its power-of-two scale mode (tests/golden/fp8_layer_ue8m0.npz) through the CUDA path."""
    g = golden("fp8_layer_ue8m0")
    k = int(g["k"])
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(DEV)
    f8 = lambda a: torch.from_numpy(a).view(torch.float8_e4m3fn).to(DEV)
    out = ops.forward_fp8(bf(g["x"]), f8(g["w1"]), torch.from_numpy(g["w1_s"]).to(DEV), f8(g["w2"]),
                          torch.from_numpy(g["w2_s"]).to(DEV), k, logits=bf(g["logits"]), act_scale="ue8m0")
    l2, mx = rel_err(bits(out), g["out"])
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)


def test_nvfp4_t5120_matches_oracle(layer):
    """NVFP4 weights prepared from the seed-0 FP8 layer on the GPU (bit-exact with the
    reference's prepare_layer, tested elsewhere), synthetic calibration; a spread 1,024-token subset."""
    cpu, gpu = layer
    T = 5120
    nw = synth.nvfp4_device_layer(gpu, DEV)
    prep_cpu = {k: bits(nw[k]) for k in ("w1", "w2")}
    from prismyra_b200.kernels import nvfp4

    s1 = nvfp4.unblock_scales(nw["w1_sf"].cpu().reshape(-1, H // 64, 512), E * 2 * I, H // 16).numpy()
    s2 = nvfp4.unblock_scales(nw["w2_sf"].cpu().reshape(-1, I // 64, 512), E * H, I // 16).numpy()
    x = gpu["x"]
    logits, _, _ = ops.router_topk(x, gpu["router_w"], K)
    out = ops.forward_nvfp4(x, nw["w1"], nw["w1_sf"], nw["al1"], nw["a1"], nw["w2"], nw["w2_sf"], nw["al2"],
                            nw["a2"], K, router_w=gpu["router_w"])
    ws, _ = ops.workspace_for(x, T, H, I, E, K, _lib.FMT_NVFP4)
    ops.read_status(ws)
    sub = np.linspace(0, T - 1, 1024).astype(np.int64)
    ref = O.moe_forward_nvfp4(cpu["x"][sub], bits(logits)[sub], prep_cpu["w1"], s1.reshape(E, 2 * I, H // 16),
                              prep_cpu["w2"], s2.reshape(E, H, I // 16), bits(nw["al1"]), bits(nw["al2"]), nw["a1"],
                              nw["a2"], K)
    l2, mx = rel_err(bits(out)[sub], ref["out"])
    assert l2 < 1e-2 and mx < 2e-2, (l2, mx)


def test_nvfp4_layer_fixture_through_gpu(golden):
    """vLLM's NVFP4 emulation MoE layer (tests/golden/nvfp4_layer.npz: E=8, H=256, I=256, k=4, one starved expert,
    one all-zero token) through the CUDA path.  End-to-end bound 5e-2: the emulation rounds its dequantised operands
    to bf16 before the requantisation of the silu*mul rows, which moves some e2m1 codes and group scales by a
    whole step (the oracle's stage-by-stage agreement with the fixture is within 1e-2)."""
    from prismyra_b200.kernels import nvfp4

    g = golden("nvfp4_layer")
    k = int(g["k"])
    a1, a2 = float(g["a1_gs"][0]), float(g["a2_gs"][0])
    x = torch.from_numpy(g["x"].view(np.int16)).view(torch.bfloat16).to(DEV)
    logits = torch.from_numpy(g["logits"].view(np.int16)).view(torch.bfloat16).to(DEV)
    g1, g2 = torch.from_numpy(g["g1"]), torch.from_numpy(g["g2"])
    al1 = (1.0 / (g1 * a1)).float().to(DEV)
    al2 = (1.0 / (g2 * a2)).float().to(DEV)
    w1 = torch.from_numpy(g["w1"]).to(DEV)
    w2 = torch.from_numpy(g["w2"]).to(DEV)
    s1 = nvfp4.block_scales(torch.from_numpy(g["s1"])).to(DEV)
    s2 = nvfp4.block_scales(torch.from_numpy(g["s2"])).to(DEV)
    out = ops.forward_nvfp4(x, w1, s1, al1, a1, w2, s2, al2, a2, k, logits=logits)
    torch.cuda.synchronize()
    l2, mx = rel_err(bits(out), g["out"])
    assert l2 < 5e-2 and mx < 5e-2, (l2, mx)
    ref = O.moe_forward_nvfp4(g["x"], g["logits"], g["w1"], g["s1"], g["w2"], g["s2"], bits(al1), bits(al2), a1,
                              a2, k)
    l2, mx = rel_err(bits(out), ref["out"])
    assert l2 < 1e-2 and mx < 2e-2, (l2, mx)
