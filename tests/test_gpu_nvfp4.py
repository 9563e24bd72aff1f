"""Parity of the CUDA NVFP4 routed-expert path with the CPU oracle (all calls through the C ABI).

Tolerances: activation NVFP4 quantisation bit-exact in value (codes compared as decoded values, so a negative
zero equals a positive zero) and in the e4m3 scale bytes; GEMM stages and the layer output relative L2 <= 1e-2
and max <= 1e-2 * max|ref| against the oracle fed the same routing; determinism and row-count invariance bit-exact.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.conftest import cuda_ok

pytestmark = pytest.mark.gpu

if cuda_ok():
    from prismyra_b200 import ops, synth
    from prismyra_b200.kernels import nvfp4

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
    fp8 = synth.make_fp8_layer(T=512, H=H, I=I, E=E, seed=1, device="cpu")
    nv = synth.make_nvfp4_layer(fp8)
    prep, act = nv["prepared"], nv["act"]
    a1 = float(448.0 * 6.0 / (1.25 * act["w13_in_amax"]))
    a2 = float(448.0 * 6.0 / (1.25 * max(act["w2_in_amax"])))
    g = {
        "x": fp8["x"].to(DEV), "router_w": fp8["router_w"].to(DEV),
        "w1": prep["w1"].to(DEV), "w2": prep["w2"].to(DEV),
        "w1_sf": nvfp4.block_scales(prep["s1"]).to(DEV), "w2_sf": nvfp4.block_scales(prep["s2"]).to(DEV),
        "alpha1": (1.0 / (prep["g1"] * a1)).float().to(DEV), "alpha2": (1.0 / (prep["g2"] * a2)).float().to(DEV),
    }
    cpu = {"x": bits(fp8["x"]), "w1": bits(prep["w1"]), "w2": bits(prep["w2"]), "s1": bits(prep["s1"]),
           "s2": bits(prep["s2"]), "alpha1": bits(g["alpha1"]), "alpha2": bits(g["alpha2"])}
    cpu["prep"], cpu["act"], cpu["fp8"] = prep, act, fp8
    return g, cpu, a1, a2


def forward(g, a1, a2, x, **kw):
    return ops.forward_nvfp4(x, g["w1"], g["w1_sf"], g["alpha1"], a1, g["w2"], g["w2_sf"], g["alpha2"], a2, K, **kw)


@pytest.mark.parametrize("T", [1, 37, 512])
def test_quant_nvfp4_matches_oracle(layer, T):
    g, cpu, a1, _ = layer
    q, sf = ops.quant_nvfp4(g["x"][:T].contiguous(), a1)
    rq, rsf = O.nvfp4_quant_act(cpu["x"][:T], a1)
    rb = -(-T // 128)
    got_sf = nvfp4.unblock_scales(sf.cpu(), rb * 128, H // 16).numpy()[:T]
    assert np.array_equal(got_sf, rsf)
    assert np.array_equal(O.e2m1_unpack(bits(q)), O.e2m1_unpack(rq))


def test_gemm_stages_match_oracle(layer):
    g, cpu, a1, a2 = layer
    T = 512
    x = g["x"]
    _, w, ids = ops.router_topk(x, g["router_w"], K)
    s, eids, npp, _, slot_of, _ = ops.align(ids, E)
    ms = s.numel()
    a_q, a_sf = ops.quant_nvfp4(x, a1, slot_of, K, ms)
    o_q, o_sf, err = ops.gemm1_nvfp4(a_q, a_sf, g["w1"], g["w1_sf"], g["alpha1"], a2, eids, npp)
    c3, err2 = ops.gemm2_nvfp4(o_q, o_sf, g["w2"], g["w2_sf"], g["alpha2"], eids, npp, s, w.reshape(-1), T, K)
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and int(err2.item()) == 0
    n = int(npp.item())
    sv = bits(s)[:n]
    real = np.nonzero(sv < T * K)[0]
    rows = real[:: max(1, len(real) // 500)]
    row_e = bits(eids)[rows // 128]
    # gate_up: the oracle's product on the kernel's own quantised inputs
    a_sf_rows = nvfp4.unblock_scales(a_sf.cpu(), ms, H // 16).numpy()[rows]
    c1 = O.gemm_nvfp4_rows(bits(a_q)[rows], a_sf_rows, row_e, cpu["w1"], cpu["s1"], cpu["alpha1"])
    c1b = O.f32_to_bf16(c1)
    c2 = O.silu_mul(c1b[:, :I], c1b[:, I:])
    rq, rsf = O.nvfp4_quant_act(c2, a2)
    got_sf = nvfp4.unblock_scales(o_sf.cpu(), ms, I // 16).numpy()[rows]
    deq_g = O.nvfp4_dequant(bits(o_q)[rows], got_sf, a2)
    deq_r = O.nvfp4_dequant(rq, rsf, a2)
    assert np.linalg.norm(deq_g - deq_r) / np.linalg.norm(deq_r) < 2e-2
    assert np.mean(got_sf == rsf) > 0.97
    # down: the oracle's product on the kernel's own intermediate
    o = O.gemm_nvfp4_rows(bits(o_q)[rows], got_sf, row_e, cpu["w2"], cpu["s2"], cpu["alpha2"])
    flat = sv[rows]
    ref = O.f32_to_bf16(o * bits(w).reshape(-1)[flat][:, None])
    l2, mx = rel_err(bits(c3)[flat], ref)
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)


@pytest.mark.parametrize("T", [1, 5, 128, 512])
def test_forward_nvfp4_matches_oracle(layer, T):
    g, cpu, a1, a2 = layer
    x = g["x"][:T].contiguous()
    logits, _, _ = ops.router_topk(x, g["router_w"], K)
    out = forward(g, a1, a2, x, router_w=g["router_w"])
    ws, _ = ops.workspace_for(x, T, H, I, E, K, 1)
    ops.read_status(ws)
    ref = O.moe_forward_nvfp4(cpu["x"][:T], bits(logits), cpu["w1"], cpu["s1"], cpu["w2"], cpu["s2"],
                              cpu["alpha1"], cpu["alpha2"], a1, a2, K)
    l2, mx = rel_err(bits(out), ref["out"])
    assert l2 < 1e-2 and mx < 2e-2, (l2, mx)


def test_forward_nvfp4_deterministic_and_row_invariant(layer):
    g, _, a1, a2 = layer
    x = g["x"]
    a = forward(g, a1, a2, x, router_w=g["router_w"]).clone()
    b = forward(g, a1, a2, x, router_w=g["router_w"]).clone()
    assert torch.equal(a, b)
    part = forward(g, a1, a2, x[300:333].contiguous(), router_w=g["router_w"])
    assert torch.equal(part, a[300:333])


def test_nvfp4_module_matches_routed_plus_shared(layer):
    g, cpu, a1, a2 = layer

    class Block(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.gate = torch.nn.Linear(H, E, bias=False).to(DEV, torch.bfloat16)
            self.gate.weight.data.copy_(g["router_w"])
            self.shared_expert = torch.nn.Linear(H, H, bias=False).to(DEV, torch.bfloat16)
            self.shared_expert_gate = torch.nn.Linear(H, 1, bias=False).to(DEV, torch.bfloat16)

    blk = Block()
    mod = nvfp4.FusedExpertsFp4(blk, K, cpu["prep"], cpu["act"], DEV)
    assert mod.a1_gscale == a1 and mod.a2_gscale == a2
    assert torch.equal(mod.w1_scale, g["w1_sf"]) and torch.equal(mod.g1_alphas, g["alpha1"])
    x = g["x"][:64].reshape(2, 32, H)
    y = mod(x)
    xf = x.reshape(-1, H)
    routed = forward(g, a1, a2, xf.contiguous(), router_w=g["router_w"])
    shared = torch.sigmoid(torch.nn.functional.linear(xf, blk.shared_expert_gate.weight)) * blk.shared_expert(xf)
    assert torch.equal(y.reshape(-1, H), routed + shared)


def test_prepare_on_gpu_matches_cpu_prepare_and_oracle(layer):
    """pm_nvfp4_prepare on the full stacks (E=128; w13 1536 x 2048, w2 2048 x 768): bit-identical to the torch
    prepare_layer on the CPU (the reference's arithmetic), and on four experts to the C oracle."""
    _, cpu, _, _ = layer
    fp8, prep = cpu["fp8"], cpu["prep"]
    got = nvfp4.prepare_layer(fp8["w1"], fp8["w1_s"], fp8["w2"], fp8["w2_s"], DEV)
    for key in ("w1", "s1", "g1", "w2", "s2", "g2"):
        assert got[key].dtype == prep[key].dtype and got[key].shape == prep[key].shape, key
        assert np.array_equal(bits(got[key]), bits(prep[key])), key
    for wk, sk, tag in (("w1", "w1_s", "1"), ("w2", "w2_s", "2")):
        packed, sf, gs = O.nvfp4_prepare(bits(fp8[wk][:4]), fp8[sk][:4].float().numpy())
        assert np.array_equal(packed, bits(got["w" + tag][:4]))
        assert np.array_equal(sf, bits(got["s" + tag][:4]))
        assert np.array_equal(gs, bits(got["g" + tag][:4]))


def test_prepare_on_gpu_matches_reference_fixture(golden):
    """The reference's own prepare_layer outputs (tests/golden/nvfp4.npz) from the same FP8 stacks."""
    g = golden("nvfp4")
    for wk, sk, tag in (("fp8_w", "fp8_s", "1"), ("fp8_w2", "fp8_s2", "2")):
        w = torch.from_numpy(g[wk]).to(DEV)
        s = torch.from_numpy(g[sk]).to(DEV)
        packed, sf, gs = ops.nvfp4_prepare(w, s)
        assert np.array_equal(bits(packed), g["prep_w" + tag])
        assert np.array_equal(bits(sf), g["prep_s" + tag])
        assert np.array_equal(bits(gs), g["prep_g" + tag])


@pytest.mark.parametrize("stack", ["w1", "w2"])
def test_prepare_search_on_gpu_matches_torch_restatement(layer, stack):
    """The search kernel on two experts of each layer stack with spread-out importance weights (and, for the
    second, a weight of 1 everywhere) against the torch restatement (_prepare_stack, the reference's
    quantize_search arithmetic) on the CPU, where the reference's outputs were made: bit-exact.  Also the search
    without importance against the restatement with a weight of 1."""
    _, cpu, _, _ = layer
    fp8 = cpu["fp8"]
    w, s = fp8[stack][:2].contiguous(), fp8[stack + "_s"][:2].float().contiguous()
    C = w.shape[2]
    gen = torch.Generator(device="cpu").manual_seed(11)
    imp = torch.exp(torch.randn(2, C, generator=gen) * 2.0).float()
    imp[1] = 1.0
    packed, sf, gs = ops.nvfp4_prepare(w.to(DEV).view(torch.uint8), s.to(DEV), importance=imp.to(DEV))
    rp, rs, rg = nvfp4._prepare_stack(w, s, "cpu", imp)
    assert np.array_equal(bits(packed), bits(rp)) and np.array_equal(bits(sf), bits(rs))
    assert np.array_equal(bits(gs), bits(rg))
    p1, s1, _ = ops.nvfp4_prepare(w.to(DEV).view(torch.uint8), s.to(DEV), search=True)
    rp1, rs1, _ = nvfp4._prepare_stack(w, s, "cpu", torch.ones(2, C))
    assert np.array_equal(bits(p1), bits(rp1)) and np.array_equal(bits(s1), bits(rs1))


def test_prepare_search_on_gpu_matches_reference_fixture(golden):
    """pm_nvfp4_prepare_search through prepare_layer(imp_in=..., imp_mid=..., tok=...) on the GPU against the
    reference's own prepare_layer outputs with importance weights (tests/golden/nvfp4_search.npz; one expert there
    saw no tokens and is searched with weight 1): codes, scale bytes and global scales bit-exact."""
    g = golden("nvfp4_search")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    got = nvfp4.prepare_layer(t(g["fp8_w"]).view(torch.float8_e4m3fn), t(g["fp8_s"]),
                              t(g["fp8_w2"]).view(torch.float8_e4m3fn), t(g["fp8_s2"]), DEV,
                              imp_in=t(g["imp_in"]), imp_mid=t(g["imp_mid"]), tok=t(g["tok"]))
    for k in ("w1", "s1", "g1", "w2", "s2", "g2"):
        assert np.array_equal(bits(got[k]), g["prep_" + k]), k
