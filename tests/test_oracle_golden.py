"""The CPU oracle against the golden fixtures made from the reference's own code (tests/golden/make_golden.py).

No device needed.  These pins are what make the oracle a trustworthy checker for the CUDA kernels:
* alignment: bit-exact against the moe_align_block_size docstring example;
* router: ids bit-exact and weights within 2 fp32 ulps against transformers' Qwen3_5MoeTopKRouter;
* activation FP8 quantisation: codes and scales bit-exact against vLLM's Triton kernel (interpreted);
* silu-and-mul: bit-exact against vLLM's SiluAndMul.forward_native;
* the whole FP8 layer: every intermediate against vLLM's Triton fused_moe_kernel chain -- bf16 results within
  one bf16 ulp (the interpreter's fp32 dot-product order differs from the oracle's exact sum);
* NVFP4: weight codes and scales bit-exact against prismyra.kernels.nvfp4.quantize/prepare_layer, activation
  quantise-dequantise bit-exact against vLLM's Triton emulation kernel.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O


def _ulp_bf16_diff(a_bits, b_bits):
    a = O.bf16_to_f32(a_bits).astype(np.float64)
    b = O.bf16_to_f32(b_bits).astype(np.float64)
    scale = np.maximum(np.abs(b), 1e-30)
    # one bf16 ulp relative to the magnitude is 2^-7 at the bottom of the binade, 2^-8 at the top
    return np.abs(a - b) / scale


def test_align_docstring_example(golden):
    g = golden("align_kat")
    s, e, n = O.align(g["ids"], int(g["num_experts"]), int(g["block_m"]))
    assert np.array_equal(s, g["sorted_ids"])
    assert np.array_equal(e, g["expert_ids"])
    assert n == int(g["num_post_pad"])


def test_align_properties_on_random_ids():
    rng = np.random.default_rng(0)
    for T, k, E, bm in [(1, 1, 4, 128), (7, 2, 8, 16), (513, 8, 128, 128), (64, 8, 128, 128)]:
        ids = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
        s, e, n = O.align(ids, E, bm)
        flat = ids.reshape(-1)
        assert n % bm == 0 and n == len(s) and len(e) == n // bm
        real = s[s < T * k]
        assert sorted(real.tolist()) == list(range(T * k))  # a permutation of every flat index
        for b, ex in enumerate(e):
            blk = s[b * bm:(b + 1) * bm]
            r = blk[blk < T * k]
            assert np.all(flat[r] == ex) and np.all(np.diff(r) > 0)
        assert np.all(np.diff(e) >= 0)


def test_router_matches_transformers(golden):
    """Same experts and weights as transformers' router.  bf16 logits tie often; torch.topk orders tied experts
    arbitrarily, while the oracle (like vLLM's topk_softmax, whose warp argmax lets the lower index win) orders
    them by index.  So the comparison is per selected expert, and at a tie straddling the top-k cut the oracle
    must take the lower index."""
    g = golden("router")
    k = int(g["k"])
    w, ids = O.route_topk(g["logits"], k)
    lg = O.bf16_to_f32(g["logits"])
    cut_ties = 0
    for t in range(lg.shape[0]):
        vals = lg[t][ids[t]]
        assert np.all(np.diff(vals) <= 0)
        for j in range(k - 1):  # equal values come in ascending expert order
            if vals[j] == vals[j + 1]:
                assert ids[t, j] < ids[t, j + 1]
        kth = np.sort(lg[t])[::-1][k - 1]
        if np.sum(lg[t] >= kth) > k:  # a tie straddles the cut
            cut_ties += 1
            tied = np.nonzero(lg[t] == kth)[0]
            need = k - int(np.sum(lg[t] > kth))
            assert set(ids[t][vals == kth]) == set(tied[:need].tolist())
            continue
        assert set(ids[t]) == set(g["ids"][t])
        ref = dict(zip(g["ids"][t].tolist(), g["scores"][t].tolist()))
        np.testing.assert_allclose(w[t], [ref[i] for i in ids[t]], rtol=1e-6, atol=0)
    assert cut_ties == int(g["ties_at_cut"])


def test_router_logits_match_transformers(golden):
    """bf16(F.linear) on CPU accumulates in fp32; the oracle rounds the exact sum once -- at most one bf16
    ulp apart, and on all but a few entries identical."""
    g = golden("router")
    lg = O.router_logits(g["x"], g["weight"])
    d = _ulp_bf16_diff(lg, g["logits"])
    assert np.all(d <= 2.0 ** -7)
    assert np.mean(lg == g["logits"]) > 0.97


def test_router_tie_rule_prefers_lower_expert_index():
    logits = np.zeros((2, 8), np.float32)
    logits[0] = [1, 3, 3, 0, 3, 2, 2, -1]
    logits[1] = 0.5
    w, ids = O.route_topk(O.f32_to_bf16(logits), 4)
    assert ids[0].tolist() == [1, 2, 4, 5]
    assert ids[1].tolist() == [0, 1, 2, 3]
    np.testing.assert_allclose(w[1], 0.25, rtol=1e-7)


def test_act_quant_matches_vllm_triton(golden):
    g = golden("act_quant")
    q, s = O.quant_fp8_groups(g["x"], scale="fp32_rcp")  # the fixture ran vLLM's Triton kernel
    assert np.array_equal(s, g["s"])
    assert np.array_equal(q, g["q"])
    # the library's default rule, the correctly rounded quotient, is at most one ulp away from it
    q2, s2 = O.quant_fp8_groups(g["x"])
    assert np.all(np.abs(s2.view(np.int32) - s.view(np.int32)) <= 1) and np.mean(q2 == q) > 0.99


def test_act_quant_ue8m0_matches_vllm_triton(golden):
    """vLLM's power-of-two scale mode (use_ue8m0, fp8_utils.py:145) on the same edge rows: bit-exact, every scale a
    power of two no smaller than the fp32 scale."""
    g = golden("act_quant")
    q, s = O.quant_fp8_groups(g["x"], scale="ue8m0")
    assert np.array_equal(s, g["s_ue8m0"]) and np.array_equal(q, g["q_ue8m0"])
    m, _ = np.frexp(s)
    assert np.all(m == 0.5) and np.all(s >= g["s"])


@pytest.mark.parametrize("fixture,scale", [("fp8_layer", "fp32_rcp"), ("fp8_layer_ue8m0", "ue8m0")])
def test_fp8_layer_intermediates_match_vllm_triton(golden, fixture, scale):
    g = golden(fixture)
    k = int(g["k"])
    T, H = g["x"].shape
    E = g["w1"].shape[0]
    # routing
    w, ids = O.route_topk(g["logits"], k)
    assert np.array_equal(ids, g["top_i"])
    np.testing.assert_allclose(w, g["top_w"], rtol=3e-7)
    s, e, n = O.align(ids, E, int(g["block_m"]))
    assert np.array_equal(s, g["sorted_ids"]) and np.array_equal(e, g["expert_ids"])
    assert E - 1 not in e.tolist()  # the starved expert owns no block
    # the whole layer with intermediates
    r = O.moe_forward_fp8(g["x"], g["logits"], g["w1"], g["w1_s"], g["w2"], g["w2_s"], k, want_intermediates=True,
                          scale=scale)
    assert np.array_equal(r["x_q"], g["x_q"]) and np.array_equal(r["x_s"], g["x_s"])
    # GEMM1 + silu: c2 is the bf16 activation the Triton chain fed to its requantisation
    c2 = g["c2"].reshape(T * k, -1)
    c2q_ref, c2s_ref = O.quant_fp8_groups(c2, scale=scale)
    assert np.array_equal(c2q_ref, g["c2q"]) and np.array_equal(c2s_ref, g["c2s"])
    assert np.mean(r["c2q"] == g["c2q"]) > 0.99
    np.testing.assert_allclose(r["c2s"], g["c2s"], rtol=2 ** -7)
    # GEMM2 + weight, and the top-k sum
    assert np.all(_ulp_bf16_diff(r["c3"], g["c3"]) <= 2 ** -6)
    assert np.all(_ulp_bf16_diff(r["out"], g["out"]) <= 2 ** -6)
    rel = np.linalg.norm(O.bf16_to_f32(r["out"]) - O.bf16_to_f32(g["out"])) / np.linalg.norm(O.bf16_to_f32(g["out"]))
    assert rel < 1e-3


def test_gemm_rows_matches_vllm_triton_gemm1(golden):
    """The oracle's block-scaled GEMM on the Triton chain's own quantised inputs reproduces c1 within one ulp."""
    g = golden("fp8_layer")
    k = int(g["k"])
    ids = g["top_i"].reshape(-1)
    T = g["x"].shape[0]
    a = np.repeat(g["x_q"], k, axis=0)
    a_s = np.repeat(g["x_s"], k, axis=0)
    out = O.gemm_fp8_rows(a, a_s, ids, g["w1"], g["w1_s"])
    c1 = g["c1"].reshape(T * k, -1)
    assert np.all(_ulp_bf16_diff(O.f32_to_bf16(out), c1) <= 2 ** -7)


def test_silu_mul_matches_vllm_native(golden):
    g = golden("fp8_layer")
    k = int(g["k"])
    T = g["x"].shape[0]
    c1 = g["c1"].reshape(T * k, -1)
    I = c1.shape[1] // 2
    assert np.array_equal(O.silu_mul(c1[:, :I], c1[:, I:]), g["c2"].reshape(T * k, I))


def test_nvfp4_weight_quant_matches_reference(golden):
    g = golden("nvfp4")
    packed, sf = O.nvfp4_quant_weight(g["w"], float(g["gs"]))
    assert np.array_equal(sf, g["scale"])
    assert np.array_equal(packed, g["packed"])


def test_nvfp4_prepare_layer_matches_reference(golden):
    """prepare_layer = FP8-block dequant, per-matrix global scale g = reciprocal(amax) * 2688, then quantize."""
    g = golden("nvfp4")
    wq = g["fp8_w"]
    R, C = wq[0].shape
    d = (O.e4m3_to_f32(wq[0]).reshape(R // 128, 128, C // 128, 128)
         * g["fp8_s"][0].reshape(R // 128, 1, C // 128, 1)).reshape(R, C).astype(np.float32)
    assert np.array_equal(d, g["dequant0"])
    for wk, sk, tag in (("fp8_w", "fp8_s", "1"), ("fp8_w2", "fp8_s2", "2")):
        packed, sf, gs = O.nvfp4_prepare(g[wk], g[sk])
        assert np.array_equal(gs, g["prep_g" + tag])
        assert np.array_equal(sf, g["prep_s" + tag]) and np.array_equal(packed, g["prep_w" + tag])


def test_nvfp4_global_scale_is_reciprocal_times_2688(golden):
    """The reference's `448.0 * 6.0 / t` is t.reciprocal() * 2688 in torch: two fp32 roundings.  The oracle's
    rule reproduces all 4096 fixture maxima; a single true division would not."""
    g = golden("nvfp4_search")
    amax = g["amax"].astype(np.float32)
    two = (np.float32(1.0) / amax).astype(np.float32) * np.float32(2688.0)
    assert np.array_equal(two.astype(np.float32), g["gscale"])
    assert not np.array_equal((np.float32(2688.0) / amax).astype(np.float32), g["gscale"])
    # the same rule inside the oracle's prepare, one single-block matrix per maximum
    E = 64
    w = np.zeros((E, 128, 128), np.uint8)
    w[:, 5, 7] = 0x7E  # e4m3 448
    s = (amax[:E] / np.float32(448.0)).astype(np.float32).reshape(E, 1, 1)
    _, _, gs = O.nvfp4_prepare(w, s)
    d_max = (np.float32(448.0) * s.reshape(E)).astype(np.float32)
    assert np.array_equal(gs, ((np.float32(1.0) / d_max).astype(np.float32) * np.float32(2688.0)).astype(np.float32))


def test_nvfp4_act_quant_matches_vllm_emulation(golden):
    g = golden("nvfp4")
    gs = float(g["act_gs"][0])
    packed, sf = O.nvfp4_quant_act(g["act_x"], gs)
    vals = O.e2m1_unpack(packed).reshape(packed.shape[0], -1, 16)
    deq = (vals * (O.e4m3_to_f32(sf) / np.float32(gs))[..., None]).reshape(packed.shape[0], -1)
    assert np.array_equal(deq.astype(np.float32), g["act_dequant"])


def _nvfp4_layer_case(golden):
    g = golden("nvfp4_layer")
    a1, a2 = float(g["a1_gs"][0]), float(g["a2_gs"][0])
    # alpha = 1/(g_w * a_gs) per expert, fp32 (reference prismyra/kernels/nvfp4.py:141-142)
    al1 = (np.float32(1.0) / (g["g1"] * np.float32(a1)).astype(np.float32)).astype(np.float32)
    al2 = (np.float32(1.0) / (g["g2"] * np.float32(a2)).astype(np.float32)).astype(np.float32)
    return g, a1, a2, al1, al2


def _rel(got_bits, ref_bits):
    a = O.bf16_to_f32(got_bits).astype(np.float64)
    b = O.bf16_to_f32(ref_bits).astype(np.float64)
    return np.linalg.norm(a - b) / np.linalg.norm(b), np.abs(a - b).max() / np.abs(b).max()


def test_nvfp4_layer_stages_match_vllm_emulation(golden):
    """The oracle's NVFP4 layer against vLLM's NVFP4 emulation MoE (nvfp4_emulation_moe.py:83-160) stage by stage:
    the activation quantise-dequantise bit-exact, the gate_up GEMM within 1e-2, the requantisation of the same
    silu*mul rows bit-exact, and the down GEMM times the routing weight on vLLM's own requantised rows within 1e-2.
    The emulation rounds its dequantised operands to bf16 (2^-9 relative), which the FP4 GEMM does not."""
    g, a1, a2, al1, al2 = _nvfp4_layer_case(golden)
    k = int(g["k"])
    T, H = g["x"].shape
    rows = np.repeat(np.arange(T), k)
    re = g["top_i"].reshape(-1)
    w, ids = O.route_topk(g["logits"], k)
    assert np.array_equal(ids, g["top_i"])
    np.testing.assert_allclose(w, g["top_w"], rtol=1e-6)
    xq, xsf = O.nvfp4_quant_act(g["x"], a1)
    assert np.array_equal(O.f32_to_bf16(O.nvfp4_dequant(xq, xsf, a1)), g["x_dq"])
    c1 = O.f32_to_bf16(O.gemm_nvfp4_rows(xq[rows], xsf[rows], re, g["w1"], g["s1"], al1))
    l2, mx = _rel(c1, g["c1"].reshape(T * k, -1))
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)
    c2 = g["c2"].reshape(T * k, -1)
    q2, s2 = O.nvfp4_quant_act(c2, a2)
    assert np.array_equal(O.f32_to_bf16(O.nvfp4_dequant(q2, s2, a2)), g["c2_dq"].reshape(T * k, -1))
    c3 = O.gemm_nvfp4_rows(q2, s2, re, g["w2"], g["s2"], al2) * g["top_w"].reshape(-1)[:, None]
    l2, mx = _rel(O.f32_to_bf16(c3), g["c3"])
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)


def test_nvfp4_layer_end_to_end_matches_vllm_emulation(golden):
    """The whole oracle NVFP4 layer against the emulation's output.  The two chains differ before the requantisation
    of the silu*mul rows only by the emulation's bf16 operand rounding, but that requantisation is discontinuous: a
    1-ulp difference in a row moves about 1% of its e2m1 codes by a whole step and about 3% of its group scales by
    an e4m3 step, so the end-to-end bound is 5e-2 (each stage is within 1e-2, test above)."""
    g, a1, a2, al1, al2 = _nvfp4_layer_case(golden)
    r = O.moe_forward_nvfp4(g["x"], g["logits"], g["w1"], g["s1"], g["w2"], g["s2"], al1, al2, a1, a2, int(g["k"]))
    l2, mx = _rel(r["out"], g["out"])
    assert l2 < 5e-2 and mx < 5e-2, (l2, mx)


@pytest.mark.parametrize("n", [0, 1, 37])
def test_conversions_round_to_nearest_even(n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(4096) * 10 ** rng.uniform(-3, 2.6, 4096)).astype(np.float32)
    x = np.clip(x, -448, 448)
    back = O.e4m3_to_f32(O.f32_to_e4m3(x))
    # the nearest grid value: no other e4m3 value is closer
    grid = np.unique(O.e4m3_to_f32(np.arange(256, dtype=np.uint8)))
    grid = grid[np.isfinite(grid)]
    nearest = grid[np.abs(x[:, None] - grid[None, :]).argmin(1)]
    assert np.all(np.abs(back - x) <= np.abs(nearest - x))
