"""Parity of the CUDA FP8 routed-expert path with the CPU oracle, stage by stage and end to end.

Every call goes through the C ABI (``libprismyra_moe.so`` via ``prismyra_b200.ops``).  Tolerances:
* routing ids, the expert alignment (sorted slots, block->expert table, padded count) and the activation FP8
  codes/scales: bit-exact;
* routing weights: 1e-6 relative (fp32 softmax; only the order of the exponent sum differs);
* router logits: at most one bf16 ulp from the exactly-rounded sum (fp32 accumulation);
* GEMM outputs and the layer output: relative L2 error <= 1e-2 and max error <= 1e-2 * max|ref| against the
  oracle fed the same routing (the BASELINE north-star tolerance for bf16 output with fp32 accumulation);
* determinism and row-count invariance: bit-exact.
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


def from_bits_bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def rel_err(got_bits, ref_bits):
    g = O.bf16_to_f32(got_bits).astype(np.float64)
    r = O.bf16_to_f32(ref_bits).astype(np.float64)
    l2 = np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30)
    mx = np.abs(g - r).max() / max(np.abs(r).max(), 1e-30)
    return l2, mx


@pytest.fixture(scope="module")
def layer():
    torch.manual_seed(0)
    L = synth.make_fp8_layer(T=512, H=H, I=I, E=E, seed=0, device="cpu")
    gpu = {k: v.to(DEV) for k, v in L.items()}
    return L, gpu


# ------------------------------------------------------------------------------------------- routing
@pytest.mark.parametrize("T", [1, 7, 128, 5120])
def test_topk_from_logits_matches_oracle(T):
    g = torch.Generator().manual_seed(T)
    logits = (torch.randn(T, E, generator=g) * 1.5).to(torch.bfloat16)
    if T >= 7:  # exact ties inside and across the top-k boundary
        logits[3, :] = 0.5
        logits[5, 10:20] = 3.0
    w, ids = ops.topk(logits.to(DEV), K)
    rw, rids = O.route_topk(bits(logits), K)
    assert np.array_equal(bits(ids), rids)
    np.testing.assert_allclose(bits(w), rw, rtol=1e-6, atol=0)


@pytest.mark.parametrize("E_, k_", [(8, 4), (64, 6), (256, 16), (128, 1)])
def test_topk_other_shapes(E_, k_):
    g = torch.Generator().manual_seed(E_ * 100 + k_)
    logits = torch.randn(300, E_, generator=g).to(torch.bfloat16)
    w, ids = ops.topk(logits.to(DEV), k_)
    rw, rids = O.route_topk(bits(logits), k_)
    assert np.array_equal(bits(ids), rids)
    np.testing.assert_allclose(bits(w), rw, rtol=1e-6, atol=0)


def test_router_logits_and_topk(layer):
    """Logits within one bf16 ulp of the exact product sum plus the fp32 accumulation error (2^-20 of the sum of
    magnitudes, which matters only where the sum cancels to near zero)."""
    L, gpu = layer
    logits, w, ids = ops.router_topk(gpu["x"], gpu["router_w"], K)
    xf = O.bf16_to_f32(bits(L["x"])).astype(np.float64)
    wf = O.bf16_to_f32(bits(L["router_w"])).astype(np.float64)
    exact = xf @ wf.T
    mag = np.abs(xf) @ np.abs(wf).T
    got = O.bf16_to_f32(bits(logits)).astype(np.float64)
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(exact), 1e-30))) - 7)
    assert np.all(np.abs(got - exact) <= ulp + mag * 2.0 ** -20)
    ref = O.router_logits(bits(L["x"]), bits(L["router_w"]))
    assert np.mean(bits(logits) == ref) > 0.97
    rw, rids = O.route_topk(bits(logits), K)  # ranking of the kernel's own logits is bit-exact
    assert np.array_equal(bits(ids), rids)
    np.testing.assert_allclose(bits(w), rw, rtol=1e-6)


@pytest.mark.parametrize("T", [1, 37, 512, 2048, 2049])
def test_router_split_and_fused_shapes_agree(layer, T):
    """The layer forward runs the split router shape for small T (fp32 chunk partials summed by the top-k kernel),
    the stage entry point the fused one; both must give the same logits and routing bit for bit."""
    _, gpu = layer
    x = gpu["x"][torch.arange(T, device=DEV) % 512].contiguous()
    fused, w, ids = ops.router_topk(x, gpu["router_w"], K)
    ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, router_w=gpu["router_w"])
    ws, _ = ops.workspace_for(x, T, H, I, E, K)
    torch.cuda.synchronize()
    split = _lib.workspace_region(T, H, I, E, K, 0, "router_part")[1] > 0
    assert split == (T <= 2048)  # 16 x 4 fused CTAs at most for the split shape
    region = lambda name: _lib.workspace_region(T, H, I, E, K, 0, name)
    off, n = region("logits")
    assert torch.equal(ws[off:off + n].view(torch.bfloat16).view(T, E), fused)
    off, n = region("topk_ids")
    assert torch.equal(ws[off:off + n].view(torch.int32).view(T, K), ids)
    off, n = region("topk_w")
    assert torch.equal(ws[off:off + n].view(torch.float32).view(T, K), w)


def test_router_is_row_count_invariant(layer):
    _, gpu = layer
    full, _, _ = ops.router_topk(gpu["x"], gpu["router_w"], K)
    part, _, _ = ops.router_topk(gpu["x"][100:133].contiguous(), gpu["router_w"], K)
    assert torch.equal(full[100:133], part)


@pytest.mark.parametrize("T,E_,k_", [(1, 128, 8), (7, 8, 4), (128, 128, 8), (513, 128, 8), (5120, 128, 8),
                                     (40000 // 8, 128, 8), (1000, 256, 16), (300, 1024, 16), (1 << 17, 128, 8)])
def test_align_matches_oracle(T, E_, k_):
    # (1 << 17) x 8 = 2^20 indices: the largest chunks (4096) and the most chunks (256); E = 1024: four experts
    # per thread in the scan
    g = torch.Generator().manual_seed(T + E_)
    ids = torch.rand(T, E_, generator=g).argsort(dim=1)[:, :k_].contiguous().to(torch.int32)
    if T >= 7:
        ids[:, 0] = 0  # a hot expert
    s, eids, npp, off, slot_of, _ = ops.align(ids.to(DEV), E_)
    rs, re, rn = O.align(bits(ids), E_, 128)
    n = int(npp.item())
    assert n == rn
    assert np.array_equal(bits(s)[:n], rs)
    assert np.array_equal(bits(eids)[: n // 128], re)
    offs = bits(off)
    assert offs[E_] == n
    inv = bits(slot_of)  # the inverse permutation: slot_of[flat] = slot
    assert np.array_equal(bits(s)[inv], np.arange(T * k_))
    for e in range(E_):
        blk = re == e
        if blk.any():
            assert offs[e] == np.argmax(blk) * 128


@pytest.mark.parametrize("shift", [1, 2, 3])
def test_align_into_outputs_that_are_not_16_byte_aligned(shift):
    """The C ABI takes plain int32 pointers: the vectorised padding writes must respect any 4-byte alignment."""
    T, E_, k_ = 300, 64, 4
    g = torch.Generator().manual_seed(shift)
    ids = torch.rand(T, E_, generator=g).argsort(dim=1)[:, :k_].contiguous().to(torch.int32).to(DEV)
    ms = _lib.max_slots(T, E_, k_)
    big = torch.full((ms + 8,), -7, dtype=torch.int32, device=DEV)
    sorted_ids = big[shift:shift + ms]
    eids = torch.full((ms // 128,), -1, dtype=torch.int32, device=DEV)
    npp = torch.zeros(1, dtype=torch.int32, device=DEV)
    scratch = torch.zeros(_lib.align_workspace_bytes(T, k_, E_) // 4, dtype=torch.int32, device=DEV)
    P = lambda t: t.data_ptr()
    _lib.call("pm_moe_align", P(ids), T, k_, E_, P(sorted_ids), P(eids), P(npp), None, None, P(scratch),
              scratch.numel() * 4, torch.cuda.current_stream().cuda_stream)
    rs, re, rn = O.align(bits(ids), E_, 128)
    n = int(npp.item())
    assert n == rn and np.array_equal(bits(sorted_ids)[:n], rs) and np.array_equal(bits(eids)[: n // 128], re)
    assert (bits(big)[:shift] == -7).all() and (bits(big)[shift + n:] == -7).all()  # nothing outside the range


def test_align_docstring_example(golden):
    kat = golden("align_kat")
    s, eids, npp, _, _, _ = ops.align(torch.from_numpy(kat["ids"]).to(DEV), int(kat["num_experts"]))
    # block 128 instead of the docstring's 4: same grouping and order, wider padding
    rs, re, rn = O.align(kat["ids"], int(kat["num_experts"]), 128)
    n = int(npp.item())
    assert n == rn == 4 * 128
    assert np.array_equal(bits(s)[:n], rs)
    assert bits(s)[:3].tolist() == [3, 6, 9] and bits(s)[128:131].tolist() == [0, 4, 10]
    assert np.array_equal(bits(eids)[:4], [1, 2, 3, 4])


def test_quant_matches_oracle(layer):
    L, gpu = layer
    x_q, x_s = ops.quant_fp8(gpu["x"])
    xq, xs = O.quant_fp8_groups(bits(L["x"]))
    assert np.array_equal(bits(x_q), xq)
    assert np.array_equal(bits(x_s), xs)


def test_quant_edge_rows_match_vllm_golden(golden):
    g = golden("act_quant")
    x_q, x_s = ops.quant_fp8(from_bits_bf16(g["x"]).to(DEV), act_scale="fp32_rcp")  # vLLM's Triton rule
    assert np.array_equal(bits(x_q), g["q"])
    assert np.array_equal(bits(x_s), g["s"])


# ------------------------------------------------------------------------------------------- GEMMs
def test_gemm1_matches_oracle(layer):
    L, gpu = layer
    T = 512
    _, w, ids = ops.router_topk(gpu["x"], gpu["router_w"], K)
    s, eids, npp, _, slot_of, _ = ops.align(ids, E)
    a_q, a_s = ops.quant_fp8(gpu["x"], slot_of, K, s.numel())
    out_q, out_s, err = ops.gemm1_fp8(a_q, a_s, gpu["w1"], gpu["w1_s"], eids, npp)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    n = int(npp.item())
    sv = bits(s)[:n]
    real = np.nonzero(sv < T * K)[0]
    rows = real[:: max(1, len(real) // 600)]  # a spread sample of slots across experts
    row_e = bits(eids)[rows // 128]
    xq, xs = O.quant_fp8_groups(bits(L["x"]))
    tok = sv[rows] // K
    assert np.array_equal(bits(a_q)[rows], xq[tok]) and np.array_equal(bits(a_s)[rows], xs[tok])
    c1 = O.gemm_fp8_rows(bits(a_q)[rows], bits(a_s)[rows], row_e, bits(L["w1"]), bits(L["w1_s"]))
    c1b = O.f32_to_bf16(c1)
    c2 = O.silu_mul(c1b[:, :I], c1b[:, I:])
    rq, rsc = O.quant_fp8_groups(c2)
    got_q, got_s = bits(out_q)[rows], bits(out_s)[rows]
    np.testing.assert_allclose(got_s, rsc, rtol=1e-2)
    deq_g = O.e4m3_to_f32(got_q).reshape(len(rows), -1, 128) * got_s[:, :, None]
    deq_r = O.e4m3_to_f32(rq).reshape(len(rows), -1, 128) * rsc[:, :, None]
    assert np.linalg.norm(deq_g - deq_r) / np.linalg.norm(deq_r) < 1e-2
    assert np.mean(got_q == rq) > 0.95


def test_gemm2_matches_oracle(layer):
    L, gpu = layer
    T = 512
    _, w, ids = ops.router_topk(gpu["x"], gpu["router_w"], K)
    s, eids, npp, _, slot_of, _ = ops.align(ids, E)
    a_q, a_s = ops.quant_fp8(gpu["x"], slot_of, K, s.numel())
    out_q, out_s, _ = ops.gemm1_fp8(a_q, a_s, gpu["w1"], gpu["w1_s"], eids, npp)
    c3, err = ops.gemm2_fp8(out_q, out_s, gpu["w2"], gpu["w2_s"], eids, npp, s, w.reshape(-1), T, K)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    n = int(npp.item())
    sv = bits(s)[:n]
    real = np.nonzero(sv < T * K)[0]
    rows = real[:: max(1, len(real) // 600)]
    row_e = bits(eids)[rows // 128]
    c = O.gemm_fp8_rows(bits(out_q)[rows], bits(out_s)[rows], row_e, bits(L["w2"]), bits(L["w2_s"]))
    flat = sv[rows]
    ref = O.f32_to_bf16(c * bits(w).reshape(-1)[flat][:, None])
    l2, mx = rel_err(bits(c3)[flat], ref)
    assert l2 < 1e-2 and mx < 1e-2


# ------------------------------------------------------------------------------------------- the layer
@pytest.mark.parametrize("T", [1, 5, 128, 512])
def test_forward_matches_oracle(layer, T):
    L, gpu = layer
    x = gpu["x"][:T].contiguous()
    logits, _, _ = ops.router_topk(x, gpu["router_w"], K)
    out = ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, router_w=gpu["router_w"])
    ws, _ = ops.workspace_for(x, T, H, I, E, K)
    ops.read_status(ws)
    ref = O.moe_forward_fp8(bits(L["x"][:T]), bits(logits), bits(L["w1"]), bits(L["w1_s"]), bits(L["w2"]),
                            bits(L["w2_s"]), K)
    l2, mx = rel_err(bits(out), ref["out"])
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)


def test_small_token_gate_up_equals_the_large_tile_kernel(layer):
    """At T*k <= 32 E the layer runs the swap-AB GEMMs (weights as the 128-row MMA operand).  Their gate_up output
    must equal the large-tile kernel's on the same expert-ordered inputs: the same products and K-block
    promotion, with the MMA operands exchanged."""
    _, gpu = layer
    T = 512
    x = gpu["x"][:T].contiguous()
    ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, router_w=gpu["router_w"])
    ws, _ = ops.workspace_for(x, T, H, I, E, K)
    ms = _lib.max_slots(T, E, K)
    reg = lambda name, dt, shape: ops.region(ws, T, H, I, E, K, 0, name, dt, shape).clone()
    a1, a1s = reg("a1", torch.uint8, (ms, H)), reg("a1_scale", torch.float32, (ms, H // 128))
    a2, a2s = reg("a2", torch.uint8, (ms, I)), reg("a2_scale", torch.float32, (ms, I // 128))
    eids, npp = reg("expert_ids", torch.int32, (ms // 128,)), reg("num_post_pad", torch.int32, (1,))
    srt = reg("sorted", torch.int32, (ms,))
    big_q, big_s, err = ops.gemm1_fp8(a1, a1s, gpu["w1"], gpu["w1_s"], eids, npp)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # the filled slots below num_post_pad (padding slots, and slots past the last block, hold unspecified values --
    # the latter whatever an earlier, larger call left in the workspace)
    in_use = torch.arange(ms, device=srt.device) < int(npp.item())
    real = ((srt < T * K) & in_use).nonzero().squeeze(1)
    assert torch.equal(a2[real], big_q[real]) and torch.equal(a2s[real], big_s[real])


def test_small_token_path_with_one_expert_taking_every_token(layer):
    """Skewed routing at small T: one expert gets all 300 tokens (three 128-slot blocks, up to four 32-slot
    sub-blocks per unit) while the rest share the other slots."""
    L, gpu = layer
    T = 300
    x = gpu["x"][:T].contiguous()
    g = torch.Generator().manual_seed(7)
    logits = (torch.randn(T, E, generator=g) * 0.5)
    logits[:, 5] = 6.0  # expert 5 is in every token's top-k
    logits = logits.to(torch.bfloat16)
    out = ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, logits=logits.to(DEV))
    ws, _ = ops.workspace_for(x, T, H, I, E, K)
    ops.read_status(ws)
    ref = O.moe_forward_fp8(bits(L["x"][:T]), bits(logits), bits(L["w1"]), bits(L["w1_s"]), bits(L["w2"]),
                            bits(L["w2_s"]), K)
    l2, mx = rel_err(bits(out), ref["out"])
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)


@pytest.mark.parametrize("T,edge", [(512, 100), (300, 64), (5120, 512), (4096, 1000)])
def test_host_pipelined_forward_equals_the_device_forward(layer, T, edge):
    """Rows copied in, computed and copied out in chunks on three streams: the same bits as one device call (at
    T=5120 the 512-row edge chunks take the few-tokens GEMMs and the middle the large-tile ones)."""
    _, gpu = layer
    x = gpu["x"][torch.arange(T, device=DEV) % 512].contiguous()
    ref = ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, router_w=gpu["router_w"]).cpu()
    x_host = x.cpu().pin_memory()
    assert len(ops.host_chunks(T, edge)) == 3
    out = ops.forward_fp8_host(x_host, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, gpu["router_w"],
                               edge_rows=edge)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_host_calls_overlapping_each_other_equal_device_forwards(layer):
    """Consecutive asynchronous host-to-host calls (each upload overlapping the previous call's layer and
    download, two alternating device buffer sets) with different inputs: every result equals its own device
    forward bit for bit, also when a later call grows the buffers."""
    _, gpu = layer
    args = (gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, gpu["router_w"])
    cases = []
    for i, T in enumerate((512, 512, 300, 512, 700, 512)):
        x = gpu["x"][(torch.arange(T, device=DEV) * (i + 3)) % 512].contiguous()
        cases.append((x.cpu().pin_memory(), ops.forward_fp8(x, *args[:5], router_w=gpu["router_w"]).cpu()))
    torch.cuda.synchronize()
    outs = [ops.forward_fp8_host_async(xh, *args, out_host=torch.empty_like(xh).pin_memory()) for xh, _ in cases]
    for out_host, done in outs:
        done.synchronize()
    for (out_host, _), (_, ref) in zip(outs, cases):
        assert torch.equal(out_host, ref)


def test_host_async_around_a_function_with_its_own_output(layer):
    """ops.host_async around a device function that returns a tensor of its own (as the expert-parallel layer does)
    rather than filling the given rows: consecutive overlapping calls still return each batch's own result."""
    _, gpu = layer

    def fn(xs, _rows):
        return ops.forward_fp8(xs, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, router_w=gpu["router_w"])

    cases = []
    for i in range(4):
        x = gpu["x"][(torch.arange(400, device=DEV) * (i + 5)) % 512].contiguous()
        cases.append((x.cpu().pin_memory(), fn(x, None).cpu()))
    torch.cuda.synchronize()
    outs = [ops.host_async(fn, xh, torch.empty_like(xh).pin_memory(), device=torch.device(DEV)) for xh, _ in cases]
    for out_host, done in outs:
        done.synchronize()
    for (out_host, _), (_, ref) in zip(outs, cases):
        assert torch.equal(out_host, ref)


def test_forward_with_given_logits_equals_in_kernel_router(layer):
    _, gpu = layer
    x = gpu["x"][:256].contiguous()
    logits, _, _ = ops.router_topk(x, gpu["router_w"], K)
    a = ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, router_w=gpu["router_w"])
    b = ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, logits=logits)
    assert torch.equal(a, b)


def test_forward_is_deterministic_and_row_count_invariant(layer):
    _, gpu = layer
    x = gpu["x"]
    a = ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, router_w=gpu["router_w"]).clone()
    b = ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, router_w=gpu["router_w"]).clone()
    assert torch.equal(a, b)
    part = ops.forward_fp8(x[200:231].contiguous(), gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K,
                           router_w=gpu["router_w"])
    assert torch.equal(part, a[200:231])
    # right padding with other rows does not change the real rows
    padded = torch.cat([x[:40], torch.zeros(24, H, dtype=x.dtype, device=x.device)])
    p = ops.forward_fp8(padded, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K, router_w=gpu["router_w"])
    assert torch.equal(p[:40], a[:40])


def test_golden_fp8_layer_through_gpu(golden):
    """The vLLM-Triton golden layer (E=8, H=256, I=128, k=4, one starved expert) through the CUDA path."""
    g = golden("fp8_layer")
    k = int(g["k"])
    x = from_bits_bf16(g["x"]).to(DEV)
    logits = from_bits_bf16(g["logits"]).to(DEV)
    w1 = torch.from_numpy(g["w1"]).view(torch.float8_e4m3fn).to(DEV)
    w2 = torch.from_numpy(g["w2"]).view(torch.float8_e4m3fn).to(DEV)
    w1_s = torch.from_numpy(g["w1_s"]).to(DEV)
    w2_s = torch.from_numpy(g["w2_s"]).to(DEV)
    out = ops.forward_fp8(x, w1, w1_s, w2, w2_s, k, logits=logits, act_scale="fp32_rcp")  # the fixture's rule
    l2, mx = rel_err(bits(out), g["out"])
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)
    w, ids = ops.topk(logits, k)
    assert np.array_equal(bits(ids), g["top_i"])


def test_forward_rejects_bad_shapes(layer):
    _, gpu = layer
    with pytest.raises(ValueError):
        ops.forward_fp8(gpu["x"][:, :1000], gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], K,
                        router_w=gpu["router_w"])
    with pytest.raises(_lib.MoEKernelError):
        ops.topk(torch.zeros(4, 300, dtype=torch.bfloat16, device=DEV), 8)  # E > 256
