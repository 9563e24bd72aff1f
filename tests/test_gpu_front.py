"""The one-launch front end of the FP8 forward (512 <= T*k <= 4096): top-k, expert alignment and the quantisation of
the token rows into their slots run as one kernel with a grid barrier.  Its outputs, read back from the forward's
workspace, must equal the oracle's bit for bit -- routing ids, the sorted slots, the block->expert table, the padded
count, the inverse permutation, every slot's FP8 codes and scales -- and the routing weights within 1e-6 relative
(the fp32 softmax sums in another order); the layer output within the layer tolerance of test_gpu_fp8.

Cases: a 256-expert top-16 router (8 logits per lane), tokens per CTA above one (T > the SM count), top-1, a hot
expert spanning several 128-slot blocks, given logits instead of the router, and the headline shapes.
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
    l2 = np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30)
    mx = np.abs(g - r).max() / max(np.abs(r).max(), 1e-30)
    return l2, mx


@pytest.mark.parametrize("T,H,I,E,k,source", [
    (40, 256, 128, 256, 16, "router"),   # T*k = 640, 256 experts: 8 logits per lane
    (300, 256, 128, 128, 8, "logits"),   # three tokens per CTA, hot expert 5 (three blocks)
    (1000, 256, 128, 64, 1, "router"),   # top-1, seven tokens per CTA
    (512, 2048, 768, 128, 8, "router"),  # the headline shapes at the largest T*k of the path
])
def test_front_end_matches_oracle(T, H, I, E, k, source):
    L = synth.make_fp8_layer(T=T, H=H, I=I, E=E, seed=T + E, device="cpu")
    gpu = {n: v.to(DEV) for n, v in L.items()}
    x = gpu["x"]
    if source == "logits":
        g = torch.Generator().manual_seed(T)
        logits = torch.randn(T, E, generator=g) * 0.5
        logits[:, 5] = 6.0  # expert 5 is in every token's top-k
        logits = logits.to(torch.bfloat16)
        out = ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], k, logits=logits.to(DEV))
    else:
        logits, _, _ = ops.router_topk(x, gpu["router_w"], k)
        logits = logits.cpu()
        out = ops.forward_fp8(x, gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], k, router_w=gpu["router_w"])
    ws, _ = ops.workspace_for(x, T, H, I, E, k)
    ops.read_status(ws)
    ms = _lib.max_slots(T, E, k)
    reg = lambda name, dt, shape: ops.region(ws, T, H, I, E, k, 0, name, dt, shape).clone()

    rw, rids = O.route_topk(bits(logits), k)
    ids = bits(reg("topk_ids", torch.int32, (T, k)))
    w = bits(reg("topk_w", torch.float32, (T, k)))
    assert np.array_equal(ids, rids)
    np.testing.assert_allclose(w, rw, rtol=1e-6, atol=0)

    rs, re, rn = O.align(rids, E, 128)
    npp = int(reg("num_post_pad", torch.int32, (1,)).item())
    assert npp == rn
    srt = bits(reg("sorted", torch.int32, (ms,)))
    assert np.array_equal(srt[:npp], rs)
    assert np.array_equal(bits(reg("expert_ids", torch.int32, (ms // 128,)))[: npp // 128], re)
    off = bits(reg("expert_off", torch.int32, (E + 1,)))
    assert off[E] == npp
    slot_of = bits(reg("slot_of", torch.int32, (T * k,)))
    assert np.array_equal(srt[slot_of], np.arange(T * k))

    q, s = O.quant_fp8_groups(bits(L["x"]))
    a1 = bits(reg("a1", torch.uint8, (ms, H)))
    a1s = bits(reg("a1_scale", torch.float32, (ms, H // 128)))
    tok = np.arange(T * k) // k
    assert np.array_equal(a1[slot_of], q[tok])
    assert np.array_equal(a1s[slot_of], s[tok])

    ref = O.moe_forward_fp8(bits(L["x"]), bits(logits), bits(L["w1"]), bits(L["w1_s"]), bits(L["w2"]),
                            bits(L["w2_s"]), k)
    l2, mx = rel_err(bits(out), ref["out"])
    assert l2 < 1e-2 and mx < 1e-2, (l2, mx)


def test_front_end_is_deterministic_over_calls():
    """Two forwards in a row (the grid barrier's counter is cleared by each call) give the same bits."""
    T = 200
    L = synth.make_fp8_layer(T=T, H=256, I=128, E=128, seed=3, device="cpu")
    gpu = {n: v.to(DEV) for n, v in L.items()}
    run = lambda: ops.forward_fp8(gpu["x"], gpu["w1"], gpu["w1_s"], gpu["w2"], gpu["w2_s"], 8,
                                  router_w=gpu["router_w"]).clone()
    a, b = run(), run()
    torch.cuda.synchronize()
    assert torch.equal(a, b)
