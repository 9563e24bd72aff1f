"""The layer inside a CUDA graph, as the reference's recordings call it (prismyra/onepass.py:183-206): the forward
and the whole block (its shared expert forks onto a side stream and joins back) are captured once after a warm-up
call and replayed; replays equal eager calls bit for bit, also after new inputs are copied into the captured
input buffer.  The kernels are launched with programmatic stream serialisation, which capture records as
programmatic edges."""

from __future__ import annotations

import pytest
import torch

from tests.conftest import cuda_ok

pytestmark = pytest.mark.gpu

if cuda_ok():
    from prismyra_b200 import ops, synth

DEV = "cuda:0"
H, I, E, K, IS = 2048, 768, 128, 8, 512


@pytest.fixture(scope="module")
def layer():
    L = synth.make_fp8_layer(T=1200, H=H, I=I, E=E, seed=21, device=DEV, gen_device="cuda")
    g = torch.Generator("cuda").manual_seed(5)
    L["sw13"], L["sw13_s"] = synth.quantize_fp8_blocks(torch.randn(2 * IS, H, generator=g, device=DEV) * 0.02)
    L["sw2"], L["sw2_s"] = synth.quantize_fp8_blocks(torch.randn(H, IS, generator=g, device=DEV) * 0.02)
    L["w_sg"] = (torch.randn(H, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    L["x2"] = torch.randn(1200, H, generator=g, device=DEV).to(torch.bfloat16)
    return L


def _forward(L, x):
    return ops.forward_fp8(x, L["w1"], L["w1_s"], L["w2"], L["w2_s"], K, router_w=L["router_w"])


def _block(L, x):
    return ops.block_fp8(x, L["w1"], L["w1_s"], L["w2"], L["w2_s"], K, L["w_sg"], L["sw13"], L["sw13_s"], L["sw2"],
                         L["sw2_s"], router_w=L["router_w"])


def _capture(fn, x):
    """Warm up on the capture stream's thread (workspace, tensor maps, side stream), then capture fn(x)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn(x)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = fn(x)
    return graph, out


@pytest.mark.parametrize("T", [300, 1200])  # the few-tokens and the large-tile GEMM shapes
@pytest.mark.parametrize("which", ["forward", "block"])
def test_captured_layer_replays_like_eager_calls(layer, T, which):
    fn = (lambda x: _forward(layer, x)) if which == "forward" else (lambda x: _block(layer, x))
    x = layer["x"][:T].clone()
    eager1 = fn(x).clone()
    eager2 = fn(layer["x2"][:T].contiguous()).clone()
    graph, out = _capture(fn, x)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager1)
    x.copy_(layer["x2"][:T])
    graph.replay()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager2)
    del graph


def test_two_lanes_on_two_threads_match_sequential_calls(layer):
    """Two threads, each on its own stream, call the forward and the block concurrently (the reference's two
    lanes, prismyra/kernels/qwen3_moe.py:277-279): every result equals the sequential call bit for bit (workspace
    and side stream are per thread)."""
    import threading

    xs = [layer["x"][:700].contiguous(), layer["x2"][:900].contiguous()]
    want = [(_forward(layer, x).clone(), _block(layer, x).clone()) for x in xs]
    torch.cuda.synchronize()
    got = [None, None]
    errors = []

    def lane(i):
        try:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                outs = []
                for _ in range(3):
                    outs.append((_forward(layer, xs[i]), _block(layer, xs[i])))
                s.synchronize()
            got[i] = outs
        except Exception as e:  # pragma: no cover - reported below
            errors.append(e)

    threads = [threading.Thread(target=lane, args=(i,)) for i in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not errors, errors
    for i in range(2):
        for f, b in got[i]:
            assert torch.equal(f, want[i][0]) and torch.equal(b, want[i][1]), i
