"""Bounded device-side waits made to run out on purpose, without faulting the GPU: the expert-parallel barrier is
given a target no arrival can reach and a 50 ms limit.  It must give up, set its error word and return, and the
stream must stay usable (the next barrier and a layer forward on it succeed)."""

from __future__ import annotations

import time

import pytest
import torch

from tests.conftest import cuda_ok

pytestmark = pytest.mark.gpu

if cuda_ok():
    from prismyra_b200 import _lib, ops, synth

DEV = "cuda:0"


def test_barrier_wait_runs_out_and_the_stream_stays_usable():
    flag = torch.zeros(64, dtype=torch.int32, device=DEV)            # this "rank's" barrier counter
    peer = torch.tensor([flag.data_ptr()], dtype=torch.int64, device=DEV)  # world of one: its own counter
    err = torch.zeros(4, dtype=torch.int32, device=DEV)
    s = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    # one arrival (this call's) against a target of 2: nothing else will ever arrive
    _lib.call("pm_ep_barrier", peer.data_ptr(), flag.data_ptr(), 1, 2, err.data_ptr(), 50_000_000, s)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(err[0].item()) == 1
    assert 0.045 <= waited < 2.0, waited
    assert int(flag[0].item()) == 1
    # the counter now holds 1; the next call's own arrival reaches the target 2 and passes
    err.zero_()
    _lib.call("pm_ep_barrier", peer.data_ptr(), flag.data_ptr(), 1, 2, err.data_ptr(), 50_000_000, s)
    torch.cuda.synchronize()
    assert int(err[0].item()) == 0 and int(flag[0].item()) == 2
    # and the layer still runs on the same stream
    L = synth.make_fp8_layer(T=64, H=2048, I=768, E=128, seed=3, device=DEV, gen_device="cuda")
    out = ops.forward_fp8(L["x"], L["w1"], L["w1_s"], L["w2"], L["w2_s"], 8, router_w=L["router_w"])
    ws, _ = ops.workspace_for(L["x"], 64, 2048, 768, 128, 8)
    ops.read_status(ws)
    assert torch.isfinite(out.float()).all()
