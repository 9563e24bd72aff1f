"""Expert-parallel dispatch / exchange / combine on CPU ranks (gloo, world size 2), with the CPU oracle as the
per-rank compute: the sharded layer must reproduce the single-process oracle layer bit for bit."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from prismyra_b200 import ep, synth

H, I, E, K, T = 256, 128, 8, 4, 40


def _bits(t):
    return t.contiguous().view(torch.uint16).numpy() if t.dtype == torch.bfloat16 else t.contiguous().numpy()


class OracleBackend:
    """The per-rank compute restated with the oracle (FP8 experts [lo, hi) of the layer)."""

    def __init__(self, L, lo, hi, k):
        self.L, self.lo, self.hi, self.k = L, lo, hi, k

    def route(self, x):
        logits = O.router_logits(_bits(x), _bits(self.L["router_w"]))
        w, ids = O.route_topk(logits, self.k)
        return torch.from_numpy(w), torch.from_numpy(ids)

    def quant_dispatch(self, x, send_pos, k, rows):
        xq, xs = O.quant_fp8_groups(_bits(x))
        n = rows
        q = np.zeros((n, H), np.uint8)
        s = np.zeros((n, H // 128), np.float32)
        sp = send_pos.numpy().reshape(-1, k)
        for j in range(k):
            q[sp[:, j]] = xq
            s[sp[:, j]] = xs
        return torch.from_numpy(q), torch.from_numpy(s)

    def local_experts(self, rq, rs, re, rw):
        L = self.L
        w1 = L["w1"][self.lo:self.hi].view(torch.uint8).numpy()
        w2 = L["w2"][self.lo:self.hi].view(torch.uint8).numpy()
        c1 = O.f32_to_bf16(O.gemm_fp8_rows(rq.numpy(), rs.numpy(), re.numpy(), w1, L["w1_s"][self.lo:self.hi].numpy()))
        c2 = O.silu_mul(c1[:, :I], c1[:, I:])
        c2q, c2s = O.quant_fp8_groups(c2)
        o = O.gemm_fp8_rows(c2q, c2s, re.numpy(), w2, L["w2_s"][self.lo:self.hi].numpy())
        c3 = O.f32_to_bf16(o * rw.numpy()[:, None])
        return torch.from_numpy(c3.view(np.int16)).view(torch.bfloat16)

    def combine(self, back, T_, k, send_pos):
        b = O.bf16_to_f32(_bits(back))
        sp = send_pos.numpy().reshape(T_, k)
        acc = np.zeros((T_, H), np.float32)
        for j in range(k):
            acc = (acc + b[sp[:, j]]).astype(np.float32)
        return torch.from_numpy(O.f32_to_bf16(acc).view(np.int16)).view(torch.bfloat16)


def _rank_main(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        L = synth.make_fp8_layer(world * T, H, I, E, seed=5)
        epr = E // world
        layer = ep.ExpertParallelLayer(OracleBackend(L, rank * epr, (rank + 1) * epr, K), E, K, rank, world)
        out = layer.forward(L["x"][rank * T:(rank + 1) * T].contiguous())
        results[rank] = _bits(out).copy()
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_plan_dispatch_groups_pairs_by_owner_in_flat_order():
    ids = torch.tensor([[0, 5, 2], [7, 1, 4], [3, 6, 0]], dtype=torch.int32)
    send_pos, counts, order, local = ep.plan_dispatch(ids, experts_per_rank=4, world=2)
    assert counts.tolist() == [5, 4]
    # rank 0 gets flat pairs 0,2,4,6,8 (experts 0,2,1,3,0) in that order, rank 1 gets 1,3,5,7 (5,7,4,6)
    assert order.tolist() == [0, 2, 4, 6, 8, 1, 3, 5, 7]
    assert local.tolist() == [0, 2, 1, 3, 0, 1, 3, 0, 2]
    assert send_pos[order].tolist() == list(range(9))


def test_world_of_one_is_the_plain_layer():
    L = synth.make_fp8_layer(T, H, I, E, seed=5)
    layer = ep.ExpertParallelLayer(OracleBackend(L, 0, E, K), E, K, 0, 1)
    out = _bits(layer.forward(L["x"][:T].contiguous()))
    logits = O.router_logits(_bits(L["x"][:T]), _bits(L["router_w"]))
    ref = O.moe_forward_fp8(_bits(L["x"][:T]), logits, L["w1"].view(torch.uint8).numpy(), L["w1_s"].numpy(),
                            L["w2"].view(torch.uint8).numpy(), L["w2_s"].numpy(), K)["out"]
    assert np.array_equal(out, ref)


@pytest.mark.timeout(240)
def test_two_gloo_ranks_reproduce_the_single_process_layer_bit_for_bit():
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(200)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        outs = [results[r] for r in range(world)]
    L = synth.make_fp8_layer(world * T, H, I, E, seed=5)
    logits = O.router_logits(_bits(L["x"]), _bits(L["router_w"]))
    ref = O.moe_forward_fp8(_bits(L["x"]), logits, L["w1"].view(torch.uint8).numpy(), L["w1_s"].numpy(),
                            L["w2"].view(torch.uint8).numpy(), L["w2_s"].numpy(), K)["out"]
    assert np.array_equal(np.concatenate(outs), ref)
