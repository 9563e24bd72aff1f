"""Expert parallelism on the GPU: the sharded layer is bit-identical to the single-GPU layer.

One GPU: world size 1 through the full EP code path.  Two GPUs (when visible): two NCCL ranks, each holding half of
the experts, each checking its tokens against the single-GPU layer computed with all experts.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from tests.conftest import cuda_ok

pytestmark = pytest.mark.gpu

if cuda_ok():
    from prismyra_b200 import ep, ops, synth

H, I, E, K, T = 2048, 768, 128, 8, 640


def _layer(dev):
    return synth.make_fp8_layer(T, H, I, E, seed=3, device=dev, gen_device="cuda")


def test_world_of_one_matches_the_plain_layer():
    L = _layer("cuda:0")
    b = ep.CudaBackend(L["w1"], L["w1_s"], L["w2"], L["w2_s"], L["router_w"], K)
    out = ep.ExpertParallelLayer(b, E, K, 0, 1).forward(L["x"])
    ref = ops.forward_fp8(L["x"], L["w1"], L["w1_s"], L["w2"], L["w2_s"], K, router_w=L["router_w"])
    assert torch.equal(out, ref)


def test_zipf_bias_skews_the_load_and_ranks_like_the_oracle():
    from oracle import oracle as O

    L = _layer("cuda:0")
    bias = synth.zipf_bias(E).to("cuda:0")
    logits, w, ids = ops.router_topk(L["x"], L["router_w"], K, bias=bias)
    load = torch.bincount(ids.reshape(-1).long(), minlength=E).float()
    assert load.max() > 4 * load.mean()  # the hottest expert takes several times its uniform share
    scores = (logits.float() + bias).cpu().numpy()  # the kernel adds the bias to the bf16 logit in fp32
    rw, rids = O.route_topk_f32(scores, K)
    assert (ids.cpu().numpy() == rids).all()
    assert abs(w.cpu().numpy() - rw).max() <= 1e-6 * abs(rw).max() * 4


def _rank(rank, world, port, errors):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        dev = torch.device("cuda", rank)
        L = _layer(dev)
        g = torch.Generator("cuda").manual_seed(100 + rank)
        x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
        epr = E // world
        lo, hi = rank * epr, (rank + 1) * epr
        b = ep.CudaBackend(L["w1"][lo:hi].contiguous(), L["w1_s"][lo:hi].contiguous(), L["w2"][lo:hi].contiguous(),
                           L["w2_s"][lo:hi].contiguous(), L["router_w"], K)
        out = ep.ExpertParallelLayer(b, E, K, rank, world).forward(x)
        ref = ops.forward_fp8(x, L["w1"], L["w1_s"], L["w2"], L["w2_s"], K, router_w=L["router_w"])
        torch.cuda.synchronize()
        if not torch.equal(out, ref):
            errors[rank] = float((out.float() - ref.float()).abs().max())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not cuda_ok() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_nccl_ranks_match_the_single_gpu_layer():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        errors = mgr.dict()
        procs = [ctx.Process(target=_rank, args=(r, 2, port, errors)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        assert dict(errors) == {}


def _peer_rank(rank, world, port, errors, groups):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    layer = None
    try:
        dev = torch.device("cuda", rank)
        L = _layer(dev)
        epr = E // world
        lo, hi = rank * epr, (rank + 1) * epr
        b = ep.CudaBackend(L["w1"][lo:hi].contiguous(), L["w1_s"][lo:hi].contiguous(), L["w2"][lo:hi].contiguous(),
                           L["w2_s"][lo:hi].contiguous(), L["router_w"], K)
        layer = ep.PeerExpertParallelLayer(b, E, K, rank, world, max_tokens=T, groups=groups)
        for call, (seed, n) in enumerate(((100 + rank, T), (200 + rank, T - 37))):  # buffers reused, fewer tokens
            g = torch.Generator("cuda").manual_seed(seed)
            x = torch.randn(n, H, generator=g, device=dev).to(torch.bfloat16)
            out = layer.forward(x)
            ref = ops.forward_fp8(x, L["w1"], L["w1_s"], L["w2"], L["w2_s"], K, router_w=L["router_w"])
            torch.cuda.synchronize()
            if layer.errors():
                errors[(rank, call)] = "kernel error flag"
            elif not torch.equal(out, ref):
                errors[(rank, call)] = float((out.float() - ref.float()).abs().max())
    finally:
        if layer is not None:
            layer.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not cuda_ok() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("groups", [1, 2, 4])
def test_two_ranks_over_peer_memory_match_the_single_gpu_layer(groups):
    """The peer-memory expert-parallel layer (rows stored straight into the owners' slots and back over NVLink,
    device barriers, no host synchronisation): bit-identical to one GPU, twice in a row on the same buffers; with
    the experts dispatched in 1, 2 or 4 groups (later groups on a side stream beside the earlier groups' GEMMs)."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        errors = mgr.dict()
        procs = [ctx.Process(target=_peer_rank, args=(r, 2, port, errors, groups)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        assert dict(errors) == {}
