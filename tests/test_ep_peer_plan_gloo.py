"""The planning of the expert-parallel layer over peer memory, on CPU ranks (gloo, world size 2 and 4).

The kernels pm_ep_count / pm_ep_offsets / pm_ep_dispatch_quant (prismyra_b200/csrc/moe_ep.cu) decide, with no host
synchronisation, where every (token, slot) pair of every rank lands in its expert owner's slot space.  Here that
planning is restated in numpy and run by real ranks that exchange only what the kernels exchange (each rank's row of
per-expert counts, which the kernels store into every rank's count matrix):

* ep_count: rank r's row of the count matrix [G][E] = its pairs per global expert;
* ep_offsets: for every global expert e owned by rank d = e // epr, the first slot of rank r's pairs of e in d's slot
  space is (padded sizes of d's experts before e) + (pairs of e on ranks before r); the owner's block table marks
  every 128-slot block with its local expert and its slot count is the sum of its padded expert sizes;
* ep_dispatch_quant: a pair goes to that base plus its rank among rank r's own pairs of e in ascending flat order.

Every owner's resulting slot table (source rank, pair) and block table must equal the single-GPU alignment (the
oracle's restatement of vLLM's moe_align_block_size) of all ranks' pairs concatenated in rank order, restricted to
that owner's experts.  Ranks have different token counts and a hot expert spanning several blocks.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O

E, K, BM = 16, 4, 128


def _ids(rank: int) -> np.ndarray:
    T = 150 + 61 * rank  # uneven token counts over the ranks
    rng = np.random.default_rng(100 + rank)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    ids[: T // 2, 0] = 3  # a hot expert: well over one block on every rank
    ids[: T // 2, 1:] = np.where(ids[: T // 2, 1:] == 3, 4, ids[: T // 2, 1:])
    return ids


def plan_offsets(cm: np.ndarray, rank: int, epr: int):
    """ep_offsets_kernel: per global expert the first slot of this rank's pairs in the owner's slot space, and this
    rank's own block table and slot count."""
    G, E_ = cm.shape
    padded = (cm.sum(0) + BM - 1) // BM * BM
    pre = cm[:rank].sum(0)
    base = np.empty(E_, np.int64)
    for e in range(E_):
        d = e // epr
        base[e] = padded[d * epr:e].sum() + pre[e]
    own = range(rank * epr, (rank + 1) * epr)
    blocks = np.concatenate([np.full(padded[e] // BM, e - rank * epr, np.int32) for e in own])
    return base, blocks, int(padded[rank * epr:(rank + 1) * epr].sum())


def dispatch_slots(ids: np.ndarray, base: np.ndarray) -> np.ndarray:
    """ep_dispatch_quant_kernel: slot of every flat pair = base[e] + its rank among this rank's pairs of e."""
    flat = ids.reshape(-1)
    slot = np.empty(flat.size, np.int64)
    for e in np.unique(flat):
        where = np.nonzero(flat == e)[0]  # ascending flat order, as the local alignment sorts them
        slot[where] = base[e] + np.arange(where.size)
    return slot


def _rank_main(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        epr = E // world
        ids = _ids(rank)
        row = torch.from_numpy(np.bincount(ids.reshape(-1), minlength=E).astype(np.int64))
        rows = [torch.empty_like(row) for _ in range(world)]
        dist.all_gather(rows, row)  # the count matrix every rank holds after the counts' peer stores
        cm = torch.stack(rows).numpy()
        base, blocks, npp = plan_offsets(cm, rank, epr)
        slots = dispatch_slots(ids, base)
        flat = ids.reshape(-1)
        owner = flat // epr
        # what each owner receives: (slot, source rank, source pair) -- the kernels' stores of meta into its region
        sent = [np.stack([slots[owner == d], np.full((owner == d).sum(), rank), np.nonzero(owner == d)[0]], 1)
                for d in range(world)]
        results[rank] = {"ids": ids, "blocks": blocks, "npp": npp, "sent": sent}
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(240)
@pytest.mark.parametrize("world", [2, 4])
def test_peer_plan_equals_the_single_gpu_alignment_restricted_to_each_owner(world):
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
        res = [dict(results[r]) for r in range(world)]
    epr = E // world
    # the single-GPU alignment of all ranks' pairs concatenated in rank order
    all_ids = np.concatenate([r["ids"] for r in res])
    sorted_ids, expert_ids, n = O.align(all_ids, E, BM)
    first_pair = np.cumsum([0] + [r["ids"].size for r in res])  # global flat index of each rank's pair 0
    for d in range(world):
        own = [e for e in range(d * epr, (d + 1) * epr)]
        # the oracle's slots of d's experts, in order, with global flat indices (padding = all_ids.size)
        keep = np.isin(np.repeat(expert_ids, BM), own)
        want = sorted_ids[keep]
        want_blocks = expert_ids[np.isin(expert_ids, own)] - d * epr
        assert np.array_equal(res[d]["blocks"], want_blocks)
        assert res[d]["npp"] == want.size
        table = np.full(res[d]["npp"], all_ids.size, np.int64)
        for r in range(world):
            slot, src, pair = res[r]["sent"][d].T
            assert np.all((slot >= 0) & (slot < res[d]["npp"]))
            assert np.all(table[slot] == all_ids.size)  # no slot is written twice
            table[slot] = first_pair[src] + pair
        assert np.array_equal(table, want)
    assert sum(r["npp"] for r in res) == n  # every pair found exactly one owner's slot
