"""pm_moe_align_noalloc: the expert alignment for callers that cannot give the library scratch memory.

Such callers -- hosts whose own pool owns every device byte, or hot loops that cannot risk the implicit
synchronisation of cudaMalloc/cudaFree -- get the same alignment as pm_moe_align with the count table held in a
fixed device array inside the library.  This file is collected last so that, if it fails, a run stopping at the
first failure has already run every other test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from tests.conftest import cuda_ok

pytestmark = pytest.mark.gpu

if cuda_ok():
    from prismyra_b200 import _lib, ops

DEV = "cuda:0"


def _noalloc(ids: torch.Tensor, E: int):
    T, k = ids.shape
    ms = _lib.max_slots(T, E, k)
    sorted_ids = torch.full((ms,), -7, dtype=torch.int32, device=DEV)
    expert_ids = torch.full((ms // 128,), -7, dtype=torch.int32, device=DEV)
    npp = torch.full((1,), -7, dtype=torch.int32, device=DEV)
    off = torch.full((E + 1,), -7, dtype=torch.int32, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = _lib.load().pm_moe_align_noalloc(
        ctypes.c_void_p(ids.data_ptr()), T, k, E, ctypes.c_void_p(sorted_ids.data_ptr()),
        ctypes.c_void_p(expert_ids.data_ptr()), ctypes.c_void_p(npp.data_ptr()), ctypes.c_void_p(off.data_ptr()),
        stream)
    return st, sorted_ids, expert_ids, npp, off


def _ids(T: int, E: int, k: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    ids[: T // 3, 0] = 1  # a hot expert, so expert sizes differ between the two calls
    return ids.to(DEV)


def _ids_fast(T: int, E: int, k: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    ids = torch.rand(T, E, generator=g).argsort(dim=1)[:, :k].to(torch.int32)
    ids[: T // 3, 0] = 1
    return ids.to(DEV)


@pytest.mark.parametrize("T,E,k", [(5120, 128, 8), (300, 64, 4), ((1 << 20) // 8, 256, 8)])
def test_noalloc_matches_the_workspace_entry_point_twice_in_a_row(T, E, k):
    # the last case fills the static table exactly: T*k = 2^20 pairs (256 chunks) and E = 256 experts
    for call, seed in enumerate((11, 12)):  # two calls in a row: the shared scratch must not leak between them
        ids = (_ids_fast if T * k > 100_000 else _ids)(T, E, k, seed + T)
        st, s, eids, npp, off = _noalloc(ids, E)
        assert st == 0, _lib.load().pm_moe_status_string(st)
        rs, reids, rnpp, roff, _, _ = ops.align(ids, E)
        torch.cuda.synchronize()
        n = int(rnpp.item())
        assert int(npp.item()) == n, f"call {call}"
        assert torch.equal(s[:n], rs[:n]), f"call {call}"
        assert torch.equal(eids[: n // 128], reids[: n // 128]), f"call {call}"
        assert torch.equal(off, roff), f"call {call}"


def test_noalloc_rejects_sizes_beyond_its_fixed_scratch():
    lib = _lib.load()
    dummy = torch.zeros(16, dtype=torch.int32, device=DEV)
    p = ctypes.c_void_p(dummy.data_ptr())
    assert lib.pm_moe_align_noalloc(p, (1 << 20) // 8 + 1, 8, 128, p, p, p, None, None) == 8
    assert lib.pm_moe_align_noalloc(p, 4, 8, 512, p, p, p, None, None) == 8
    assert b"fixed scratch" in lib.pm_moe_status_string(8)
