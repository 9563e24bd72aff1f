"""The C-ABI library without a GPU: it loads, exports exactly what include/prismyra_moe.h declares, and rejects
bad arguments before touching a device."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from prismyra_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def declared_functions() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(pm_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    names = declared_functions()
    assert len(names) >= 14
    for n in sorted(names):
        assert hasattr(lib, n), f"{n} is declared but not exported"


def test_binding_covers_every_declared_symbol():
    assert declared_functions() == set(_lib.SIGNATURES)


def test_abi_version_and_status_strings():
    lib = _lib.load()
    assert lib.pm_moe_abi_version() == 1
    for st in range(8):
        assert lib.pm_moe_status_string(st)
    assert b"unknown" in lib.pm_moe_status_string(99)


def test_workspace_sizes():
    n = _lib.workspace_bytes(5120, 2048, 768, 128, 8)
    # dominated by the slot-ordered activations (57216 x 2048), the down input and the [T*k, H] bf16 outputs
    assert 300e6 < n < 400e6
    assert _lib.max_slots(5120, 128, 8) == 57216
    assert _lib.max_slots(1, 128, 8) == 8 + 128 * 127 + 120
    off, size = _lib.workspace_region(5120, 2048, 768, 128, 8, 0, "c3")
    assert size == 5120 * 8 * 2048 * 2 and off % 256 == 0 and off + size <= n
    off0, size0 = _lib.workspace_region(5120, 2048, 768, 128, 8, 0, "status")
    assert off0 == 0 and size0 == 16


@pytest.mark.parametrize("shape", [(16, 2000, 768, 128, 8), (16, 2048, 700, 128, 8), (16, 2048, 768, 300, 8),
                                   (16, 2048, 768, 128, 17), (16, 2048, 768, 4, 8), (-1, 2048, 768, 128, 8)])
def test_bad_shapes_are_rejected_without_a_device(shape):
    assert _lib.workspace_bytes(*shape, 0) == 0
    lib = _lib.load()
    T, H, I, E, k = shape
    st = lib.pm_moe_forward_fp8(None, None, None, None, None, None, None, T, H, I, E, k, None, None, 0, None)
    assert st in (1, 2)


def test_null_pointers_are_rejected_without_a_device():
    lib = _lib.load()
    st = lib.pm_moe_forward_fp8(None, None, None, None, None, None, None, 16, 2048, 768, 128, 8, None, None, 0, None)
    assert st == 1
    assert lib.pm_moe_topk(None, None, 4, 128, 8, None, None, None) == 1
    assert lib.pm_moe_combine(None, None, 4, 8, 2048, None, None) == 1
    assert lib.pm_moe_read_status(None, None) == 1
    assert lib.pm_nvfp4_prepare(None, None, 4, 256, 256, None, None, None, None) == 1
    assert lib.pm_nvfp4_prepare(None, None, 4, 200, 256, None, None, None, None) == 2
    assert lib.pm_nvfp4_prepare(None, None, 4, 256, 100, None, None, None, None) == 2
    assert lib.pm_nvfp4_prepare(None, None, 0, 256, 256, None, None, None, None) == 0
    assert lib.pm_nvfp4_prepare_search(None, None, None, 4, 256, 256, None, None, None, None) == 1
    assert lib.pm_nvfp4_prepare_search(None, None, None, 4, 200, 256, None, None, None, None) == 2
    assert lib.pm_nvfp4_prepare_search(None, None, None, 4, 256, 100, None, None, None, None) == 2
    assert lib.pm_nvfp4_prepare_search(None, None, None, 0, 256, 256, None, None, None, None) == 0
    assert lib.pm_fp8_linear(None, None, None, 4, 2048, 2048, None, None, 0, None) == 1
    assert lib.pm_fp8_linear(None, None, None, 4, 2000, 2048, None, None, 0, None) == 2
    assert lib.pm_fp8_linear(None, None, None, 4, 2048, 1920, None, None, 0, None) == 2
    assert lib.pm_fp8_linear_workspace_bytes(4, 2048, 1920) == 0
    assert lib.pm_moe_shared_fp8(None, None, None, None, None, None, 4, 2048, 512, None, None, 0, None) == 1
    assert lib.pm_moe_shared_fp8(None, None, None, None, None, None, 4, 2048, 500, None, None, 0, None) == 2
    assert lib.pm_moe_block_workspace_bytes(4, 2048, 768, 500, 128, 8) == 0
    assert lib.pm_moe_block_workspace_bytes(4, 2048, 768, 512, 128, 8) > lib.pm_moe_workspace_bytes(4, 2048, 768,
                                                                                                   128, 8, 0)


def test_zero_tokens_is_a_no_op():
    lib = _lib.load()
    assert lib.pm_moe_forward_fp8(None, None, None, None, None, None, None, 0, 2048, 768, 128, 8, None, None, 0,
                                  None) == 0
