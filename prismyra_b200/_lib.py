"""ctypes binding of ``libprismyra_moe.so`` (the C ABI declared in ``include/prismyra_moe.h``).

The library is the only compute path: there is no CPU or PyTorch fallback.  Loading fails loudly when the
library is missing, and every call raises :class:`MoEKernelError` on a non-zero status.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libprismyra_moe.so"

PM_OK = 0
PM_ERR_TIMEOUT = 7
FMT_FP8 = 0
FMT_NVFP4 = 1
FLAG_ACT_SCALE_UE8M0 = 1
FLAG_ACT_SCALE_RCP = 2

# Workspace regions (enum pm_region).
WS = {
    "status": 0, "logits": 1, "topk_w": 2, "topk_ids": 3, "counts": 4, "expert_off": 5, "sorted": 6,
    "expert_ids": 7, "num_post_pad": 8, "a1": 9, "a1_scale": 10, "a2": 11, "a2_scale": 12, "c3": 13,
    "slot_of": 14,
    "router_part": 15, "sched": 16,
}

_P = ctypes.c_void_p
_I = ctypes.c_int
_Z = ctypes.c_size_t

# name -> (restype, argtypes); must cover every function declared in include/prismyra_moe.h
SIGNATURES: dict[str, tuple] = {
    "pm_moe_abi_version": (_I, []),
    "pm_moe_status_string": (ctypes.c_char_p, [_I]),
    "pm_moe_max_slots": (_I, [_I, _I, _I]),
    "pm_moe_align_workspace_bytes": (ctypes.c_size_t, [_I, _I, _I]),
    "pm_moe_workspace_bytes": (_Z, [_I, _I, _I, _I, _I, _I]),
    "pm_moe_workspace_region": (_I, [_I, _I, _I, _I, _I, _I, _I, ctypes.POINTER(_Z), ctypes.POINTER(_Z)]),
    "pm_moe_router_topk": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "pm_moe_topk": (_I, [_P, _P, _I, _I, _I, _P, _P, _P]),
    "pm_moe_align": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P, _P, _Z, _P]),
    "pm_moe_quant_fp8": (_I, [_P, _I, _I, _I, _P, _P, _P, _P]),
    "pm_moe_gemm1_fp8": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "pm_moe_gemm2_fp8": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P]),
    "pm_moe_combine": (_I, [_P, _P, _I, _I, _I, _P, _P]),
    "pm_moe_scatter_rows": (_I, [_P, _I, _I, _I, _P, _P, _I, _P]),
    "pm_moe_forward_fp8": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _Z, _P]),
    "pm_moe_quant_fp8_ex": (_I, [_P, _I, _I, _I, _P, _P, _P, _I, _P]),
    "pm_moe_forward_fp8_ex": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _Z, _P]),
    "pm_moe_read_status": (_I, [_P, _P]),
    "pm_moe_align_noalloc": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P]),
    "pm_moe_quant_nvfp4": (_I, [_P, _I, _I, _I, _P, ctypes.c_float, _P, _P, _P]),
    "pm_moe_gemm1_nvfp4": (_I, [_P, _P, _P, _P, _P, ctypes.c_float, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "pm_moe_gemm2_nvfp4": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P]),
    "pm_moe_forward_nvfp4": (_I, [_P, _P, _P, _P, _P, _P, ctypes.c_float, _P, _P, _P, ctypes.c_float, _I, _I, _I,
                                  _I, _I, _P, _P, _Z, _P]),
    "pm_nvfp4_prepare": (_I, [_P, _P, _I, _I, _I, _P, _P, _P, _P]),
    "pm_nvfp4_prepare_search": (_I, [_P, _P, _P, _I, _I, _I, _P, _P, _P, _P]),
    "pm_fp8_linear_workspace_bytes": (_Z, [_I, _I, _I]),
    "pm_fp8_linear": (_I, [_P, _P, _P, _I, _I, _I, _P, _P, _Z, _P]),
    "pm_moe_shared_workspace_bytes": (_Z, [_I, _I, _I]),
    "pm_moe_shared_fp8": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P, _P, _Z, _P]),
    "pm_moe_block_workspace_bytes": (_Z, [_I, _I, _I, _I, _I, _I]),
    "pm_moe_block_fp8": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _Z,
                              _P]),
    "pm_ep_alloc": (_I, [_Z, ctypes.POINTER(_P), _P]),
    "pm_ep_open": (_I, [_P, ctypes.POINTER(_P)]),
    "pm_ep_close": (_I, [_P]),
    "pm_ep_free": (_I, [_P]),
    "pm_ep_count": (_I, [_P, _I, _I, _I, _I, _P, _P]),
    "pm_ep_barrier": (_I, [_P, _P, _I, ctypes.c_uint, _P, ctypes.c_uint64, _P]),
    "pm_ep_offsets": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _I, _P, _P, _I, _P]),
    "pm_ep_dispatch_quant": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _I, _I,
                                  _P]),
    "pm_ep_gemm1_fp8": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _I, _P]),
    "pm_ep_local_rows": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "pm_ep_gemm2_fp8": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
}


class MoEKernelError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed with status {status}: {msg}")
        self.status = status


_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load the library (idempotent).  Raises if it has not been built -- there is nothing to fall back to."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m prismyra_b200.build` "
                    "(prismyra_b200 has no CPU fallback)"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                f = getattr(lib, name)
                f.restype = res
                f.argtypes = args
            _lib = lib
    return _lib


def call(name: str, *args) -> None:
    lib = load()
    st = getattr(lib, name)(*args)
    if st != PM_OK:
        raise MoEKernelError(name, st, lib.pm_moe_status_string(st).decode())


def workspace_bytes(T: int, H: int, I: int, E: int, k: int, fmt: int = FMT_FP8) -> int:
    return int(load().pm_moe_workspace_bytes(T, H, I, E, k, fmt))


def workspace_region(T: int, H: int, I: int, E: int, k: int, fmt: int, region: str) -> tuple[int, int]:
    off, n = _Z(0), _Z(0)
    call("pm_moe_workspace_region", T, H, I, E, k, fmt, WS[region], ctypes.byref(off), ctypes.byref(n))
    return off.value, n.value


def max_slots(T: int, E: int, k: int) -> int:
    return int(load().pm_moe_max_slots(T, E, k))


def align_workspace_bytes(T: int, k: int, E: int) -> int:
    """Scratch bytes pm_moe_align needs for T tokens, top-k and E experts."""
    return int(load().pm_moe_align_workspace_bytes(T, k, E))
