"""ctypes/numpy front end of the C oracle in ``oracle/moe_oracle.c`` -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` leg may import this module;
the product path (``prismyra_b200``) never does.  Every function mirrors a C function whose header comment
cites the reference source it restates.  Arrays are numpy; bf16 travels as its uint16 bit pattern.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libmoe_oracle.so"

_lib = None


def build() -> Path:
    """Compile the oracle with the committed Makefile (gcc only; no reference code is built)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < (HERE / "moe_oracle.c").stat().st_mtime:
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a), dtype=dtype)


# ------------------------------------------------------------------------------------------- formats
def bf16_to_f32(bits) -> np.ndarray:
    b = _c(bits, np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().or_f32_to_bf16_n(_p(x), ctypes.c_long(x.size), _p(out))
    return out


def f32_to_e4m3(x) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint8)
    lib().or_f32_to_e4m3_n(_p(x), ctypes.c_long(x.size), _p(out))
    return out


def e4m3_to_f32(b) -> np.ndarray:
    b = _c(b, np.uint8)
    table = np.empty(256, np.float32)
    f = lib().or_e4m3_to_f32
    f.restype = ctypes.c_float
    for i in range(256):
        table[i] = f(ctypes.c_uint8(i))
    return table[b]


def f32_to_e2m1(x) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint8)
    lib().or_f32_to_e2m1_n(_p(x), ctypes.c_long(x.size), _p(out))
    return out


E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)


def e2m1_unpack(packed) -> np.ndarray:
    """uint8 [..., n/2] -> float32 [..., n]: low nibble is the even column, high nibble the odd one."""
    p = _c(packed, np.uint8)
    codes = np.stack([p & 15, p >> 4], axis=-1).reshape(*p.shape[:-1], p.shape[-1] * 2)
    v = E2M1[codes & 7]
    return np.where(codes & 8, -v, v).astype(np.float32)


# ------------------------------------------------------------------------------------------- stages
def route_topk(logits_bits, k: int):
    lg = _c(logits_bits, np.uint16)
    T, E = lg.shape
    w = np.empty((T, k), np.float32)
    ids = np.empty((T, k), np.int32)
    lib().or_route_topk(_p(lg), T, E, k, _p(w), _p(ids))
    return w, ids


def route_topk_f32(scores, k: int):
    sc = _c(scores, np.float32)
    T, E = sc.shape
    w = np.empty((T, k), np.float32)
    ids = np.empty((T, k), np.int32)
    lib().or_route_topk_f32(_p(sc), T, E, k, _p(w), _p(ids))
    return w, ids


def align(ids, num_experts: int, block_m: int):
    flat = _c(ids, np.int32).reshape(-1)
    n = flat.size
    cap = n + num_experts * (block_m - 1)
    sorted_ids = np.empty(cap, np.int32)
    expert_ids = np.empty((cap + block_m - 1) // block_m, np.int32)
    npp = np.zeros(1, np.int32)
    nb = lib().or_align(_p(flat), n, num_experts, block_m, _p(sorted_ids), _p(expert_ids), _p(npp))
    return sorted_ids[: int(npp[0])].copy(), expert_ids[:nb].copy(), int(npp[0])


#: Activation-scale rules, numbered as the library's flags (include/prismyra_moe.h PM_FLAG_ACT_SCALE_*): "fp32" the
#: correctly rounded max(amax, 1e-10)/448 (vLLM's compiled quantiser), "ue8m0" that rounded up to a power of two,
#: "fp32_rcp" max(amax, 1e-10) * fl(1/448) (vLLM's Triton kernel, what the golden fixtures were made with).
SCALE_RULES = {"fp32": 0, "ue8m0": 1, "fp32_rcp": 2}


def quant_fp8_groups(x_bits, scale: str = "fp32"):
    x = _c(x_bits, np.uint16)
    R, C = x.shape
    q = np.empty((R, C), np.uint8)
    s = np.empty((R, C // 128), np.float32)
    lib().or_quant_fp8_groups_ex(_p(x), R, C, _p(q), _p(s), SCALE_RULES[scale])
    return q, s


def silu_mul(g_bits, u_bits) -> np.ndarray:
    g = _c(g_bits, np.uint16)
    u = _c(u_bits, np.uint16)
    out = np.empty(g.shape, np.uint16)
    lib().or_silu_mul_n(_p(g), _p(u), ctypes.c_long(g.size), _p(out))
    return out


def gemm_fp8_rows(a, a_s, row_expert, w, w_s) -> np.ndarray:
    a = _c(a, np.uint8)
    a_s = _c(a_s, np.float32)
    re = _c(row_expert, np.int32)
    w = _c(w, np.uint8)
    w_s = _c(w_s, np.float32)
    rows, K = a.shape
    E, N, _ = w.shape
    out = np.empty((rows, N), np.float32)
    lib().or_gemm_fp8_rows(_p(a), _p(a_s), _p(re), rows, _p(w), _p(w_s), N, K, _p(out))
    return out


def router_logits(x_bits, w_bits) -> np.ndarray:
    x = _c(x_bits, np.uint16)
    w = _c(w_bits, np.uint16)
    T, H = x.shape
    E = w.shape[0]
    out = np.empty((T, E), np.uint16)
    lib().or_router_logits(_p(x), _p(w), T, H, E, _p(out))
    return out


def moe_forward_fp8(x_bits, logits_bits, w1, w1_s, w2, w2_s, k: int, want_intermediates: bool = False,
                    scale: str = "fp32"):
    """The whole routed FP8 layer; returns a dict with ``out`` (bf16 bits [T,H]) and, on request, the
    routing and the intermediates the CUDA stages produce (x_q, x_s, c2q, c2s, c3).  ``scale``: the activation-scale
    rule of both quantisations (:data:`SCALE_RULES`)."""
    x = _c(x_bits, np.uint16)
    lg = _c(logits_bits, np.uint16)
    w1 = _c(w1, np.uint8)
    w1_s = _c(w1_s, np.float32)
    w2 = _c(w2, np.uint8)
    w2_s = _c(w2_s, np.float32)
    T, H = x.shape
    E, I2, _ = w1.shape
    I = I2 // 2
    out = np.empty((T, H), np.uint16)
    r = {"out": out}
    if want_intermediates:
        r.update(
            weights=np.empty((T, k), np.float32),
            ids=np.empty((T, k), np.int32),
            x_q=np.empty((T, H), np.uint8),
            x_s=np.empty((T, H // 128), np.float32),
            c2q=np.empty((T * k, I), np.uint8),
            c2s=np.empty((T * k, I // 128), np.float32),
            c3=np.empty((T * k, H), np.uint16),
        )
    g = r.get
    lib().or_moe_forward_fp8_ex(
        _p(x), _p(lg), _p(w1), _p(w1_s), _p(w2), _p(w2_s), T, H, I, E, k, _p(out),
        _p(g("weights")), _p(g("ids")), _p(g("x_q")), _p(g("x_s")), _p(g("c2q")), _p(g("c2s")), _p(g("c3")),
        SCALE_RULES[scale],
    )
    return r


def shared_gate(x_bits, w_sg_bits) -> np.ndarray:
    """bf16(sigmoid(bf16(x . w_sg))) per token as fp32 (reference qwen3_moe.py:172-183 and :198): the dot is
    exact in float64 before its bf16 rounding; the sigmoid is evaluated in float64 and rounded to fp32, then
    bf16."""
    x = bf16_to_f32(_c(x_bits, np.uint16)).astype(np.float64)
    w = bf16_to_f32(_c(w_sg_bits, np.uint16).reshape(-1)).astype(np.float64)
    logit = bf16_to_f32(f32_to_bf16((x @ w).astype(np.float32))).astype(np.float64)
    sig = (1.0 / (1.0 + np.exp(-logit))).astype(np.float32)
    return bf16_to_f32(f32_to_bf16(sig))


def shared_expert_fp8(x_bits, w_sg_bits, w13, w13_s, w2, w2_s) -> np.ndarray:
    """The shared expert sigmoid(gate) * MLP(x) as bf16 bits [T, H] (reference qwen3_moe.py:198 with Fp8Linear
    projections, :211-230): the MLP is the routed restatement with one expert and top-1 (weight exactly 1), so it
    shares its quantisation, block-scaled GEMM and two-rounding silu*mul; the bf16 MLP output is then multiplied
    by the bf16 gate and rounded."""
    x = _c(x_bits, np.uint16)
    T = x.shape[0]
    one = np.zeros((T, 1), np.uint16)
    mlp = moe_forward_fp8(x, one, _c(w13, np.uint8)[None], _c(w13_s, np.float32)[None], _c(w2, np.uint8)[None],
                          _c(w2_s, np.float32)[None], 1)["out"]
    g = shared_gate(x, w_sg_bits)
    return f32_to_bf16(g[:, None] * bf16_to_f32(mlp))


def add_bf16(a_bits, b_bits) -> np.ndarray:
    """bf16(a + b) of two bf16 tensors (`routed + shared`, reference qwen3_moe.py:199)."""
    return f32_to_bf16(bf16_to_f32(_c(a_bits, np.uint16)) + bf16_to_f32(_c(b_bits, np.uint16)))


def nvfp4_quant_act(x_bits, gs: float):
    x = _c(x_bits, np.uint16)
    R, C = x.shape
    packed = np.empty((R, C // 2), np.uint8)
    sf = np.empty((R, C // 16), np.uint8)
    lib().or_nvfp4_quant_act(_p(x), R, C, ctypes.c_float(gs), _p(packed), _p(sf))
    return packed, sf


def nvfp4_quant_weight(w, g: float):
    w = _c(w, np.float32)
    R, C = w.shape
    packed = np.empty((R, C // 2), np.uint8)
    sf = np.empty((R, C // 16), np.uint8)
    lib().or_nvfp4_quant_weight(_p(w), R, C, ctypes.c_float(g), _p(packed), _p(sf))
    return packed, sf


def nvfp4_prepare(w_bits, s):
    """FP8 stack e4m3 bytes [E, R, C] + fp32 multipliers [E, R/128, C/128] -> (packed, sf, g) as prepare_layer."""
    w = _c(w_bits, np.uint8)
    s = _c(s, np.float32)
    E, R, C = w.shape
    packed = np.empty((E, R, C // 2), np.uint8)
    sf = np.empty((E, R, C // 16), np.uint8)
    g = np.empty(E, np.float32)
    lib().or_nvfp4_prepare(_p(w), _p(s), E, R, C, _p(packed), _p(sf), _p(g))
    return packed, sf, g


def moe_forward_nvfp4(x_bits, logits_bits, w1, s1, w2, s2, alpha1, alpha2, a1_gs: float, a2_gs: float, k: int,
                      want_c3: bool = False):
    x = _c(x_bits, np.uint16)
    lg = _c(logits_bits, np.uint16)
    w1 = _c(w1, np.uint8)
    s1 = _c(s1, np.uint8)
    w2 = _c(w2, np.uint8)
    s2 = _c(s2, np.uint8)
    al1 = _c(alpha1, np.float32)
    al2 = _c(alpha2, np.float32)
    T, H = x.shape
    E, I2, _ = w1.shape
    I = I2 // 2
    out = np.empty((T, H), np.uint16)
    c3 = np.empty((T * k, H), np.uint16) if want_c3 else None
    lib().or_moe_forward_nvfp4(
        _p(x), _p(lg), _p(w1), _p(s1), _p(w2), _p(s2), _p(al1), _p(al2), ctypes.c_float(a1_gs),
        ctypes.c_float(a2_gs), T, H, I, E, k, _p(out), _p(c3),
    )
    return {"out": out, "c3": c3}


def gemm_nvfp4_rows(a, a_sf, row_expert, w, w_sf, alpha) -> np.ndarray:
    a = _c(a, np.uint8)
    a_sf = _c(a_sf, np.uint8)
    re = _c(row_expert, np.int32)
    w = _c(w, np.uint8)
    w_sf = _c(w_sf, np.uint8)
    al = _c(alpha, np.float32)
    rows, K2 = a.shape
    E, N, _ = w.shape
    out = np.empty((rows, N), np.float32)
    lib().or_gemm_nvfp4_rows(_p(a), _p(a_sf), _p(re), rows, _p(w), _p(w_sf), _p(al), N, K2 * 2, _p(out))
    return out


def nvfp4_dequant(packed, sf, gs: float) -> np.ndarray:
    """Values of an NVFP4 tensor (unblocked scales [R, K/16]) divided by its global scale."""
    v = e2m1_unpack(packed)
    R, K = v.shape
    s = e4m3_to_f32(sf).reshape(R, K // 16, 1) / np.float32(gs)
    return (v.reshape(R, K // 16, 16) * s).reshape(R, K).astype(np.float32)
