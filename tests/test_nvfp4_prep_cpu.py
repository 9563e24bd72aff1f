"""The NVFP4 weight preparation of ``prismyra_b200.kernels.nvfp4`` on the CPU against the reference's own
outputs (``tests/golden/nvfp4.npz`` and ``nvfp4_search.npz``, made by the reference's prepare_layer, quantize and
quantize_search): bit-exact codes, scale bytes and global scales."""

from __future__ import annotations

import numpy as np
import torch

from prismyra_b200.kernels import nvfp4

FP8 = torch.float8_e4m3fn


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.view(dtype) if dtype is not None else t


def _b(t: torch.Tensor) -> np.ndarray:
    t = t.contiguous()
    return (t.view(torch.uint8) if t.dtype == FP8 else t).numpy()


def test_quantize_matches_reference(golden):
    g = golden("nvfp4")
    packed, scale = nvfp4.quantize(_t(g["w"]), float(g["gs"]))
    assert np.array_equal(_b(packed), g["packed"]) and np.array_equal(_b(scale), g["scale"])


def test_quantize_search_matches_reference(golden):
    g = golden("nvfp4_search")
    w, gs = _t(g["w"]), _t(g["gs"])[0]
    for imp, pk, sk in ((_t(g["imp"]), "p_imp", "s_imp"), (None, "p_one", "s_one")):
        packed, scale = nvfp4.quantize_search(w, gs, imp)
        assert np.array_equal(_b(packed), g[pk]) and np.array_equal(_b(scale), g[sk])


def test_prepare_layer_matches_reference(golden):
    g = golden("nvfp4")
    prep = nvfp4.prepare_layer(_t(g["fp8_w"], FP8), _t(g["fp8_s"]), _t(g["fp8_w2"], FP8), _t(g["fp8_s2"]), "cpu")
    for k in ("w1", "s1", "g1", "w2", "s2", "g2"):
        assert np.array_equal(_b(prep[k]), g["prep_" + k]), k


def test_prepare_layer_with_importance_matches_reference(golden):
    g = golden("nvfp4_search")
    prep = nvfp4.prepare_layer(_t(g["fp8_w"], FP8), _t(g["fp8_s"]), _t(g["fp8_w2"], FP8), _t(g["fp8_s2"]), "cpu",
                               imp_in=_t(g["imp_in"]), imp_mid=_t(g["imp_mid"]), tok=_t(g["tok"]))
    for k in ("w1", "s1", "g1", "w2", "s2", "g2"):
        assert np.array_equal(_b(prep[k]), g["prep_" + k]), k
