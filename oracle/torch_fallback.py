"""The reference's CPU implementation of the routed-expert layer, timed as the CPU baseline -- BENCH/TEST ONLY.

On a host without CUDA the reference never installs its fused kernels (prismyra/engine.py:690-695): the
framework's own ``Qwen3_5MoeSparseMoeBlock`` runs, i.e. transformers' ``Qwen3_5MoeTopKRouter`` (fp32 softmax,
top-k, renormalise) and ``Qwen3_5MoeExperts`` (a per-expert eager loop with ``index_add_``) on weights that
transformers dequantised from FP8 at load time, in float32 (the engine's CPU dtype, prismyra/engine.py:467).
This module builds exactly those transformers modules (transformers 5.5, the version installed here) around the
synthetic layer's dequantised weights and times the routed path on the host cores.
"""

from __future__ import annotations

import os
import time
from types import SimpleNamespace

import torch


def build_block(router_w: torch.Tensor, w1_deq: torch.Tensor, w2_deq: torch.Tensor, top_k: int,
                dtype=torch.float32):
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeExperts, Qwen3_5MoeTopKRouter

    E, I2, H = w1_deq.shape
    cfg = SimpleNamespace(num_experts=E, num_experts_per_tok=top_k, hidden_size=H, moe_intermediate_size=I2 // 2,
                          hidden_act="silu", _experts_implementation="eager")
    router = Qwen3_5MoeTopKRouter(cfg)
    experts = Qwen3_5MoeExperts(cfg)
    with torch.no_grad():
        router.weight = torch.nn.Parameter(router_w.to(dtype), requires_grad=False)
        experts.gate_up_proj = torch.nn.Parameter(w1_deq.to(dtype), requires_grad=False)
        experts.down_proj = torch.nn.Parameter(w2_deq.to(dtype), requires_grad=False)
    return router, experts


@torch.no_grad()
def routed(router, experts, x: torch.Tensor) -> torch.Tensor:
    _, weights, ids = router(x)
    return experts(x, ids, weights)


def cpu_model() -> str:
    """The host CPU's model name (from /proc/cpuinfo), or the platform's processor string."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.lower().startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


@torch.no_grad()
def time_routed(router, experts, x: torch.Tensor, warmup: int = 2, min_calls: int = 5, max_seconds: float = 30.0,
                max_calls: int = 50) -> dict:
    """Tokens/s of the routed path on this host's cores: ``warmup`` untimed calls, then calls timed one by one with
    ``time.perf_counter`` -- at least ``min_calls``, more while the total stays under ``max_seconds`` (at most
    ``max_calls``) -- and the median call time."""
    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(warmup):
        routed(router, experts, x)
    times: list[float] = []
    t_start = time.perf_counter()
    while len(times) < min_calls or (time.perf_counter() - t_start < max_seconds and len(times) < max_calls):
        t0 = time.perf_counter()
        routed(router, experts, x)
        times.append(time.perf_counter() - t0)
    med = sorted(times)[len(times) // 2]
    return {"tokens_per_s": x.shape[0] / med, "median_s": med, "calls": len(times), "warmup": warmup,
            "seconds": sum(times), "threads": torch.get_num_threads(), "cpu_count": os.cpu_count(),
            "cpu_model": cpu_model(), "dtype": str(x.dtype).replace("torch.", "")}
