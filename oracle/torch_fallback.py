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


@torch.no_grad()
def time_routed(router, experts, x: torch.Tensor, min_seconds: float = 10.0, max_iters: int = 50,
                warmup: int = 1) -> dict:
    """Tokens/s of the routed path on this host's cores: warm-up calls, then repeated calls until at least
    ``min_seconds`` of CPU work (or ``max_iters`` calls) have been timed with ``time.perf_counter``."""
    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(warmup):
        routed(router, experts, x)
    n, t0 = 0, time.perf_counter()
    while True:
        routed(router, experts, x)
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or n >= max_iters:
            break
    return {"tokens_per_s": x.shape[0] * n / el, "seconds": el, "calls": n, "threads": torch.get_num_threads(),
            "cpu_count": os.cpu_count()}
