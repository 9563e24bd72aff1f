"""Expert parallelism for the routed-expert layer: experts sharded over the ranks of one node.

The reference runs the layer on one device (it has no multi-GPU inference path); this module adds the sharding the
layer admits.  Rank r owns experts [r*E/G, (r+1)*E/G) and a batch of its own tokens.  One call:

1. routes its tokens (router GEMM + softmax/top-k, optionally with a per-expert logit bias that skews the load);
2. plans the dispatch: every (token, slot) pair goes to the rank that owns its expert; pairs are grouped by
   destination in ascending flat order (``send_pos`` = the pair's row in the send buffer);
3. quantises each token once (FP8, per-128-column scales) straight into its rows of the send buffer, and sends
   rows, scales and (local expert, routing weight) with NCCL all-to-all;
4. runs the local grouped GEMMs on what it received, producing one weighted bf16 row per received pair;
5. sends those rows back with the inverse all-to-all and sums each token's k rows in fixed slot order.

Every pair is computed exactly as on one GPU (the same quantised row, the same expert weights, rows independent of
their neighbours) and summed in the same order, so the result is bit-identical to the single-GPU layer.

The compute steps go through a backend object (:class:`CudaBackend` by default) so that the planning and exchange
logic can be exercised on CPU ranks (gloo) with a reference backend.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def plan_dispatch(ids: torch.Tensor, experts_per_rank: int, world: int):
    """ids [T, k] (global expert ids) -> send_pos [T*k] int32 (row of each flat pair in the send buffer),
    send_counts [world] int64, and the local expert id / destination of each send row."""
    flat = ids.reshape(-1).long()
    dest = torch.div(flat, experts_per_rank, rounding_mode="floor")
    order = torch.argsort(dest, stable=True)
    send_pos = torch.empty_like(order)
    send_pos[order] = torch.arange(order.numel(), device=order.device)
    send_counts = torch.bincount(dest, minlength=world)
    local_sorted = (flat[order] - dest[order] * experts_per_rank).to(torch.int32)
    return send_pos.to(torch.int32), send_counts, order, local_sorted


def _a2a(out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits, group):
    dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)
    return out


class CudaBackend:
    """The per-rank compute on the B200 kernels (FP8 experts)."""

    def __init__(self, w1, w1_s, w2, w2_s, router_w, top_k: int, bias=None):
        self.w1, self.w1_s, self.w2, self.w2_s = w1, w1_s, w2, w2_s
        self.router_w, self.top_k, self.bias = router_w, top_k, bias
        self.local_experts_n = w1.shape[0]

    def route(self, x):
        from . import ops

        _, w, ids = ops.router_topk(x, self.router_w, self.top_k, bias=self.bias)
        return w, ids

    def quant_dispatch(self, x, send_pos, k):
        from . import ops

        T = x.shape[0]
        return ops.quant_fp8(x, send_pos, k, T * k)

    def local_experts(self, rq, rs, re, rw):
        from . import ops

        N, H = rq.shape
        if N == 0:
            return torch.empty(0, H, dtype=torch.bfloat16, device=rq.device)
        s, eids, npp, _, slot_of, _ = ops.align(re.view(N, 1), self.local_experts_n)
        ms = s.numel()
        a_q = torch.empty(ms, H, dtype=torch.uint8, device=rq.device)
        a_s = torch.empty(ms, H // 128, dtype=torch.float32, device=rq.device)
        ops.scatter_rows(rq, slot_of, a_q)
        ops.scatter_rows(rs, slot_of, a_s)
        o_q, o_s, _ = ops.gemm1_fp8(a_q, a_s, self.w1, self.w1_s, eids, npp)
        c3, _ = ops.gemm2_fp8(o_q, o_s, self.w2, self.w2_s, eids, npp, s, rw, N, 1)
        return c3

    def combine(self, back, T, k, send_pos):
        from . import ops

        return ops.combine(back, T, k, row_of=send_pos)


class ExpertParallelLayer:
    """One routed-expert layer sharded over ``world`` ranks (this rank holds ``backend``'s experts)."""

    def __init__(self, backend, num_experts: int, top_k: int, rank: int, world: int, group=None):
        if num_experts % world:
            raise ValueError(f"{num_experts} experts do not split over {world} ranks")
        self.b, self.E, self.k, self.rank, self.world, self.group = backend, num_experts, top_k, rank, world, group
        self.epr = num_experts // world

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        k = self.k
        w, ids = self.b.route(x)
        send_pos, send_counts, order, local_sorted = plan_dispatch(ids, self.epr, self.world)
        q, s = self.b.quant_dispatch(x, send_pos, k)
        meta = torch.stack([local_sorted, w.reshape(-1)[order].contiguous().view(torch.int32)], 1).contiguous()
        if self.world == 1:
            rq, rs, rmeta = q, s, meta
            sc = rc = None
        else:
            counts_in = send_counts.to(x.device)
            counts_out = torch.empty_like(counts_in)
            dist.all_to_all_single(counts_out, counts_in, group=self.group)
            sc, rc = send_counts.tolist(), counts_out.tolist()
            n = int(sum(rc))
            rq = _a2a(torch.empty(n, H, dtype=q.dtype, device=x.device), q, rc, sc, self.group)
            rs = _a2a(torch.empty(n, s.shape[1], dtype=s.dtype, device=x.device), s, rc, sc, self.group)
            rmeta = _a2a(torch.empty(n, 2, dtype=meta.dtype, device=x.device), meta, rc, sc, self.group)
        re = rmeta[:, 0].contiguous()
        rw = rmeta[:, 1].contiguous().view(torch.float32)
        c3 = self.b.local_experts(rq, rs, re, rw)
        if self.world == 1:
            back = c3
        else:
            back = _a2a(torch.empty(T * k, H, dtype=c3.dtype, device=x.device), c3, sc, rc, self.group)
        return self.b.combine(back, T, k, send_pos)
