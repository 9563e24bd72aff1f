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

from typing import NamedTuple

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


class Plan(NamedTuple):
    """Where each (token, slot) pair goes: ``send_pos`` [T*k] int32 (its row of the send buffer), ``counts``
    [world] (rows of the send buffer for each destination rank, in rank order; padding rows included), ``rows``
    (allocated send-buffer rows) and ``meta`` [rows, 2] int32 per send row: the local expert id at the
    destination (-1 for a padding row) and the routing weight's fp32 bits."""

    send_pos: torch.Tensor
    counts: torch.Tensor
    rows: int
    meta: torch.Tensor


def plan_on_host_order(ids: torch.Tensor, w: torch.Tensor, experts_per_rank: int, world: int) -> Plan:
    """The plan from :func:`plan_dispatch` (unpadded; runs on any device, e.g. CPU ranks)."""
    send_pos, counts, order, local_sorted = plan_dispatch(ids, experts_per_rank, world)
    meta = torch.stack([local_sorted, w.reshape(-1)[order].contiguous().view(torch.int32)], 1).contiguous()
    return Plan(send_pos, counts, ids.numel(), meta)


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

    def plan(self, ids, w, experts_per_rank: int, world: int) -> Plan:
        """The dispatch plan on the GPU: the expert alignment run on the destination ranks (a stable counting sort
        of the pairs by rank, each rank's segment padded to 128 rows), then each send row's local expert and
        weight gathered from its pair."""
        from . import ops

        T, k = ids.shape
        n = T * k
        dest = torch.div(ids, experts_per_rank, rounding_mode="floor").to(torch.int32)
        srt, _, _, off, slot_of, _ = ops.align(dest, world)
        p = srt.long()
        valid = p < n
        pc = torch.where(valid, p, torch.zeros_like(p))
        local = torch.where(valid, ids.reshape(-1)[pc] - dest.reshape(-1)[pc] * experts_per_rank,
                            torch.full_like(pc, -1).to(ids.dtype))
        wv = torch.where(valid, w.reshape(-1)[pc], torch.zeros((), dtype=w.dtype, device=w.device))
        meta = torch.stack([local.to(torch.int32), wv.contiguous().view(torch.int32)], 1).contiguous()
        return Plan(slot_of, (off[1:] - off[:-1]).to(torch.int64), srt.numel(), meta)

    def quant_dispatch(self, x, send_pos, k, rows=None):
        from . import ops

        T = x.shape[0]
        return ops.quant_fp8(x, send_pos, k, T * k if rows is None else rows)

    def local_experts(self, rq, rs, re, rw):
        from . import ops

        N, H = rq.shape
        if N == 0:
            return torch.empty(0, H, dtype=torch.bfloat16, device=rq.device)
        # padding rows (local expert -1) keep slot -1 and are skipped by the row scatter and the GEMMs
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
        if hasattr(self.b, "plan"):
            plan = self.b.plan(ids, w, self.epr, self.world)
        else:
            plan = plan_on_host_order(ids, w, self.epr, self.world)
        q, s = self.b.quant_dispatch(x, plan.send_pos, k, plan.rows)
        if self.world == 1:
            n = int(plan.counts.sum())
            rq, rs, rmeta = q[:n], s[:n], plan.meta[:n]
            sc = rc = None
        else:
            counts_out = torch.empty_like(plan.counts)
            dist.all_to_all_single(counts_out, plan.counts, group=self.group)
            both = torch.cat([plan.counts, counts_out]).tolist()  # the one host synchronisation: split sizes
            sc, rc = both[: self.world], both[self.world:]
            ns, n = int(sum(sc)), int(sum(rc))
            rq = _a2a(torch.empty(n, H, dtype=q.dtype, device=x.device), q[:ns], rc, sc, self.group)
            rs = _a2a(torch.empty(n, s.shape[1], dtype=s.dtype, device=x.device), s[:ns], rc, sc, self.group)
            rmeta = _a2a(torch.empty(n, 2, dtype=plan.meta.dtype, device=x.device), plan.meta[:ns], rc, sc,
                         self.group)
        re = rmeta[:, 0].contiguous()
        rw = rmeta[:, 1].contiguous().view(torch.float32)
        c3 = self.b.local_experts(rq, rs, re, rw)
        if self.world == 1:
            back = c3
        else:
            back = _a2a(torch.empty(ns, H, dtype=c3.dtype, device=x.device), c3, sc, rc, self.group)
        return self.b.combine(back, T, k, plan.send_pos)


# ------------------------------------------------------------------------------------------- peer memory path
class _DeviceMemory:
    """A zero-copy view of raw device memory for torch (``__cuda_array_interface__``)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


def _view(ptr: int, nbytes: int, dev: torch.device) -> torch.Tensor:
    return torch.as_tensor(_DeviceMemory(ptr, nbytes), device=dev)


kMaxGroups = 4  # expert groups of the overlapped dispatch (one barrier counter each in the flag region)


def _align256(n: int) -> int:
    return (n + 255) // 256 * 256


class PeerExchange:
    """The peer-mapped region and local buffers of :class:`PeerExpertParallelLayer`, shareable by every layer of a
    stack with the same shapes (one layer runs at a time on a stream).

    Every rank allocates one region (count matrix, barrier counter, its experts' slot-ordered FP8 rows, scales,
    per-slot source and weight, and the result rows of its own pairs) and maps every other rank's region through
    CUDA IPC here (a host-side exchange of handles over ``group``), for up to ``max_tokens`` tokens per rank and
    call.  ``close()`` releases the mappings (all ranks call it together)."""

    def __init__(self, num_experts: int, top_k: int, hidden: int, intermediate: int, rank: int, world: int,
                 max_tokens: int, device: torch.device, group=None):
        from . import _lib

        if num_experts % world:
            raise ValueError(f"{num_experts} experts do not split over {world} ranks")
        self.E, self.k, self.rank, self.world, self.group = num_experts, top_k, rank, world, group
        self.epr = num_experts // world
        self.max_tokens, self.H, self.I, self.dev = max_tokens, hidden, intermediate, device
        G, E, k, H, I = world, num_experts, top_k, hidden, intermediate
        self.cap = (G * max_tokens * k + self.epr * 127 + 127) // 128 * 128
        cap = self.cap
        sizes = [("cm", G * E * 4), ("flag", 256), ("a1", cap * H), ("a1s", cap * (H // 128) * 4),
                 ("meta", cap * 4), ("wgt", cap * 4), ("back", max_tokens * k * H * 2)]
        self.off, total = {}, 0
        for name, n in sizes:
            self.off[name] = total
            total += _align256(n)
        own = _lib.ctypes.c_void_p()
        handle = (_lib.ctypes.c_ubyte * 64)()
        _lib.call("pm_ep_alloc", total, _lib.ctypes.byref(own), _lib.ctypes.addressof(handle))
        self._own = own.value
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        ptrs, self._opened = [], []
        for d in range(world):
            if d == rank:
                ptrs.append(self._own)
                continue
            p = _lib.ctypes.c_void_p()
            buf = (_lib.ctypes.c_ubyte * 64).from_buffer_copy(handles[d])
            _lib.call("pm_ep_open", _lib.ctypes.addressof(buf), _lib.ctypes.byref(p))
            ptrs.append(p.value)
            self._opened.append(p.value)
        mk = lambda name: torch.tensor([p + self.off[name] for p in ptrs], dtype=torch.int64, device=device)
        self.peer = {name: mk(name) for name, _ in sizes}
        region = _view(self._own, total, device)

        def own_view(name, dtype, shape):
            o, n = self.off[name], 1
            for s_ in shape:
                n *= s_
            nb = n * torch.tensor([], dtype=dtype).element_size()
            return region[o:o + nb].view(dtype).view(*shape)

        self.cm = own_view("cm", torch.int32, (G, E))
        self.flag = own_view("flag", torch.int32, (64,))
        self.a1 = own_view("a1", torch.uint8, (cap, H))
        self.a1s = own_view("a1s", torch.float32, (cap, H // 128))
        self.meta = own_view("meta", torch.int32, (cap,))
        self.wgt = own_view("wgt", torch.float32, (cap,))
        self.back = own_view("back", torch.bfloat16, (max_tokens * k, H))
        self.a2 = torch.empty(cap, I, dtype=torch.uint8, device=device)
        self.a2s = torch.empty(cap, I // 128, dtype=torch.float32, device=device)
        self.dst_rows = torch.zeros(cap, dtype=torch.int64, device=device)  # per slot: its source's result row
        self.base = torch.empty(E, dtype=torch.int32, device=device)
        self.eids = torch.zeros(cap // 128, dtype=torch.int32, device=device)
        self.npp = torch.zeros(1, dtype=torch.int32, device=device)
        self.err = torch.zeros(4, dtype=torch.int32, device=device)
        self.bounds = torch.zeros(kMaxGroups + 1, dtype=torch.int32, device=device)
        self.sms = torch.cuda.get_device_properties(device).multi_processor_count
        # four barrier counters, 64 bytes apart in the flag region: one per stream of barriers that may run at once
        self.peer_flag = [self.peer["flag"] + 64 * c for c in range(kMaxGroups)]
        self.epochs = [0] * kMaxGroups
        torch.cuda.synchronize(device)
        dist.barrier(group=group)  # every rank has mapped every region

    def barrier(self, stream: int, wait_limit_ns: int = 0, counter: int = 0) -> None:
        """Device barrier over the ranks (stream-ordered; the wait gives up after ``wait_limit_ns``, 0 = the
        library's 2 s, and then sets the error word).  Barriers on one counter pair up by count across the ranks;
        barriers that may run at the same time (on different streams) use different counters."""
        from . import _lib

        self.epochs[counter] += 1
        _lib.call("pm_ep_barrier", self.peer_flag[counter].data_ptr(), self.flag.data_ptr() + 64 * counter,
                  self.world, (self.epochs[counter] * self.world) & 0xFFFFFFFF, self.err.data_ptr(), wait_limit_ns,
                  stream)

    def errors(self) -> int:
        """Non-zero if any kernel gave up on a bounded wait or met an out-of-range slot (synchronises)."""
        return int(self.err.sum().item())

    def close(self) -> None:
        from . import _lib

        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)  # no rank still reads or writes a peer region
        for p in self._opened:
            _lib.call("pm_ep_close", p)
        self._opened = []
        if self._own:
            _lib.call("pm_ep_free", self._own)
            self._own = 0


class PeerExpertParallelLayer:
    """The expert-parallel layer with its exchanges done by the kernels themselves over NVLink peer memory
    (``pm_ep_*`` in the C ABI): no host synchronisation and no collective library on the data path.

    ``forward(x)`` for up to ``max_tokens`` tokens per rank: route; count pairs per expert into every rank's count
    matrix; barrier; offsets; quantise and store each token's rows into the owners' slots; barrier; local gate_up
    GEMM; down GEMM whose epilogue stores each weighted row straight into its source rank's result row; barrier;
    fixed-order combine.  Bit-identical to the
    single-GPU layer.  All ranks must call ``forward`` the same number of times (the barriers pair up by count).
    Give ``exchange`` to share one :class:`PeerExchange` among the layers of a stack; otherwise the layer makes
    its own, released by ``close()``."""

    def __init__(self, backend: CudaBackend, num_experts: int, top_k: int, rank: int, world: int,
                 max_tokens: int = 0, group=None, exchange: PeerExchange | None = None, groups: int | None = None,
                 reserve_sms: int = 16):
        """``groups`` (1-4, dividing the experts per rank): the owners' experts are dispatched in that many groups;
        group g + 1 is dispatched and its barrier passed on a side stream, on ``reserve_sms`` SMs, while the
        gate_up GEMM of group g runs on the others.  1 (the default): one dispatch, then the GEMMs.  Measured on two
        B200s the grouped form is slower: a dispatch kernel confined to a few SMs cannot keep its stores in flight,
        and one spread over the GPU holds the SMs the GEMM needs."""
        epr = num_experts // world
        if groups is None:
            groups = 1
        if not 1 <= groups <= kMaxGroups or epr % groups:
            raise ValueError(f"groups must be 1..{kMaxGroups} and divide the {epr} experts per rank")
        self.groups, self.reserve_sms = groups, reserve_sms
        self._side = None
        self.b, self.E, self.k, self.rank, self.world = backend, num_experts, top_k, rank, world
        _, I2, H = backend.w1.shape
        self._own_exchange = exchange is None
        self.x = exchange or PeerExchange(num_experts, top_k, H, I2 // 2, rank, world, max_tokens,
                                          backend.w1.device, group)
        if (self.x.E, self.x.k, self.x.H, self.x.I, self.x.world) != (num_experts, top_k, H, I2 // 2, world):
            raise ValueError("the exchange was made for another layer shape")

    PHASES = ("route", "count", "dispatch", "gate_up", "down", "combine")

    def forward(self, x: torch.Tensor, marks: list | None = None) -> torch.Tensor:
        """``marks`` (a list, optional): a CUDA event is recorded on the stream after each phase of :data:`PHASES`
        (preceded by one at the start) and appended, for per-phase device times; the work is unchanged."""
        from . import _lib, ops

        def mark():
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append(ev)

        mark()
        X = self.x
        T, H = x.shape
        if T > X.max_tokens or H != X.H:
            raise ValueError(f"x [{T}, {H}] exceeds the exchange's buffers ([{X.max_tokens}, {X.H}])")
        k, E, G = self.k, self.E, self.world
        P = lambda t: t.data_ptr()
        stream = torch.cuda.current_stream(X.dev).cuda_stream
        w, ids = self.b.route(x)
        _, _, _, off, slot_of, _ = ops.align(ids, E)  # own pairs by global expert: rank within the expert
        mark()
        X.meta.fill_(-1)
        _lib.call("pm_ep_count", P(ids), T * k, E, G, self.rank, P(X.peer["cm"]), stream)
        X.barrier(stream)
        mark()
        ng, epr = self.groups, X.epr
        _lib.call("pm_ep_offsets", P(X.cm), G, E, epr, self.rank, P(X.base), P(X.eids), P(X.npp), X.cap,
                  P(X.err), P(X.bounds), ng, stream)

        def dispatch(g, s_, max_sms):
            lo, hi = g * epr // ng, (g + 1) * epr // ng
            _lib.call("pm_ep_dispatch_quant", P(x), T, H, k, P(ids), P(w), P(slot_of), P(off), P(X.base), E, epr,
                      self.rank, X.cap, P(X.peer["a1"]), P(X.peer["a1s"]), P(X.peer["meta"]), P(X.peer["wgt"]),
                      P(X.err), lo, hi, max_sms, s_)

        def gate_up(g, max_sms):
            _lib.call("pm_ep_gemm1_fp8", P(X.a1), P(X.a1s), P(ops._u8(self.b.w1)), P(self.b.w1_s), P(X.eids),
                      P(X.bounds), g, X.cap, H, X.I, self.b.w1.shape[0], P(X.a2), P(X.a2s), P(X.err[1:2]), max_sms,
                      stream)

        dispatch(0, stream, 0)
        done = []
        if ng > 1:
            # groups 1.. are dispatched on a side stream (on reserve_sms SMs) while group 0's gate_up runs
            if self._side is None:
                self._side = torch.cuda.Stream(X.dev)
            side = self._side
            ev = torch.cuda.Event()
            ev.record()
            side.wait_event(ev)
            with torch.cuda.stream(side):
                for g in range(1, ng):
                    dispatch(g, side.cuda_stream, self.reserve_sms)
                    X.barrier(side.cuda_stream, counter=g)
                    d = torch.cuda.Event()
                    d.record(side)
                    done.append(d)
        X.barrier(stream)
        mark()
        for g in range(ng):
            if g > 0:
                torch.cuda.current_stream(X.dev).wait_event(done[g - 1])
            # while a later group is still being dispatched, leave reserve_sms SMs to its kernels
            gate_up(g, X.sms - self.reserve_sms if (g < ng - 1 and 0 < self.reserve_sms < X.sms) else 0)
        _lib.call("pm_ep_local_rows", P(X.meta), P(X.npp), X.cap, H, G, X.max_tokens * k, P(X.peer["back"]),
                  P(X.dst_rows), P(X.err), stream)
        mark()
        # the down GEMM stores each weighted row straight into its source rank's result row
        w2 = self.b.w2
        _lib.call("pm_ep_gemm2_fp8", P(X.a2), P(X.a2s), P(ops._u8(w2)), P(self.b.w2_s), P(X.eids), P(X.npp),
                  P(X.wgt), P(X.dst_rows), X.cap, H, X.I, w2.shape[0], P(X.err[2:3]), stream)
        X.barrier(stream)
        mark()
        out = ops.combine(X.back[: T * k], T, k)
        mark()
        return out

    def errors(self) -> int:
        return self.x.errors()

    def close(self) -> None:
        if self._own_exchange:
            self.x.close()
