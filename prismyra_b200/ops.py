"""Torch-facing calls into the C ABI: tensors in, tensors out, on the caller's current CUDA stream.

PyTorch is used for device memory and streams only; all arithmetic runs in ``libprismyra_moe.so``.  Each
function checks dtypes, shapes and devices before calling, so a wrong argument raises here rather than
inside a kernel.
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib

FP8 = torch.float8_e4m3fn
_NULL = None


def _p(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(dev: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _cuda(t: torch.Tensor, name: str, dtype, shape=None) -> None:
    _need(t.is_cuda, f"{name} must be a CUDA tensor")
    if isinstance(dtype, tuple):
        _need(t.dtype in dtype, f"{name} must have dtype in {dtype}, got {t.dtype}")
    else:
        _need(t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}")
    _need(t.is_contiguous(), f"{name} must be contiguous")
    if shape is not None:
        _need(tuple(t.shape) == tuple(shape), f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")


def _u8(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint8) if t.dtype != torch.uint8 else t


# ------------------------------------------------------------------------------------------- workspace
class WorkspacePool:
    """One scratch buffer per (device, calling thread, format), grown to the largest token count seen and never
    released.  A CUDA graph captured over a forward keeps the buffer's address, so a superseded buffer stays
    referenced for the life of the process instead of being returned to the allocator -- the same policy as the
    reference's per-thread NVFP4 workspace (prismyra/kernels/nvfp4.py:213-245)."""

    def __init__(self):
        self._bufs: dict = {}
        self._retired: list = []
        self._lock = threading.Lock()

    def get(self, device: torch.device, nbytes: int, fmt: int) -> torch.Tensor:
        key = (device.index, threading.get_ident(), fmt)
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                if buf is not None:
                    self._retired.append(buf)
                buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
                self._bufs[key] = buf
            return buf


POOL = WorkspacePool()


def workspace_for(x: torch.Tensor, T: int, H: int, I: int, E: int, k: int, fmt: int = _lib.FMT_FP8):
    n = _lib.workspace_bytes(T, H, I, E, k, fmt)
    _need(n > 0, f"unsupported MoE shape T={T} H={H} I={I} E={E} k={k}")
    return POOL.get(x.device, n, fmt), n


def region(ws: torch.Tensor, T, H, I, E, k, fmt, name: str, dtype, shape) -> torch.Tensor:
    """A typed view of one workspace region (for inspection of intermediates)."""
    off, n = _lib.workspace_region(T, H, I, E, k, fmt, name)
    numel = 1
    for s in shape:
        numel *= s
    elem = torch.tensor([], dtype=dtype).element_size()
    _need(numel * elem <= n, f"region {name} holds {n} bytes, asked for {numel * elem}")
    return ws[off: off + numel * elem].view(dtype).view(*shape)


# ------------------------------------------------------------------------------------------- the layer
#: Activation-scale rules of the FP8 quantisations (include/prismyra_moe.h, PM_FLAG_ACT_SCALE_*): "fp32" the correctly
#: rounded max(amax, 1e-10)/448 (vLLM's compiled quantiser, what the reference runs on a GPU); "ue8m0" that scale
#: rounded up to a power of two (vLLM with DeepGEMM E8M0 scales); "fp32_rcp" max(amax, 1e-10) * fl(1/448) (vLLM's
#: Triton quantiser).
ACT_SCALES = {"fp32": 0, "ue8m0": _lib.FLAG_ACT_SCALE_UE8M0, "fp32_rcp": _lib.FLAG_ACT_SCALE_RCP}


def forward_fp8(x: torch.Tensor, w1: torch.Tensor, w1_s: torch.Tensor, w2: torch.Tensor, w2_s: torch.Tensor,
                top_k: int, router_w: torch.Tensor | None = None, logits: torch.Tensor | None = None,
                out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                act_scale: str = "fp32", bias: torch.Tensor | None = None) -> torch.Tensor:
    """Routed FP8 experts for x [T, H] bf16; give ``router_w`` [E, H] bf16 or ``logits`` [T, E] bf16.
    ``act_scale`` picks the activation-scale rule (:data:`ACT_SCALES`): "fp32" (default) the correctly rounded
    max(amax, 1e-10)/448, as the reference's fused_experts computes on a GPU; "ue8m0" those scales rounded up to
    powers of two, as vLLM does when it runs DeepGEMM with E8M0 scales; "fp32_rcp" vLLM's Triton rule.  ``bias``
    (fp32 [E]) is added to every logit before the ranking (a benchmark's expert-load skew)."""
    _need(act_scale in ACT_SCALES, f"act_scale must be one of {sorted(ACT_SCALES)}")
    _need(x.dim() == 2, "x must be [T, H]")
    T, H = x.shape
    E, I2, H1 = w1.shape
    I = I2 // 2
    _cuda(x, "x", torch.bfloat16)
    _cuda(w1, "w1", (FP8, torch.uint8), (E, 2 * I, H))
    _cuda(w2, "w2", (FP8, torch.uint8), (E, H, I))
    _cuda(w1_s, "w1_s", torch.float32, (E, 2 * I // 128, H // 128))
    _cuda(w2_s, "w2_s", torch.float32, (E, H // 128, I // 128))
    _need(router_w is not None or logits is not None, "give router_w or logits")
    if logits is not None:
        _cuda(logits, "logits", torch.bfloat16, (T, E))
    else:
        _cuda(router_w, "router_w", torch.bfloat16, (E, H))
    if bias is not None:
        _cuda(bias, "bias", torch.float32, (E,))
    if out is None:
        out = torch.empty_like(x)
    _cuda(out, "out", torch.bfloat16, (T, H))
    if T == 0:
        return out
    if workspace is None:
        workspace, nbytes = workspace_for(x, T, H, I, E, top_k, _lib.FMT_FP8)
    else:
        nbytes = workspace.numel()
    _lib.call(
        "pm_moe_forward_fp8_ex", _p(x), _p(router_w), _p(logits), _p(bias), _p(_u8(w1)), _p(w1_s), _p(_u8(w2)),
        _p(w2_s),
        T, H, I, E, top_k, ACT_SCALES[act_scale], _p(out), _p(workspace), nbytes, _stream(x.device),
    )
    return out


def _shared_checks(x, w_sg, w13, w13_s, w2, w2_s):
    T, H = x.shape
    I2s = w13.shape[0]
    Is = I2s // 2
    _cuda(w_sg, "w_sg", torch.bfloat16)
    _need(w_sg.numel() == H, f"w_sg must hold H={H} values")
    _cuda(w13, "w13", (FP8, torch.uint8), (2 * Is, H))
    _cuda(w13_s, "w13_s", torch.float32, (2 * Is // 128, H // 128))
    _cuda(w2, "w2", (FP8, torch.uint8), (H, Is))
    _cuda(w2_s, "w2_s", torch.float32, (H // 128, Is // 128))
    return T, H, Is


def fp8_linear(x: torch.Tensor, w: torch.Tensor, w_s: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """A dense block-FP8 projection x [..., K] bf16 -> [..., N] bf16 with w e4m3 [N, K] and fp32 block multipliers
    [N/128, K/128] (the reference's Fp8Linear, qwen3_moe.py:211-230)."""
    _cuda(x, "x", torch.bfloat16)
    N, K = w.shape
    _need(x.shape[-1] == K, f"x must end in K={K}")
    _cuda(w, "w", (FP8, torch.uint8), (N, K))
    _cuda(w_s, "w_s", torch.float32, (N // 128, K // 128))
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    T = x2.shape[0]
    if out is None:
        out = torch.empty(*lead, N, dtype=torch.bfloat16, device=x.device)
    _cuda(out, "out", torch.bfloat16)
    _need(out.numel() == T * N, f"out must hold {T} x {N} values")
    if T == 0:
        return out
    n = _lib.load().pm_fp8_linear_workspace_bytes(T, K, N)
    _need(n > 0, f"unsupported projection shape T={T} K={K} N={N} (need K % 128 == 0, N % 256 == 0)")
    ws = POOL.get(x.device, n, "dense")
    _lib.call("pm_fp8_linear", _p(x2), _p(_u8(w)), _p(w_s), T, K, N, _p(out), _p(ws), n, _stream(x.device))
    return out


def shared_fp8(x: torch.Tensor, w_sg: torch.Tensor, w13: torch.Tensor, w13_s: torch.Tensor, w2: torch.Tensor,
               w2_s: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """The shared expert on block-FP8 weights: sigmoid(x . w_sg) * down(silu(gate x) * up x) -> bf16 [T, H]
    (reference qwen3_moe.py:198); w13 = gate_proj rows then up_proj rows [2 Is, H]."""
    _need(x.dim() == 2, "x must be [T, H]")
    _cuda(x, "x", torch.bfloat16)
    T, H, Is = _shared_checks(x, w_sg, w13, w13_s, w2, w2_s)
    if out is None:
        out = torch.empty_like(x)
    _cuda(out, "out", torch.bfloat16, (T, H))
    if T == 0:
        return out
    n = _lib.load().pm_moe_shared_workspace_bytes(T, H, Is)
    _need(n > 0, f"unsupported shared-expert shape T={T} H={H} Is={Is}")
    ws = POOL.get(x.device, n, "shared")
    _lib.call("pm_moe_shared_fp8", _p(x), _p(w_sg), _p(_u8(w13)), _p(w13_s), _p(_u8(w2)), _p(w2_s), T, H, Is,
              _p(out), _p(ws), n, _stream(x.device))
    return out


def block_fp8(x: torch.Tensor, w1: torch.Tensor, w1_s: torch.Tensor, w2: torch.Tensor, w2_s: torch.Tensor,
              top_k: int, w_sg: torch.Tensor, sw13: torch.Tensor, sw13_s: torch.Tensor, sw2: torch.Tensor,
              sw2_s: torch.Tensor, router_w: torch.Tensor | None = None, logits: torch.Tensor | None = None,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """Routed experts plus the shared expert, summed as two bf16 tensors: the whole FusedExperts.forward
    (reference qwen3_moe.py:184-199) in one library call."""
    _need(x.dim() == 2, "x must be [T, H]")
    _cuda(x, "x", torch.bfloat16)
    T, H = x.shape
    E, I2, _ = w1.shape
    I = I2 // 2
    _cuda(w1, "w1", (FP8, torch.uint8), (E, 2 * I, H))
    _cuda(w2, "w2", (FP8, torch.uint8), (E, H, I))
    _cuda(w1_s, "w1_s", torch.float32, (E, 2 * I // 128, H // 128))
    _cuda(w2_s, "w2_s", torch.float32, (E, H // 128, I // 128))
    _, _, Is = _shared_checks(x, w_sg, sw13, sw13_s, sw2, sw2_s)
    _need(router_w is not None or logits is not None, "give router_w or logits")
    if logits is not None:
        _cuda(logits, "logits", torch.bfloat16, (T, E))
    else:
        _cuda(router_w, "router_w", torch.bfloat16, (E, H))
    if out is None:
        out = torch.empty_like(x)
    _cuda(out, "out", torch.bfloat16, (T, H))
    if T == 0:
        return out
    n = _lib.load().pm_moe_block_workspace_bytes(T, H, I, Is, E, top_k)
    _need(n > 0, f"unsupported MoE block shape T={T} H={H} I={I} Is={Is} E={E} k={top_k}")
    ws = POOL.get(x.device, n, "block")
    _lib.call("pm_moe_block_fp8", _p(x), _p(router_w), _p(logits), _p(_u8(w1)), _p(w1_s), _p(_u8(w2)), _p(w2_s),
              _p(w_sg), _p(_u8(sw13)), _p(sw13_s), _p(_u8(sw2)), _p(sw2_s), T, H, I, Is, E, top_k, _p(out), _p(ws),
              n, _stream(x.device))
    return out


class _HostPipe:
    """Per-(device, thread) copy streams and two sets of device row buffers for the host-to-host calls (grow-only,
    never freed, so addresses stay stable across calls).  Calls alternate between the two sets, so that one call's
    upload can run while the previous call's layer and download are still in flight; each set carries the events
    after which its input rows may be overwritten (its layer has read them) and its output rows may be overwritten
    (its download has read them).

    Growing replaces both sets.  The superseded buffers may still be read or written by copies queued on the upload
    and download streams (and by the layer on the caller's stream), so they are retired -- kept referenced for the
    life of the process, never handed back to the caching allocator -- rather than dropped: no later allocation on
    any stream can reuse their memory while those copies run."""

    def __init__(self):
        self._lock = threading.Lock()
        self._state = {}
        self._retired: list = []

    def get(self, device: torch.device, T: int, H: int):
        key = (device.index, threading.get_ident())
        with self._lock:
            st = self._state.get(key)
            if st is None:
                st = {"h2d": torch.cuda.Stream(device), "d2h": torch.cuda.Stream(device), "rows": 0, "H": H,
                      "next": 0, "sets": [{}, {}]}
                self._state[key] = st
            if st["rows"] < T or st["H"] != H:
                for bs in st["sets"]:
                    self._retired.extend(bs[name] for name in ("x", "out") if name in bs)
                    bs.clear()
                    bs["x"] = torch.empty(T, H, dtype=torch.bfloat16, device=device)
                    bs["out"] = torch.empty(T, H, dtype=torch.bfloat16, device=device)
                st["rows"], st["H"] = T, H
            bs = st["sets"][st["next"]]
            st["next"] ^= 1
            return st, bs


_PIPE = _HostPipe()


def host_chunks(T: int, edge_rows: int = 1024) -> list[tuple[int, int]]:
    """Row ranges of :func:`forward_fp8_host`: a short first chunk (its upload is the only copy the GPU waits for),
    one long middle chunk whose compute covers the long copies in both directions, and a short last chunk (its
    download is the only copy left after the compute).  Every chunk streams all expert weights once, so there are
    no more than three (at T=5120 on a B200 over PCIe 1024-row edges measured best: 0.96 ms per call against
    1.17 ms for one upload, layer and download in series)."""
    if T <= 4 * edge_rows:
        return [(0, T)]
    return [(0, edge_rows), (edge_rows, T - edge_rows), (T - edge_rows, T)]


def _host_args(x_host, out_host):
    _need(x_host.dim() == 2 and x_host.dtype == torch.bfloat16 and x_host.device.type == "cpu",
          "x_host must be a host bf16 [T, H] tensor")
    T, H = x_host.shape
    if out_host is None:
        out_host = torch.empty(T, H, dtype=torch.bfloat16, pin_memory=True)
    _need(tuple(out_host.shape) == (T, H) and out_host.dtype == torch.bfloat16 and out_host.device.type == "cpu",
          "out_host must be a host bf16 [T, H] tensor")
    return T, H, out_host


def host_async(fn, x_host: torch.Tensor, out_host: torch.Tensor | None = None,
               chunks: list[tuple[int, int]] | None = None, device: torch.device | None = None):
    """Run a device function over a host-resident batch: upload x_host [T, H] bf16 (pinned) on this thread's upload
    stream, call ``fn(x_rows, out_rows)`` on the caller's current stream (it returns the result rows: ``out_rows``
    itself or a tensor of its own), download on the download stream, and return (out_host, done): done is a CUDA
    event after which ``out_host`` holds the result.  Calls alternate between two device buffer sets, so
    consecutive calls overlap: a call's upload runs during the previous call's ``fn``, its download during the
    next call's.  ``chunks`` (row ranges covering [0, T) in order, default one) splits a call into pieces whose
    copies overlap its own ``fn``; use it only for a row-wise ``fn``.  Every rank of an expert-parallel layer calls
    this the same number of times, like the layer itself."""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    T, H, out_host = _host_args(x_host, out_host)
    done = torch.cuda.Event()
    comp = torch.cuda.current_stream(dev)
    if T == 0:
        done.record(comp)
        return out_host, done
    st, bs = _PIPE.get(dev, T, H)
    if "x_free" in bs:
        st["h2d"].wait_event(bs["x_free"])   # this set's input rows: read by its previous call
    if "out_free" in bs:
        comp.wait_event(bs["out_free"])      # this set's output rows: read by its previous download
    for r0, r1 in (chunks or [(0, T)]):
        xs, os_ = bs["x"][r0:r1], bs["out"][r0:r1]
        with torch.cuda.stream(st["h2d"]):
            xs.copy_(x_host[r0:r1], non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(st["h2d"])
        comp.wait_event(ready)
        res = fn(xs, os_)
        computed = torch.cuda.Event()
        computed.record(comp)
        st["d2h"].wait_event(computed)
        if res.data_ptr() != os_.data_ptr():
            res.record_stream(st["d2h"])     # a tensor of fn's own: kept until its download has read it
        with torch.cuda.stream(st["d2h"]):
            out_host[r0:r1].copy_(res, non_blocking=True)
    x_free = torch.cuda.Event()
    x_free.record(comp)
    done.record(st["d2h"])
    bs["x_free"], bs["out_free"] = x_free, done
    return out_host, done


def forward_fp8_host_async(x_host: torch.Tensor, w1: torch.Tensor, w1_s: torch.Tensor, w2: torch.Tensor,
                           w2_s: torch.Tensor, top_k: int, router_w: torch.Tensor,
                           out_host: torch.Tensor | None = None, chunks: list[tuple[int, int]] | None = None):
    """The routed FP8 experts for a host-resident x [T, H] bf16 through :func:`host_async`: returns (out_host,
    done), consecutive calls overlapping.  Every row's result equals :func:`forward_fp8` on the whole batch (rows
    are independent, and the layer's launch shapes agree bit for bit)."""
    def fn(xs, os_):
        return forward_fp8(xs, w1, w1_s, w2, w2_s, top_k, router_w=router_w, out=os_)

    return host_async(fn, x_host, out_host, chunks, device=w1.device)


def forward_fp8_host(x_host: torch.Tensor, w1: torch.Tensor, w1_s: torch.Tensor, w2: torch.Tensor,
                     w2_s: torch.Tensor, top_k: int, router_w: torch.Tensor, out_host: torch.Tensor | None = None,
                     edge_rows: int = 1024) -> torch.Tensor:
    """The routed FP8 experts for a host-resident x [T, H] bf16 (pinned, so the copies overlap): rows go to the GPU,
    through :func:`forward_fp8` and back in the chunks of :func:`host_chunks`, with the host-to-device copies, the
    layer and the device-to-host copies on three streams so that both PCIe directions overlap the compute.  Ordered
    on the caller's current stream: returns once the work is queued; ``out_host`` [T, H] (pinned bf16) holds the
    result when that stream has reached this point.  For a stream of batches, :func:`forward_fp8_host_async`
    overlaps consecutive calls instead."""
    T, H, out_host = _host_args(x_host, out_host)
    out_host, done = forward_fp8_host_async(x_host, w1, w1_s, w2, w2_s, top_k, router_w, out_host,
                                            chunks=host_chunks(T, edge_rows))
    torch.cuda.current_stream(w1.device).wait_event(done)
    return out_host


def read_status(workspace: torch.Tensor) -> None:
    """Synchronise and raise if a kernel of the last forward on this workspace gave up on a bounded wait."""
    _lib.call("pm_moe_read_status", _p(workspace), _stream(workspace.device))


# ------------------------------------------------------------------------------------------- stages
def router_topk(x: torch.Tensor, router_w: torch.Tensor, k: int, out=None, bias: torch.Tensor | None = None):
    T, H = x.shape
    E = router_w.shape[0]
    _cuda(x, "x", torch.bfloat16)
    _cuda(router_w, "router_w", torch.bfloat16, (E, H))
    if out is None:
        out = (torch.empty(T, E, dtype=torch.bfloat16, device=x.device),
               torch.empty(T, k, dtype=torch.float32, device=x.device),
               torch.empty(T, k, dtype=torch.int32, device=x.device))
    logits, w, ids = out
    if bias is not None:
        _cuda(bias, "bias", torch.float32, (E,))
    _lib.call("pm_moe_router_topk", _p(x), _p(router_w), _p(bias), T, H, E, k, _p(logits), _p(w), _p(ids),
              _stream(x.device))
    return logits, w, ids


def topk(logits: torch.Tensor, k: int, bias: torch.Tensor | None = None):
    T, E = logits.shape
    _cuda(logits, "logits", torch.bfloat16)
    if bias is not None:
        _cuda(bias, "bias", torch.float32, (E,))
    w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    _lib.call("pm_moe_topk", _p(logits), _p(bias), T, E, k, _p(w), _p(ids), _stream(logits.device))
    return w, ids


def align(ids: torch.Tensor, E: int, out=None):
    """-> sorted_ids [max_slots], expert_ids [max_slots/128], num_post_pad [1], expert_off [E+1],
    slot_of [T*k] and the per-chunk count scratch."""
    _cuda(ids, "ids", torch.int32)
    T, k = ids.shape
    ms = _lib.max_slots(T, E, k)
    dev = ids.device
    if out is None:
        out = (torch.full((ms,), -1, dtype=torch.int32, device=dev),
               torch.full((ms // 128,), -1, dtype=torch.int32, device=dev),
               torch.zeros(1, dtype=torch.int32, device=dev), torch.zeros(E + 1, dtype=torch.int32, device=dev),
               torch.full((T * k,), -1, dtype=torch.int32, device=dev),  # stays -1 for ids outside [0, E)
               torch.zeros(_lib.align_workspace_bytes(T, k, E) // 4, dtype=torch.int32, device=dev))
    sorted_ids, expert_ids, npp, off, slot_of, scratch = out
    _lib.call("pm_moe_align", _p(ids), T, k, E, _p(sorted_ids), _p(expert_ids), _p(npp), _p(off), _p(slot_of),
              _p(scratch), scratch.numel() * 4, _stream(dev))
    return sorted_ids, expert_ids, npp, off, slot_of, scratch


def scatter_rows(src: torch.Tensor, dst_index: torch.Tensor, dst: torch.Tensor) -> torch.Tensor:
    """dst[dst_index[i]] = src[i] for 2-D tensors whose rows are multiples of 16 bytes (strided views allowed)."""
    _cuda(dst_index, "dst_index", torch.int32)
    rows = src.shape[0]
    rb = src.shape[1] * src.element_size()
    _need(dst.shape[1] * dst.element_size() == rb, "row sizes differ")
    _need(src.stride(1) == 1 and dst.stride(1) == 1, "rows must be contiguous")
    _lib.call("pm_moe_scatter_rows", _p(src), rows, rb, src.stride(0) * src.element_size(), _p(dst_index), _p(dst),
              dst.stride(0) * dst.element_size(), _stream(src.device))
    return dst


def quant_fp8(x: torch.Tensor, slot_of: torch.Tensor | None = None, k: int = 1, max_slots: int = 0, out=None,
              act_scale: str = "fp32"):
    """Per-token, per-128-column e4m3 quantisation of x [T, H] bf16.  Without ``slot_of``: (x_q [T, H] u8,
    x_s [T, H/128] f32).  With it: the rows land in the k slots of each token (a_q [max_slots, H], a_s).
    ``act_scale`` as in :func:`forward_fp8`."""
    _need(act_scale in ACT_SCALES, f"act_scale must be one of {sorted(ACT_SCALES)}")
    T, H = x.shape
    _cuda(x, "x", torch.bfloat16)
    rows = T if slot_of is None else max_slots
    if out is None:
        out = (torch.zeros(rows, H, dtype=torch.uint8, device=x.device),
               torch.zeros(rows, H // 128, dtype=torch.float32, device=x.device))
    x_q, x_s = out
    _lib.call("pm_moe_quant_fp8_ex", _p(x), T, H, k, _p(slot_of), _p(x_q), _p(x_s), ACT_SCALES[act_scale],
              _stream(x.device))
    return x_q, x_s


def gemm1_fp8(a_q, a_s, w1, w1_s, expert_ids, npp, out=None):
    """gate_up GEMM over expert-ordered slots (a_q [max_slots, H], a_s [max_slots, H/128])."""
    ms, H = a_q.shape
    E, I2, _ = w1.shape
    I = I2 // 2
    if out is None:
        out = (torch.zeros(ms, I, dtype=torch.uint8, device=a_q.device),
               torch.zeros(ms, I // 128, dtype=torch.float32, device=a_q.device),
               torch.zeros(1, dtype=torch.int32, device=a_q.device))
    out_q, out_s, err = out
    _lib.call("pm_moe_gemm1_fp8", _p(a_q), _p(a_s), _p(_u8(w1)), _p(w1_s), _p(expert_ids), _p(npp), ms, H, I, E,
              _p(out_q), _p(out_s), _p(err), _stream(a_q.device))
    return out_q, out_s, err


def gemm2_fp8(a_q, a_s, w2, w2_s, expert_ids, npp, sorted_ids, topk_w, T: int, k: int, out=None):
    ms, I = a_q.shape
    E, H, _ = w2.shape
    if out is None:
        out = (torch.zeros(T * k, H, dtype=torch.bfloat16, device=a_q.device),
               torch.zeros(1, dtype=torch.int32, device=a_q.device))
    c3, err = out
    _lib.call("pm_moe_gemm2_fp8", _p(a_q), _p(a_s), _p(_u8(w2)), _p(w2_s), _p(expert_ids), _p(npp),
              _p(sorted_ids), _p(topk_w), ms, T, k, H, I, E, _p(c3), _p(err), _stream(a_q.device))
    return c3, err


def combine(c3: torch.Tensor, T: int, k: int, out=None, row_of: torch.Tensor | None = None):
    H = c3.shape[1]
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=c3.device)
    _lib.call("pm_moe_combine", _p(c3), _p(row_of), T, k, H, _p(out), _stream(c3.device))
    return out


# ------------------------------------------------------------------------------------------- NVFP4
def forward_nvfp4(x: torch.Tensor, w1: torch.Tensor, w1_sf: torch.Tensor, alpha1: torch.Tensor, a1_gs: float,
                  w2: torch.Tensor, w2_sf: torch.Tensor, alpha2: torch.Tensor, a2_gs: float, top_k: int,
                  router_w: torch.Tensor | None = None, logits: torch.Tensor | None = None,
                  out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Routed NVFP4 experts for x [T, H] bf16.  w1 u8 [E, 2I, H/2], w1_sf blocked [E, 2I/128, H/64, 512],
    w2 u8 [E, H, I/2], w2_sf blocked [E, H/128, I/64, 512], alphas f32 [E]."""
    _need(x.dim() == 2, "x must be [T, H]")
    T, H = x.shape
    E, I2, _ = w1.shape
    I = I2 // 2
    _cuda(x, "x", torch.bfloat16)
    _cuda(w1, "w1", torch.uint8, (E, 2 * I, H // 2))
    _cuda(w2, "w2", torch.uint8, (E, H, I // 2))
    _cuda(w1_sf, "w1_sf", torch.uint8, (E, 2 * I // 128, H // 64, 512))
    _cuda(w2_sf, "w2_sf", torch.uint8, (E, H // 128, I // 64, 512))
    _cuda(alpha1, "alpha1", torch.float32, (E,))
    _cuda(alpha2, "alpha2", torch.float32, (E,))
    _need(router_w is not None or logits is not None, "give router_w or logits")
    if logits is not None:
        _cuda(logits, "logits", torch.bfloat16, (T, E))
    else:
        _cuda(router_w, "router_w", torch.bfloat16, (E, H))
    if out is None:
        out = torch.empty_like(x)
    if T == 0:
        return out
    if workspace is None:
        workspace, nbytes = workspace_for(x, T, H, I, E, top_k, _lib.FMT_NVFP4)
    else:
        nbytes = workspace.numel()
    _lib.call(
        "pm_moe_forward_nvfp4", _p(x), _p(router_w), _p(logits), _p(w1), _p(w1_sf), _p(alpha1),
        ctypes.c_float(a1_gs), _p(w2), _p(w2_sf), _p(alpha2), ctypes.c_float(a2_gs), T, H, I, E, top_k, _p(out),
        _p(workspace), nbytes, _stream(x.device),
    )
    return out


def quant_nvfp4(x: torch.Tensor, gs: float, slot_of: torch.Tensor | None = None, k: int = 1, max_slots: int = 0,
                out=None):
    """NVFP4 quantisation of x [T, H] bf16 -> (packed [rows, H/2] u8, blocked scales [rows/128, H/64, 512] u8);
    rows = T (slot_of None, T padded up to 128 for the scale blocks) or max_slots."""
    T, H = x.shape
    _cuda(x, "x", torch.bfloat16)
    rows = T if slot_of is None else max_slots
    rb = -(-rows // 128)
    if out is None:
        out = (torch.zeros(rows, H // 2, dtype=torch.uint8, device=x.device),
               torch.zeros(rb, H // 64, 512, dtype=torch.uint8, device=x.device))
    q, sf = out
    _lib.call("pm_moe_quant_nvfp4", _p(x), T, H, k, _p(slot_of), ctypes.c_float(gs), _p(q), _p(sf),
              _stream(x.device))
    return q, sf


def gemm1_nvfp4(a_q, a_sf, w1, w1_sf, alpha1, a2_gs: float, expert_ids, npp, out=None):
    ms, H2 = a_q.shape
    H = 2 * H2
    E, I2, _ = w1.shape
    I = I2 // 2
    if out is None:
        out = (torch.zeros(ms, I // 2, dtype=torch.uint8, device=a_q.device),
               torch.zeros(ms // 128, I // 64, 512, dtype=torch.uint8, device=a_q.device),
               torch.zeros(1, dtype=torch.int32, device=a_q.device))
    oq, osf, err = out
    _lib.call("pm_moe_gemm1_nvfp4", _p(a_q), _p(a_sf), _p(w1), _p(w1_sf), _p(alpha1), ctypes.c_float(a2_gs),
              _p(expert_ids), _p(npp), ms, H, I, E, _p(oq), _p(osf), _p(err), _stream(a_q.device))
    return oq, osf, err


def gemm2_nvfp4(a_q, a_sf, w2, w2_sf, alpha2, expert_ids, npp, sorted_ids, topk_w, T: int, k: int, out=None):
    ms, I2 = a_q.shape
    I = 2 * I2
    E, H, _ = w2.shape
    if out is None:
        out = (torch.zeros(T * k, H, dtype=torch.bfloat16, device=a_q.device),
               torch.zeros(1, dtype=torch.int32, device=a_q.device))
    c3, err = out
    _lib.call("pm_moe_gemm2_nvfp4", _p(a_q), _p(a_sf), _p(w2), _p(w2_sf), _p(alpha2), _p(expert_ids), _p(npp),
              _p(sorted_ids), _p(topk_w), ms, T, k, H, I, E, _p(c3), _p(err), _stream(a_q.device))
    return c3, err


def nvfp4_prepare(w: torch.Tensor, s: torch.Tensor, importance: torch.Tensor | None = None, search: bool = False):
    """FP8 expert stack -> NVFP4 on the GPU: w e4m3 (or its bytes) [E, R, C], s fp32 [E, R/128, C/128] ->
    (packed u8 [E, R, C/2], row-major e4m3 scales [E, R, C/16], g fp32 [E]); bit for bit the reference's
    prepare_layer arithmetic (prismyra/kernels/nvfp4.py:315-331).  With ``importance`` (fp32 [E, C] per input
    column) or ``search``, each 16-group's scale comes from the importance search (quantize_search,
    nvfp4.py:57-94; without importance every column weighs 1)."""
    _cuda(w, "w", (torch.float8_e4m3fn, torch.uint8))
    _need(w.dim() == 3, "w must be [E, R, C]")
    E, R, C = w.shape
    _cuda(s, "s", torch.float32, (E, R // 128, C // 128))
    if importance is not None:
        _cuda(importance, "importance", torch.float32, (E, C))
    packed = torch.empty(E, R, C // 2, dtype=torch.uint8, device=w.device)
    scales = torch.empty(E, R, C // 16, dtype=torch.float8_e4m3fn, device=w.device)
    g = torch.empty(E, dtype=torch.float32, device=w.device)
    if importance is not None or search:
        _lib.call("pm_nvfp4_prepare_search", _p(w), _p(s), _p(importance), E, R, C, _p(packed), _p(scales), _p(g),
                  _stream(w.device))
    else:
        _lib.call("pm_nvfp4_prepare", _p(w), _p(s), E, R, C, _p(packed), _p(scales), _p(g), _stream(w.device))
    return packed, scales, g
