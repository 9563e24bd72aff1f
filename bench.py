"""Benchmark of the B200 routed-expert MoE layer (BASELINE metric: MoE-layer tokens/s and % of FP8 tensor peak at
T=5120; HBM GB/s at T=128).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step = one call of the routed FP8 layer (router projection, softmax/top-k, expert alignment, activation
quantisation, gate_up GEMM + silu*mul + requantisation, down GEMM + routing weight, top-k sum) on T=5120 tokens
of H=2048 with E=128 experts, top-8, I=768, synthetic seeded data, expert weights 128x128
block-FP8.  The weights (604 MB) exceed the 126 MB L2, so every step streams them from HBM; no L2 flush is added.
Under torchrun (N GPUs) the step is the expert-parallel layer: every rank owns E/N experts and its own 5120
tokens (weak scaling); the kernels move the rows themselves over NVLink (the dispatching quantisation stores each
token's rows into the owners' expert slots, the down GEMM's epilogue stores each weighted row back into its source
rank's result row, device barriers between the phases; no collective library on the data path); the step time is
the max over ranks.

``--impl reference`` times the reference's own CPU implementation of the same layer (transformers' fallback
block, float32 -- the engine's CPU dtype -- and bfloat16, all host threads, median of >= 5 calls after 2 warm-ups)
on a bounded sample of the same seeded workload and prints the same JSON line with ``"impl": "reference"``.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer tokens/s and % FP8/FP4 tensor peak at T=5120; HBM GB/s at T=128"
H, I, E, K = 2048, 768, 128, 8
T_CTX, T_BRANCH, T_CPU_SAMPLE = 5120, 128, 512
KERNELS_PER_STEP = 8  # router GEMM, top-k, 2 alignment passes, activation quant, gate_up, down, combine
# expert parallel over peer memory: router GEMM, top-k, 2 alignment passes, count, 3 barriers, offsets, dispatching
# quant, slot map, gate_up, down, return, combine
KERNELS_PER_EP_STEP = 16


def profile_traffic(kernel: str):
    """DRAM read + write bytes per launch of ``kernel`` ("gate_up") from the committed ncu summary of the T=5120
    workload (the line ``traffic_bytes_per_launch <kernel>: <bytes>``), or None without one."""
    try:
        with open(ROOT / "profiles" / "gemm_fp8_t5120.md") as f:
            for line in f:
                if line.startswith(f"traffic_bytes_per_launch {kernel}:"):
                    return int(line.split(":", 1)[1].strip())
    except (OSError, ValueError):
        pass
    return None


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def dist_init():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws == 1:
        return 0, 1, 0
    import datetime

    import torch
    import torch.distributed as dist

    rank, local = int(os.environ["RANK"]), int(os.environ.get("LOCAL_RANK", "0"))
    os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep NCCL's banner off stdout: the JSON line is the output
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return rank, ws, local


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons, running from before the warm-up until after the
    timed region; summary() keeps the samples taken inside [mark_start, mark_end] (host time), or the nearest
    one when the timed region is shorter than the sampling interval."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.rows: list = []
        self.t0 = self.t1 = None

    def _reader(self):
        for ln in self.proc.stdout:
            f = [x.strip() for x in ln.split(",")]
            if len(f) >= 7:
                try:
                    self.rows.append((time.time(), float(f[0]), float(f[1]), float(f[2]), f[3:7]))
                except ValueError:
                    pass

    def start(self):
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return self
        threading.Thread(target=self._reader, daemon=True).start()
        t = time.time()
        while not self.rows and time.time() - t < 10:
            time.sleep(0.02)
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()
        t = time.time()
        while self.proc is not None and not any(r[0] > self.t1 for r in self.rows) and time.time() - t < 2:
            time.sleep(0.02)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if not self.rows or self.t0 is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        inside = [r for r in self.rows if self.t0 - 0.05 <= r[0] <= self.t1 + 0.05]
        if not inside:
            mid = 0.5 * (self.t0 + self.t1)
            inside = [min(self.rows, key=lambda r: abs(r[0] - mid))]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in inside for i, v in enumerate(r[4]) if v.lower().startswith("active")})
        mhz = sorted(r[1] for r in inside)
        return {"sm_mhz": mhz[len(mhz) // 2], "sm_max_mhz": max(r[2] for r in inside), "reasons": reasons,
                "samples": len(inside), "power_w_max": max(r[3] for r in inside)}


def cpu_baseline(layer_cpu: dict, max_seconds: float = 12.0) -> dict:
    """The reference's CPU fallback (transformers block) on a 512-token sample of the workload, in float32 (the
    engine's CPU dtype: the reported value) and in bfloat16; median of >= 5 calls after 2 warm-ups each."""
    import torch

    from oracle import torch_fallback
    from prismyra_b200 import synth

    w1 = synth.dequantize_fp8_blocks(layer_cpu["w1"], layer_cpu["w1_s"])
    w2 = synth.dequantize_fp8_blocks(layer_cpu["w2"], layer_cpu["w2_s"])
    res = {}
    for dt in (torch.float32, torch.bfloat16):
        router, experts = torch_fallback.build_block(layer_cpu["router_w"].float(), w1, w2, K, dtype=dt)
        x = layer_cpu["x"][:T_CPU_SAMPLE].to(dt)
        res[dt] = torch_fallback.time_routed(router, experts, x, max_seconds=max_seconds)
        del router, experts
    del w1, w2
    r, rb = res[torch.float32], res[torch.bfloat16]
    return {"value": r["tokens_per_s"], "unit": "tokens/s", "cores": r["threads"], "kind": "reference",
            "sample": f"{T_CPU_SAMPLE} of the {T_CTX} tokens (the same seeded tensors as the GPU arm), median of "
                      f"{r['calls']} calls after {r['warmup']} warm-ups: transformers Qwen3_5MoeTopKRouter + "
                      "Qwen3_5MoeExperts (the reference's CPU fallback) in float32 on dequantised FP8 weights",
            "bf16_tokens_per_s": rb["tokens_per_s"], "bf16_calls": rb["calls"],
            "cpu_model": r["cpu_model"], "os_cpu_count": r["cpu_count"], "torch_threads": r["threads"]}


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    import torch

    from prismyra_b200 import synth

    layer = synth.make_fp8_layer(T_CTX, H, I, E, seed=0, device="cpu")
    per_step = max(3.0, min(20.0, 150.0 / max(1, args.steps + args.warmup)))
    cb = cpu_baseline(layer, max_seconds=min(60.0, per_step * max(1, args.steps)))
    line = {
        "metric": METRIC, "value": cb["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": T_CPU_SAMPLE / cb["value"] * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": f"routed-expert layer, T={T_CTX} (timed on a {T_CPU_SAMPLE}-token sample), H={H}, "
                               f"I={I}, E={E}, top-{K}", "tokens": T_CTX, "hidden": H, "intermediate": I,
                   "experts": E, "top_k": K},
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "torch_threads": torch.get_num_threads(),
    }
    print(json.dumps(line), flush=True)


def time_region(fn, steps: int, stream) -> float:
    """ms per call of fn over `steps` calls, CUDA events on the launching stream, synchronised both sides."""
    import torch

    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        fn()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def time_graph(fn, steps: int, per_graph: int = 10) -> float:
    """ms per call of fn replayed from a CUDA graph of `per_graph` calls (captured on a side stream after one eager
    call; the calls are capture-safe: no host synchronisation, workspace from the pool), CUDA events around the
    replays: the layer as a serving loop runs it, without the host's per-call launch cost."""
    import torch

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(per_graph):
                fn()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(2):
        g.replay()
    reps = max(1, steps // per_graph)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    del g
    return a.elapsed_time(b) / (reps * per_graph)


def vllm_gpu_path(layer: dict, tokens: list, steps: int) -> dict:
    """The reference's own GPU path for the routed layer on this box (prismyra/kernels/qwen3_moe.py:184-197): vLLM's
    batch-invariant router matmul, fused_topk and fused_experts (FP8 w8a8, 128x128 block scales) on the same seeded
    tensors, timed with CUDA events like the layer, beside this repository's layer in the activation-scale rule vLLM
    uses here (power-of-two scales when vLLM runs DeepGEMM with E8M0 scales, its default where DeepGEMM is installed;
    else the correctly rounded fp32 scales), and the relative L2 difference of the two outputs (same logits)."""
    import torch

    from prismyra_b200 import ops

    try:
        from vllm.model_executor.layers.fused_moe import fused_experts, fused_topk
        from vllm.model_executor.layers.fused_moe.config import FusedMoEQuantConfig
        try:
            from vllm.model_executor.layers.batch_invariant import linear_batch_invariant as router_linear
        except ImportError:
            router_linear = torch.nn.functional.linear
        quant = FusedMoEQuantConfig.make(quant_dtype=torch.float8_e4m3fn, block_shape=[128, 128],
                                         w1_scale=layer["w1_s"], w2_scale=layer["w2_s"])
        try:
            from vllm.utils import deep_gemm
            act_scale = "ue8m0" if deep_gemm.is_deep_gemm_e8m0_used() else "fp32"
        except Exception:  # noqa: BLE001
            act_scale = "fp32"
    except Exception as e:  # noqa: BLE001 - reported, not fatal: the comparison is optional
        return {"unavailable": f"vllm does not import here: {type(e).__name__}: {e}"[:300]}
    stream = torch.cuda.current_stream()
    res = {"path": "vllm " + __import__("vllm").__version__ + ": linear_batch_invariant + fused_topk + "
                   "fused_experts (FP8 w8a8 block 128x128)", "act_scale": act_scale}
    for T in tokens:
        x = layer["x"][:T].contiguous()

        def step():
            logits = router_linear(x, layer["router_w"])
            w, ids = fused_topk(x, logits, K, renormalize=True)[:2]
            return fused_experts(x, layer["w1"], layer["w2"], w, ids, quant_config=quant)

        try:
            ref_out = step()
            for _ in range(3):
                step()
            ms = time_region(step, 20, stream)
        except Exception as e:  # noqa: BLE001
            res[f"t{T}"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
            continue
        logits = router_linear(x, layer["router_w"])

        def mine():
            return ops.forward_fp8(x, layer["w1"], layer["w1_s"], layer["w2"], layer["w2_s"], K,
                                   router_w=layer["router_w"], act_scale=act_scale)

        for _ in range(3):
            mine()
        ours_ms = time_region(mine, 20, stream)
        same = ops.forward_fp8(x, layer["w1"], layer["w1_s"], layer["w2"], layer["w2_s"], K, logits=logits,
                               act_scale=act_scale).float()
        w, ids = fused_topk(x, logits, K, renormalize=True)[:2]
        ref_same = fused_experts(x, layer["w1"], layer["w2"], w, ids, quant_config=quant).float()
        rel = float((same - ref_same).norm() / ref_same.norm().clamp_min(1e-30))
        res[f"t{T}"] = {"ms": ms, "tokens_per_s": T / (ms * 1e-3), "ours_ms": ours_ms,
                        "speedup_ours_over_vllm": ms / ours_ms, "rel_l2_ours_vs_vllm_same_logits": rel}
    return res


def stage_times(layer: dict, T: int, reps: int = 20) -> dict:
    """Per-stage device time (ms) of one forward, each stage re-run alone on preallocated buffers and timed with
    CUDA events on the launching stream."""
    import torch

    from prismyra_b200 import ops

    s = torch.cuda.current_stream()
    x, rw = layer["x"][:T].contiguous(), layer["router_w"]
    r_out = ops.router_topk(x, rw, K)
    _, w, ids = r_out
    a_out = ops.align(ids, E)
    srt, eids, npp, _, slot_of, _ = a_out
    q_out = ops.quant_fp8(x, slot_of, K, srt.numel())
    g1_out = ops.gemm1_fp8(*q_out, layer["w1"], layer["w1_s"], eids, npp)
    g2_out = ops.gemm2_fp8(g1_out[0], g1_out[1], layer["w2"], layer["w2_s"], eids, npp, srt, w.reshape(-1), T, K)
    c_out = ops.combine(g2_out[0], T, K)
    out = {
        "router_topk": time_region(lambda: ops.router_topk(x, rw, K, out=r_out), reps, s),
        "align": time_region(lambda: ops.align(ids, E, out=a_out), reps, s),
        "quant_dispatch": time_region(lambda: ops.quant_fp8(x, slot_of, K, srt.numel(), out=q_out), reps, s),
        "gemm1": time_region(lambda: ops.gemm1_fp8(*q_out, layer["w1"], layer["w1_s"], eids, npp, out=g1_out),
                             reps, s),
        "gemm2": time_region(lambda: ops.gemm2_fp8(g1_out[0], g1_out[1], layer["w2"], layer["w2_s"], eids, npp, srt,
                                                   w.reshape(-1), T, K, out=g2_out), reps, s),
        "combine": time_region(lambda: ops.combine(g2_out[0], T, K, out=c_out), reps, s),
    }
    out["experts_hit"] = int((torch.bincount(ids.reshape(-1).long(), minlength=E) > 0).sum().item())
    out["slots"] = int(npp.item())
    return out


def ep_stack(dev, rank: int, world: int, layers: int, tokens: int, steps: int):
    """a stack of `layers` expert-parallel FP8 MoE layers (per-layer weights from seed =
    layer index, experts sharded over the ranks), `tokens` tokens per rank, router logits skewed by a Zipf(1.1)
    expert bias.  Returns ms per stack pass (max over ranks) and the peak expert load share."""
    import torch

    from prismyra_b200 import ep, synth

    epr = E // world
    lo, hi = rank * epr, (rank + 1) * epr
    bias = synth.zipf_bias(E).to(dev)
    from prismyra_b200 import ops

    stack = []
    # one peer exchange shared by all layers (a layer's exchange buffers are live only during its forward)
    exchange = ep.PeerExchange(E, K, H, I, rank, world, tokens, dev) if world > 1 else None
    for li in range(layers):
        L = synth.make_fp8_layer(8, H, I, E, seed=li, device=dev, gen_device="cuda")
        if world > 1:
            b = ep.CudaBackend(L["w1"][lo:hi].contiguous(), L["w1_s"][lo:hi].contiguous(),
                               L["w2"][lo:hi].contiguous(), L["w2_s"][lo:hi].contiguous(), L["router_w"], K,
                               bias=bias)
            stack.append(ep.PeerExpertParallelLayer(b, E, K, rank, world, exchange=exchange))
        else:  # one GPU holds every expert: the single-GPU layer itself (no dispatch to plan)
            stack.append({k: L[k] for k in ("w1", "w1_s", "w2", "w2_s", "router_w")})
        del L
    g = torch.Generator("cuda").manual_seed(1000 + rank)
    x = torch.randn(tokens, H, generator=g, device=dev).to(torch.bfloat16)
    bufs = [torch.empty_like(x), torch.empty_like(x)]

    def run():
        h = x
        for i, layer in enumerate(stack):
            if world > 1:
                h = layer.forward(h)
            else:
                h = ops.forward_fp8(h, layer["w1"], layer["w1_s"], layer["w2"], layer["w2_s"], K,
                                    router_w=layer["router_w"], bias=bias, out=bufs[i % 2])
        return h

    for _ in range(2):
        run()
    if world > 1:
        torch.distributed.barrier()
    ms = time_region(run, steps, torch.cuda.current_stream())
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    _, _, ids = ops.router_topk(x, stack[0].b.router_w if world > 1 else stack[0]["router_w"], K, bias=bias)
    load = torch.bincount(ids.reshape(-1).long(), minlength=E).float()
    del stack
    if exchange is not None:
        exchange.close()
    return ms, float(load.max() / load.sum())


def run_b200(args, rank: int, world: int, local: int) -> None:
    import torch

    from prismyra_b200 import ops, synth

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pk = peaks()
    fp8_peak = 2.0 * pk["bf16_tflops"]  # B200 FP8 dense rate is twice its BF16 dense rate
    # the seeded layer is drawn on the CPU (seed 0) and copied over: the CPU baseline times the
    # very same tensors
    layer_cpu = synth.make_fp8_layer(T_CTX, H, I, E, seed=0, device="cpu")
    layer = {k: v.to(dev) for k, v in layer_cpu.items()}
    if world > 1 or args.no_cpu_baseline:
        del layer_cpu
        layer_cpu = None
    x = layer["x"]
    stream = torch.cuda.current_stream()
    if world > 1:
        # every rank owns E/world experts and its own T_CTX tokens (weak scaling); rows move between the ranks by
        # the kernels' own NVLink peer stores (no host synchronisation, no collective library on the data path)
        from prismyra_b200 import ep

        gx = torch.Generator("cuda").manual_seed(1000 + rank)
        x = torch.randn(T_CTX, H, generator=gx, device=dev).to(torch.bfloat16)
        epr = E // world
        lo, hi = rank * epr, (rank + 1) * epr
        ep_layer = ep.PeerExpertParallelLayer(
            ep.CudaBackend(layer["w1"][lo:hi].contiguous(), layer["w1_s"][lo:hi].contiguous(),
                           layer["w2"][lo:hi].contiguous(), layer["w2_s"][lo:hi].contiguous(), layer["router_w"], K),
            E, K, rank, world, max_tokens=T_CTX)

        def step():
            return ep_layer.forward(x)
    else:
        def step():
            return ops.forward_fp8(x, layer["w1"], layer["w1_s"], layer["w2"], layer["w2_s"], K,
                                   router_w=layer["router_w"])

    clk = Clocks(local).start()
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    ws, _ = ops.workspace_for(x, T_CTX, H, I, E, K)
    ops.read_status(ws)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    barrier()
    clk.mark_start()
    ms = time_region(step, args.steps, stream)
    barrier()
    clk.mark_end()
    clk.stop()
    ops.read_status(ws)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    value = world * T_CTX / (ms * 1e-3)

    ep_phases = None
    if world > 1:
        # per-phase device times of the expert-parallel step (outside the timed region; medians of a few steps,
        # then the maximum over the ranks), and the NVLink bytes this rank's rows send: a remote pair's FP8 row
        # and scales out, its weighted bf16 row back
        runs = []
        for _ in range(5):
            marks = []
            ep_layer.forward(x, marks=marks)
            runs.append(marks)
        torch.cuda.synchronize()
        names = ep.PeerExpertParallelLayer.PHASES
        per = torch.tensor([[m[i].elapsed_time(m[i + 1]) for i in range(len(names))] for m in runs])
        med = per.median(dim=0).values.to(dev)
        torch.distributed.all_reduce(med, op=torch.distributed.ReduceOp.MAX)
        own = torch.div(ep_layer.b.route(x)[1].reshape(-1), epr, rounding_mode="floor")
        remote = int((own != rank).sum().item())
        sent = remote * (H + (H // 128) * 4 + H * 2)
        t = torch.tensor([float(sent)], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ep_phases = {"ms": {n: round(float(v), 4) for n, v in zip(names, med.tolist())},
                     "nvlink_bytes_per_rank_max": int(t.item()),
                     "nvlink_ms_at_770_gbs": float(t.item()) / 770e9 * 1e3,
                     "note": "median of 5 steps per rank, max over ranks; count/dispatch/down end with a device "
                             "barrier across the ranks"}

    # end to end through the public calls with host buffers: every step uploads its pinned x and downloads its
    # result to pinned memory, consecutive steps overlapping (a step's upload runs during the previous step's
    # layer, its download during the next step's layer): ops.forward_fp8_host_async on one GPU, ops.host_async
    # around the expert-parallel layer on every rank; the timed region ends when the last download has landed.
    x_host = x.cpu().pin_memory()
    out_hosts = [torch.empty(T_CTX, H, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    last = [None]

    def e2e_step(i=0):
        if world > 1:
            _, last[0] = ops.host_async(lambda xs, _os: ep_layer.forward(xs), x_host, out_hosts[i % 2], device=dev)
        else:
            _, last[0] = ops.forward_fp8_host_async(x_host, layer["w1"], layer["w1_s"], layer["w2"], layer["w2_s"],
                                                    K, layer["router_w"], out_host=out_hosts[i % 2])

    def e2e_region(steps):
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(steps):
            e2e_step(i)
        if last[0] is not None:
            stream.wait_event(last[0])  # the last download (the copies run on their own streams)
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / steps

    for i in range(3):
        e2e_step(i)
    barrier()
    e2e_ms = e2e_region(args.steps)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())

    st = stage_times(layer, T_CTX)
    fl = synth.layer_flops(T_CTX, H, I, K)
    g1_tflops = fl["gemm1"] / (st["gemm1"] * 1e-3) / 1e12
    layer_tflops = fl["total"] / (ms * 1e-3) / 1e12

    # the branch-readout shape: weight streaming, reported in GB/s of algorithmic bytes
    xb = x[:T_BRANCH].contiguous()

    def branch_step():
        return ops.forward_fp8(xb, layer["w1"], layer["w1_s"], layer["w2"], layer["w2_s"], K,
                               router_w=layer["router_w"])

    for _ in range(5):
        branch_step()
    b_eager_ms = time_region(branch_step, max(20, args.steps), stream)
    b_ms = time_graph(branch_step, max(20, args.steps))
    b_st = stage_times(layer, T_BRANCH)
    b_bytes = synth.layer_bytes(T_BRANCH, b_st["experts_hit"], H, I, E)
    b_gbs = b_bytes / (b_ms * 1e-3) / 1e9

    # NVFP4 variant at T=5120: weights from the same FP8 layer via the reference's
    # prepare_layer recipe, synthetic activation calibration
    nw = synth.nvfp4_device_layer(layer, dev)
    a1, a2 = nw["a1"], nw["a2"]

    def nv_step():
        return ops.forward_nvfp4(x, nw["w1"], nw["w1_sf"], nw["al1"], a1, nw["w2"], nw["w2_sf"], nw["al2"], a2, K,
                                 router_w=layer["router_w"])

    for _ in range(5):
        nv_step()
    nv_ms = time_region(nv_step, max(20, args.steps), stream)
    nv_tflops = fl["total"] / (nv_ms * 1e-3) / 1e12
    fp4_peak = 4.0 * pk["bf16_tflops"]  # B200 FP4 dense rate is four times its BF16 dense rate

    # NVFP4 weight preparation on the GPU (pm_nvfp4_prepare over both expert stacks of the layer):
    # algorithmic bytes = e4m3 read once + packed codes and e4m3 scales written (1 + 1/2 + 1/16 bytes per weight)
    def prep_step():
        ops.nvfp4_prepare(layer["w1"], layer["w1_s"])
        ops.nvfp4_prepare(layer["w2"], layer["w2_s"])

    prep_step()
    prep_ms = time_region(prep_step, 5, stream)
    n_weights = layer["w1"].numel() + layer["w2"].numel()
    prep_bytes = n_weights * (1.0 + 0.5 + 1.0 / 16.0)
    # the reference's way: prepare_layer's per-expert torch loop (dequantise, global scale, quantize) on this GPU
    from prismyra_b200.kernels import nvfp4 as nv_mod

    def torch_prep():
        for e in range(E):
            for w, sc in ((layer["w1"], layer["w1_s"]), (layer["w2"], layer["w2_s"])):
                d = nv_mod.dequant_fp8(w[e], sc[e])
                nv_mod.quantize(d, 448.0 * 6.0 / d.abs().amax().clamp_min(1e-12))

    torch.cuda.synchronize()
    t_ref = time_region(torch_prep, 1, stream)
    prep = {"ms": prep_ms, "reference_torch_ms": t_ref, "gbs": prep_bytes / (prep_ms * 1e-3) / 1e9,
            "frac_hbm": prep_bytes / (prep_ms * 1e-3) / 1e9 / pk["hbm_gbs"], "weights": n_weights,
            "algorithmic_bytes": prep_bytes,
            "note": "three launches per stack: a zeroing, the per-matrix maxima (reads the weights), the quantisation "
                    "(reads them again), so DRAM traffic is about 2.56 bytes per weight"}

    # the whole block (routed + shared expert + bf16 sum) in one library call; synthetic block-FP8 shared expert
    # with the transformers Qwen3.5-MoE default shared_expert_intermediate_size of 512
    block = None
    if world == 1:
        gs = torch.Generator("cuda").manual_seed(77)
        IS = 512
        sw13, sw13_s = synth.quantize_fp8_blocks(torch.randn(2 * IS, H, generator=gs, device=dev) * 0.02)
        sw2, sw2_s = synth.quantize_fp8_blocks(torch.randn(H, IS, generator=gs, device=dev) * 0.02)
        w_sg = (torch.randn(H, generator=gs, device=dev) * 0.02).to(torch.bfloat16)

        def block_step():
            return ops.block_fp8(x, layer["w1"], layer["w1_s"], layer["w2"], layer["w2_s"], K, w_sg, sw13, sw13_s,
                                 sw2, sw2_s, router_w=layer["router_w"])

        for _ in range(5):
            block_step()
        blk_ms = time_region(block_step, max(20, args.steps), stream)
        shared_flops = T_CTX * 2 * 3 * H * IS
        block = {"ms": blk_ms, "tokens_per_s": T_CTX / (blk_ms * 1e-3), "shared_intermediate": IS,
                 "shared_ms_over_routed": blk_ms - ms,
                 "tflops": (fl["total"] + shared_flops) / (blk_ms * 1e-3) / 1e12}

    vllm_ref = None
    if world == 1 and not args.no_vllm:
        vllm_ref = vllm_gpu_path(layer, [T_CTX, T_BRANCH], args.steps)

    if world > 1:
        ep_layer.close()  # every rank together: frees this layer's exchange before the stack makes its own
    stack_ms, stack_peak = ep_stack(dev, rank, world, args.stack_layers, 4096, max(2, args.steps // 20))

    if rank != 0:
        return
    cb = None
    if layer_cpu is not None:
        cb = cpu_baseline(layer_cpu)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3", "data": "synthetic",
        "config": {"workload": f"FP8 block-scaled routed-expert layer, T={T_CTX} tokens per GPU (BASELINE configs[1])",
                   "tokens": T_CTX, "hidden": H, "intermediate": I, "experts": E, "top_k": K,
                   "parallelism": f"expert parallel x{world} (NVLink peer stores from the kernels)" if world > 1
                   else "single GPU",
                   "l2": "no flush: 604 MB of expert weights (> 126 MB L2) stream from HBM every step"},
        "tflops": layer_tflops,
        "frac_fp8_peak": layer_tflops / fp8_peak,
        "roofline": {"bound": "tensor", "kernel": "moe_gemm_fp8_kernel<0> (gate_up)", "achieved": g1_tflops,
                     "peak": fp8_peak, "unit": "TFLOP/s", "frac": g1_tflops / fp8_peak,
                     "traffic": profile_traffic("gate_up"),
                     "peak_source": f"2 x bf16_tflops of {pk['source']} MEASURED_PEAKS.json ({pk['bf16_tflops']})",
                     "flops_per_launch": fl["gemm1"]},
        "stages_ms": {k: round(v, 4) for k, v in st.items() if isinstance(v, float)},
        "branch_t128": {"ms": b_ms, "eager_ms": b_eager_ms,
                        "timing": "ms: the forward replayed from a CUDA graph (10 calls per graph, as a serving loop "
                                  "runs a 128-token step); eager_ms: the same calls issued one by one from Python",
                        "tokens_per_s": T_BRANCH / (b_ms * 1e-3), "gbs": b_gbs,
                        "frac_hbm": b_gbs / pk["hbm_gbs"], "experts_hit": b_st["experts_hit"],
                        "algorithmic_bytes": b_bytes,
                        "stages_ms": {k: round(v, 4) for k, v in b_st.items() if isinstance(v, float)}},
        "e2e": {"value": world * T_CTX / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": T_CTX * H * 2, "d2h_bytes_per_step": T_CTX * H * 2,
                "mode": ("ops.forward_fp8_host_async" if world == 1 else "ops.host_async around the expert-parallel "
                         "layer on every rank") + " per step, consecutive steps overlapping (upload of step i+1 and "
                         "download of step i-1 during the layer of step i)"},
        "nvfp4_t5120": {"ms": nv_ms, "tokens_per_s": T_CTX / (nv_ms * 1e-3), "tflops": nv_tflops,
                        "frac_fp4_peak": nv_tflops / fp4_peak, "fp4_peak": fp4_peak,
                        "weights": "NVFP4 from the FP8 layer (reference prepare_layer recipe), synthetic calibration"},
        "ep_stack": {"layers": args.stack_layers, "tokens_per_gpu": 4096, "ms": stack_ms,
                     "tokens_per_s": world * 4096 / (stack_ms * 1e-3), "zipf_peak_expert_share": stack_peak,
                     "config": "BASELINE configs[4]: FP8 layers, per-layer weights from seed = layer, Zipf(1.1) "
                               "expert bias, experts sharded over the ranks"},
        "gpu_launches": (KERNELS_PER_EP_STEP if world > 1 else KERNELS_PER_STEP) * args.steps,
        "clocks": clk.summary(),
    }
    line["nvfp4_prepare"] = prep
    if ep_phases is not None:
        line["ep_phases"] = ep_phases
    if block is not None:
        line["block_t5120"] = block
    if vllm_ref is not None:
        line["vllm_gpu_same_box"] = vllm_ref
    if cb is not None:
        line["cpu_baseline"] = cb
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-vllm", action="store_true", help="skip timing the reference's vLLM GPU path")
    ap.add_argument("--stack-layers", type=int, default=36)
    args = ap.parse_args()
    if args.impl == "reference":
        # the CPU reference runs on rank 0 only; other ranks exit without work or a process group
        run_reference(args, int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")))
        return
    rank, world, local = dist_init()
    try:
        run_b200(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
