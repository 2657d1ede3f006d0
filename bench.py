#!/usr/bin/env python
"""FP8 MoE layer benchmark (decode step at 64 tokens per GPU).

Workload per step (one GPU): the decode projections and MoE layer of the
benchmark geometry H=2048, E=128, I=768, top-8, FP8-E4M3 with 128x128 fp32
block scales:
    qkv = fp8_gemv(x, Wqkv [4096,2048])             dense weight-only FP8
    o   = fp8_gemv(qkv[:, :2048], Wo [2048,2048])   (o_proj input stand-in)
    y   = moe_layer(o)  router -> top-8 -> routed + shared experts -> combine
Synthetic seeded weights (N(0,0.02) quantised per 128x128 block), bf16 N(0,1)
inputs. Steps rotate over `--layers` independent weight sets (4 x ~620 MB by
default, > 2x the 126 MB L2), so weights stream from HBM every step.

With torchrun (N > 1) the expert-parallel layer runs (experts sharded over the
ranks, NCCL all-to-all dispatch and combine); `--replicas` runs independent
full-layer replicas instead. `--workload prefill` (ragged ~8k-token batch) and
`--workload mixed` (64 decode + 1280 packed prompt rows) run on one GPU. Timing: CUDA events on the launching stream, barrier + synchronize on
both sides, max over ranks.

--impl reference times the reference's arithmetic on the host CPU (the oracle
port of src/drama3/kernels.py et al.; the reference itself has no CPU path and
cannot run on this box's GPU tooling), one bounded sample per step.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "drama-3-single-b300-inference_b200"
sys.path.insert(0, str(PKG))

E, I, H, TOPK = 128, 768, 2048, 8
N_QKV, N_O = 4096, 2048

# DRAM traffic of one gate_up launch of the default decode step, as ncu
# measured it (not measured by this script; see the profile named here).
GATE_UP_TRAFFIC_BYTES = 404.70e6
GATE_UP_TRAFFIC_SOURCE = ("profiles/expert_gemv_T64_full.md: dram__bytes_read.sum + "
                          "dram__bytes_write.sum of the gate_up launch, ncu --set full")


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """SM clock and throttle reasons during the timed region. NVML is read
    every 5 ms from a thread, the first sample before the region starts, so a
    region of a few tens of milliseconds still gets several samples; without
    NVML it falls back to `nvidia-smi -lms 200`. Read-only: nothing is set."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.thread = None
        self.stop = threading.Event()
        self.lines: list[str] = []
        self.samples: list[tuple[float, float, frozenset]] = []

    def _nvml(self):
        import pynvml as nv
        import torch
        nv.nvmlInit()
        try:
            p = torch.cuda.get_device_properties(self.gpu)
            h = nv.nvmlDeviceGetHandleByPciBusId(
                f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0")
        except Exception:
            h = nv.nvmlDeviceGetHandleByIndex(self.gpu)
        bits = dict(zip(self.NAMES, (nv.nvmlClocksEventReasonHwSlowdown,
                                     nv.nvmlClocksEventReasonHwThermalSlowdown,
                                     nv.nvmlClocksEventReasonSwThermalSlowdown,
                                     nv.nvmlClocksEventReasonSwPowerCap)))
        mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        return nv, h, bits, mx

    def __enter__(self):
        try:
            nv, h, bits, mx = self._nvml()

            def run():
                while True:
                    try:
                        sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                        r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((sm, mx, frozenset(n for n, b in bits.items() if r & b)))
                    except Exception:
                        pass
                    if self.stop.wait(0.005):
                        return

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.samples and time.time() - t0 < 1.0:
                time.sleep(0.001)
            return self
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=1.0)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        for s_mhz, m_mhz, rs in self.samples:
            sm.append(s_mhz)
            mx = m_mhz
            reasons |= rs
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(self.NAMES, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm),
                "source": "nvml, 5 ms" if self.samples else "nvidia-smi, 200 ms"}


def algorithmic_bytes(ids_host, T: int) -> dict:
    """Bytes a step must move at minimum (weights of the U distinct selected
    experts + shared expert + router + dense projections + activations)."""
    import numpy as np

    U = len(np.unique(ids_host))
    w13 = 2 * I * H + (2 * I // 128) * (H // 128) * 4
    w2 = H * I + (H // 128) * (I // 128) * 4
    R = T * TOPK + T
    gate_up = (U + 1) * w13 + R * (H + H // 128 * 4) + R * (I + I // 128 * 4)
    down = (U + 1) * w2 + R * (I + I // 128 * 4) + R * H * 4
    router = (E + 1) * H * 2 + T * H * 2
    dense = N_QKV * H + (N_QKV // 128) * (H // 128) * 4 + N_O * H + (N_O // 128) * (H // 128) * 4
    dense += T * H * 2 * 2 + T * (N_QKV + N_O) * 2
    total = gate_up + down + router + dense + T * H * 2
    return {"U": U, "gate_up": gate_up, "down": down, "dense": dense, "total": total}


def cpu_baseline(T: int, seconds: float, weights_cpu) -> dict:
    """Oracle port on the host cores: whole decode steps (dense projections +
    MoE layer) until `seconds` of work have been done (at least one step)."""
    import numpy as np

    sys.path.insert(0, str(ROOT))
    from oracle import moe_oracle as O

    rng = np.random.default_rng(0)
    (wqkv, sqkv, wo, so, router, ex, sh) = weights_cpu
    steps, t0 = 0, time.perf_counter()
    while True:
        x = O.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
        qkv = O.fp8_gemv(x, wqkv, sqkv)
        o = O.fp8_gemv(qkv[:, :H], wo, so)
        O.moe_layer(o, router, ex, sh, TOPK)
        steps += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    threads = int(os.environ.get("OMP_NUM_THREADS", "0")) or os.cpu_count()
    return {"value": T * steps / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{steps} decode step(s) of T={T}: fp8 QKV+o_proj GEMV + full MoE layer "
                      f"(numpy, BLAS threads={threads}), {dt:.1f} s"}


def run_reference(args) -> None:
    """--impl reference: the oracle port on host cores, bounded sample per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    sys.path.insert(0, str(ROOT))
    from oracle import moe_oracle as O

    T = args.tokens
    rng = np.random.default_rng(1)
    # CPU synthetic layer (hashed uniform weights quantised per 128x128 block)
    ex = O.Experts(*[{} for _ in range(4)])
    for e in range(E):
        ex.w13[e], ex.s13[e] = O.synth_expert(21, e, 2 * I, H, amp=0.035)
        ex.w2[e], ex.s2[e] = O.synth_expert(22, e, H, I, amp=0.035)
    sh = O.Experts({0: None}, {0: None}, {0: None}, {0: None})
    sh.w13[0], sh.s13[0] = O.synth_expert(23, 0, 2 * I, H, amp=0.035)
    sh.w2[0], sh.s2[0] = O.synth_expert(24, 0, H, I, amp=0.035)
    router = O.bf16_round((O.hash_uniform(25, (E + 1, H)) * 0.035).astype(np.float32))
    wqkv, sqkv = O.synth_expert(26, 0, N_QKV, H, amp=0.035)
    wo, so = O.synth_expert(27, 0, N_O, H, amp=0.035)

    def step():
        x = O.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
        qkv = O.fp8_gemv(x, wqkv, sqkv)
        o = O.fp8_gemv(qkv[:, :H], wo, so)
        O.moe_layer(o, router, ex, sh, TOPK)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = T * args.steps / dt
    threads = int(os.environ.get("OMP_NUM_THREADS", "0")) or os.cpu_count()
    line = {
        "impl": "reference", "metric": "fp8_moe_layer_decode_tokens_per_s", "value": value,
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1000 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp8_e4m3 x fp8_e4m3 -> f32", "data": "synthetic",
        "config": {"workload": f"decode T={T}: FP8 QKV+o_proj GEMV + MoE layer (H=2048,E=128,I=768,top-8)",
                   "tokens_per_step": T},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} full decode steps of T={T} on host cores "
                                   "(numpy oracle port of the reference arithmetic)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ep(args, world: int, rank: int, local: int, dev) -> None:
    """N > 1: the expert-parallel layer (d3moe.ep) with 128/N experts per rank
    and `--tokens` decode tokens per rank (weak scaling), after the replicated
    dense QKV / o_proj GEMVs. Dispatch and combine are NCCL all_to_all_v over
    NVLink; the time is the max over ranks."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from d3moe import _lib, ops, synth
    from d3moe.ep import CudaEPOps, ExpertParallelMoE, ep_row_bytes_fp8

    T = args.tokens
    lib = _lib.load()
    E_local = E // world
    stage = {"events": None}

    class TimedOps(CudaEPOps):
        """Marks the EP stage boundaries on the current stream (EP_STAGES) and
        records the library's stage events around the routed-expert call."""

        marks = None  # name -> torch.cuda.Event while stage timing is on
        recorded: set = set()

        def mark(self, name):
            if self.marks is not None:
                self.marks[name].record(torch.cuda.current_stream(dev))
                self.recorded.add(name)

        def router_logits(self, x, router_weight, bias=None):
            self.mark("layer")
            return super().router_logits(x, router_weight, bias)

        def pack_fp8(self, *a, **kw):
            self.mark("pack")
            return super().pack_fp8(*a, **kw)

        def unpack_fp8(self, *a, **kw):
            self.mark("dispatched")
            return super().unpack_fp8(*a, **kw)

        def local_experts_fp8(self, *a, **kw):
            self.mark("experts")
            if stage["events"] is not None:
                lib.d3_set_stage_events(stage["events"], 5)
            try:
                out = super().local_experts_fp8(*a, **kw)
            finally:
                lib.d3_set_stage_events(None, 0)
            self.mark("experts_done")
            return out

        def combine(self, *a, **kw):
            self.mark("combine")
            out = super().combine(*a, **kw)
            self.mark("end")
            return out

    eops = TimedOps()
    layers, dense, routers, experts_all, shareds = [], [], [], [], []
    for li in range(args.layers):
        gen = torch.Generator(device="cpu")
        gen.manual_seed(li)
        router = (torch.randn((E + 1, H), generator=gen) * 0.02).to(torch.bfloat16).to(dev)
        experts = synth.make_experts(E_local, I, H, 1000 * li + 7 + rank, dev)
        shared = synth.make_experts(1, I, H, 1000 * li + 3, dev)
        routers.append(router)
        experts_all.append(experts)
        shareds.append(shared)
        layers.append(ExpertParallelMoE(router, experts, shared, E, TOPK, ops=eops))
        g = torch.Generator(device=dev)
        g.manual_seed(li + 77)
        wq, sq = synth.block_quantize(torch.randn((N_QKV, H), generator=g, device=dev) * 0.02)
        wo, so = synth.block_quantize(torch.randn((N_O, H), generator=g, device=dev) * 0.02)
        dense.append((wq, sq, wo, so))
    nb = ctypes.c_size_t()
    lib.d3_fp8_gemv_workspace_size(T, N_QKV, H, ctypes.byref(nb))
    ws_dense = torch.empty(nb.value, dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    gin = torch.Generator(device=dev)
    gin.manual_seed(4242 + rank)
    xs = torch.randn((8, T, H), generator=gin, device=dev).to(torch.bfloat16)
    qkv = torch.empty((T, N_QKV), dtype=torch.bfloat16, device=dev)
    o = torch.empty((T, N_O), dtype=torch.bfloat16, device=dev)

    def gemv(x, wq, sq, n, out):
        _lib.call("d3_fp8_gemv", x.data_ptr(), x.stride(0), wq.data_ptr(), sq.data_ptr(), T, n, H,
                  out.data_ptr(), out.stride(0), ws_dense.data_ptr(), ws_dense.numel(),
                  status.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)

    ids_seen = []

    def step(i, x, keep_ids=False):
        li = i % args.layers
        wq, sq, wo_, so_ = dense[li]
        eops.mark("step")
        gemv(x, wq, sq, N_QKV, qkv)
        gemv(qkv, wo_, so_, N_O, o)
        out, ids, _ = layers[li].forward(o, return_routing=True)
        if keep_ids:
            ids_seen.append(ids)
        return out

    for i in range(args.warmup):
        step(i, xs[i % len(xs)])
    torch.cuda.synchronize(dev)
    dist.barrier()
    torch.cuda.synchronize(dev)

    # The decode step captured in one CUDA graph per weight set, like the
    # reference's captured decode step (src/drama3/engine.py:84-92): the NCCL
    # exchanges and every kernel replay without host launch overhead. The
    # input is copied into the graph's static buffer before each replay.
    graphs, x_static, y_static = [], [], []
    graph_ms = None
    kernels = None
    if not args.eager:
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            for li in range(args.layers):
                xb = xs[li % len(xs)].clone()
                step(li, xb)  # warm the capture stream's allocations
                g = torch.cuda.CUDAGraph(keep_graph=(li == 0))
                with torch.cuda.graph(g, stream=cap):
                    yb = step(li, xb)
                graphs.append(g)
                x_static.append(xb)
                y_static.append(yb)
        stream.wait_stream(cap)
        torch.cuda.synchronize(dev)
        dist.barrier()
        kernels = graph_kernels(graphs[0])
        # the replay must reproduce the eager step bit for bit
        y_eager = step(0, x_static[0]).clone()
        y_static[0].zero_()
        graphs[0].replay()
        torch.cuda.synchronize(dev)
        if not torch.equal(y_static[0], y_eager):
            raise RuntimeError("CUDA graph replay differs from the eager step")
        dist.barrier()
        for i in range(args.warmup):
            li = i % args.layers
            x_static[li].copy_(xs[i % len(xs)])
            graphs[li].replay()
        torch.cuda.synchronize(dev)
        dist.barrier()
        torch.cuda.synchronize(dev)
        gstart, gend = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        gstart.record(stream)
        for i in range(args.steps):
            li = i % args.layers
            x_static[li].copy_(xs[(args.warmup + i) % len(xs)])
            graphs[li].replay()
        gend.record(stream)
        torch.cuda.synchronize(dev)
        dist.barrier()
        graph_ms = gstart.elapsed_time(gend) / args.steps
        t = torch.tensor([graph_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        graph_ms = float(t.item())

    # per-stage split of one step, from a graph of layer 0 with timing event
    # nodes at the stage boundaries (external events), replayed and read back
    stages = ep_stage_times(eops, lambda xb: step(0, xb), xs[0].clone(), dev, stream, reps=20)
    dist.barrier()

    stage_events = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    for evs in stage_events:
        for e in evs:
            e.record(stream)
    stage_arrays = [(ctypes.c_void_p * 5)(*[e._as_parameter_.value for e in evs]) for evs in stage_events]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for i in range(args.steps):
            stage["events"] = stage_arrays[i]
            step(args.warmup + i, xs[(args.warmup + i) % len(xs)], keep_ids=True)
        stage["events"] = None
        end.record(stream)
        torch.cuda.synchronize(dev)
    dist.barrier()
    ms = start.elapsed_time(end) / args.steps
    gate_avg = statistics.mean(evs[1].elapsed_time(evs[2]) for evs in stage_events)
    down_avg = statistics.mean(evs[2].elapsed_time(evs[3]) for evs in stage_events)
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    eager_ms = float(t.item())
    ms = eager_ms if graph_ms is None else graph_ms
    # experts this rank streamed per step: distinct global ids it owns, over all ranks' tokens
    gathered = [torch.empty_like(ids_seen[0]) for _ in range(world)]
    U_local = []
    for ids in ids_seen:
        dist.all_gather(gathered, ids)
        allids = torch.cat(gathered).cpu().numpy()
        mine = allids[(allids // E_local) == rank]
        U_local.append(len(np.unique(mine)))
    u = statistics.mean(U_local)

    # end to end with host buffers
    hx = torch.randn((T, H)).to(torch.bfloat16).pin_memory()
    hy = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
    dx = torch.empty((T, H), dtype=torch.bfloat16, device=dev)

    def e2e_step(i):
        if not graphs:
            dx.copy_(hx, non_blocking=True)
            hy.copy_(step(i, dx), non_blocking=True)
        else:
            li = i % args.layers
            x_static[li].copy_(hx, non_blocking=True)
            graphs[li].replay()
            hy.copy_(y_static[li], non_blocking=True)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        e2e_step(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([e2e_ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())

    pk = peaks()
    w13 = 2 * I * H + (2 * I // 128) * (H // 128) * 4
    rows = T * world  # token rows received per rank (capacity mode: every token once)
    gate_bytes = u * w13 + rows * TOPK * (H + I)
    achieved = gate_bytes / (gate_avg * 1e-3) / 1e9
    line = {
        "metric": "fp8_moe_layer_decode_tokens_per_s",
        "value": T * world / (ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp8_e4m3 x fp8_e4m3 -> f32 (experts); fp8 weights x bf16 (dense)",
        "data": "synthetic",
        "config": {
            "workload": f"decode T={T}/GPU: FP8 QKV + o_proj weight-only GEMV + expert-parallel MoE layer "
                        f"(H=2048, E=128 sharded {E_local}/GPU, I=768, top-8, shared expert replicated)",
            "tokens_per_gpu": T, "weight_sets_rotated": args.layers,
            "l2": "inputs larger than L2: weight sets rotated per step",
            "parallelism": f"ep{world}",
            "collective": "NCCL all_to_all_single, fixed capacity (token rows + per-rank routing out, "
                          "weighted partial rows back; no host synchronisation)",
            "launch": "eager" if graph_ms is None else "one CUDA graph per weight set (kernels + NCCL), replayed",
            "eager_ms_per_step": eager_ms,
            "dispatch_row_bytes": ep_row_bytes_fp8(H, TOPK),
        },
        "stages_ms": stages,
        "roofline": {
            "bound": "hbm",
            "kernel": "expert_gemv_kernel<EPI_GATE_UP> on the rank's received rows (rank 0)",
            "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
            "peak_source": pk["source"], "traffic": None,
            "algorithmic_bytes_per_launch": gate_bytes, "avg_launch_ms": gate_avg,
            "down_avg_launch_ms": down_avg, "mean_local_active_experts": u,
        },
        "e2e": {"value": T * world / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": hx.numel() * 2, "d2h_bytes_per_step": hy.numel() * 2,
                "ms_per_step": e2e_ms},
        # counted from the captured step graph's kernel nodes when it could be read, else by hand:
        # dense 2 x (activation split + tcgen05 GEMV), router, route, FP8 pack, unpack, routed
        # experts (permute, scatter, gate_up, down, combine), shared expert (permute+quant, gate_up,
        # down, combine), combine_pairs
        "gpu_launches": (kernels["ours"] if kernels else 18) * args.steps,
        "graph_kernels_per_step": kernels,
        "clocks": clocks.summary(),
    }
    # graphs holding NCCL work are released before the process group goes
    del graphs, x_static, y_static
    torch.cuda.synchronize(dev)
    if not args.no_extras:
        line["config5"] = ep_config5(args, eops, routers, experts_all, shareds, world, rank, dev, stream)
    if rank == 0:
        print(json.dumps(line), flush=True)


def graph_kernels(g) -> dict | None:
    """Kernel nodes of a captured CUDA graph (created with keep_graph=True),
    by origin: this library's (mangled names in namespace d3), NCCL's, and
    the rest (torch copies and fills). None when the graph cannot be read."""
    try:
        from cuda.bindings import driver as cu

        h = cu.CUgraph(g.raw_cuda_graph())
        err, _, n = cu.cuGraphGetNodes(h, 0)
        if err != cu.CUresult.CUDA_SUCCESS:
            return None
        err, nodes, n = cu.cuGraphGetNodes(h, n)
        out = {"ours": 0, "nccl": 0, "other": 0}
        for nd in nodes[:n]:
            err, typ = cu.cuGraphNodeGetType(nd)
            if err != cu.CUresult.CUDA_SUCCESS or typ != cu.CUgraphNodeType.CU_GRAPH_NODE_TYPE_KERNEL:
                continue
            err, prm = cu.cuGraphKernelNodeGetParams(nd)
            if err != cu.CUresult.CUDA_SUCCESS:
                return None
            err, name = cu.cuFuncGetName(prm.func)
            name = name.decode() if err == cu.CUresult.CUDA_SUCCESS and name else ""
            key = "ours" if name.startswith("_ZN2d3") else "nccl" if "nccl" in name.lower() else "other"
            out[key] += 1
        return out
    except Exception:  # noqa: BLE001 - reported as unavailable
        return None


EP_STAGES = [  # (name, from mark, to mark): one EP step split at the marks TimedOps records
    ("dense", "step", "layer"),            # QKV + o_proj FP8 GEMVs (activation split + tcgen05 GEMV each)
    ("route", "layer", "pack"),            # router + top-8 (+ exact mode: row plan, count exchange, host read)
    ("dispatch", "pack", "dispatched"),    # FP8 row pack + all_to_all
    ("unpack", "dispatched", "experts"),
    ("local_experts", "experts", "experts_done"),
    ("return", "experts_done", "combine"),  # partial rows all_to_all back + shared-expert join
    ("combine", "combine", "end"),
]


def _stage_summary(samples: list[dict], dev) -> dict:
    """Mean per stage over samples on this rank, then the max over ranks."""
    import torch
    import torch.distributed as dist

    names = [n for n, _, _ in EP_STAGES if all(n in smp for smp in samples)]
    v = torch.tensor([statistics.mean(smp[n] for smp in samples) for n in names], device=dev)
    if dist.is_initialized():
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
    return {n: float(x) for n, x in zip(names, v.tolist())}


def _read_marks(marks: dict, recorded: set) -> dict:
    return {n: marks[a].elapsed_time(marks[b]) for n, a, b in EP_STAGES if a in recorded and b in recorded}


def ep_stage_times(eops, run, x, dev, stream, reps: int = 20) -> dict:
    """Per-stage times (ms, max over ranks) of run(x), captured once into a
    CUDA graph with timing event nodes at the stage marks and replayed."""
    import torch

    names = {m for _, a, b in EP_STAGES for m in (a, b)}
    marks = {m: torch.cuda.Event(enable_timing=True, external=True) for m in names}
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(stream)
    eops.recorded = set()
    with torch.cuda.stream(cap):
        run(x)
        g = torch.cuda.CUDAGraph()
        eops.marks = marks
        try:
            with torch.cuda.graph(g, stream=cap):
                run(x)
        finally:
            eops.marks = None
    stream.wait_stream(cap)
    torch.cuda.synchronize(dev)
    samples = []
    for _ in range(reps):
        g.replay()
        torch.cuda.synchronize(dev)
        samples.append(_read_marks(marks, eops.recorded))
    del g
    return _stage_summary(samples, dev)


def ep_config5(args, eops, routers, experts_all, shareds, world, rank, dev, stream) -> dict:
    """Expert-parallel layer at the job-level batch sizes of the fifth
    benchmark configuration: 512 decode tokens and 8192 prefill tokens split
    evenly over the ranks, bf16 N(0,1) inputs from seed 4; capacity mode
    replayed from CUDA graphs, exact mode eager. Times are the max over
    ranks."""
    import torch
    import torch.distributed as dist

    from d3moe.ep import ExpertParallelMoE

    out = {}
    nl = len(routers)
    # prefill both ways: capacity (every token to every rank, no host read,
    # graph-captured) and exact (only the owning ranks, one host read of the
    # row counts per call)
    for kind, total, mode in (("decode", 512, "capacity"), ("prefill", 8192, "capacity"),
                              ("prefill_exact", 8192, "exact")):
        T = total // world
        layers = [ExpertParallelMoE(routers[i], experts_all[i], shareds[i], E, TOPK, ops=eops, mode=mode)
                  for i in range(nl)]
        g = torch.Generator(device=dev)
        g.manual_seed(4 + 1000 * rank)
        xs = torch.randn((nl, T, H), generator=g, device=dev).to(torch.bfloat16)
        steps = args.steps if mode == "capacity" else max(5, min(args.steps, 20))
        for i in range(3):
            layers[i % nl].forward(xs[i % nl])
        torch.cuda.synchronize(dev)
        dist.barrier()
        if mode == "capacity":
            graphs, ys = [], []
            cap = torch.cuda.Stream(dev)
            cap.wait_stream(stream)
            with torch.cuda.stream(cap):
                for i in range(nl):
                    layers[i].forward(xs[i])
                    gr = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(gr, stream=cap):
                        ys.append(layers[i].forward(xs[i]))
                    graphs.append(gr)
            stream.wait_stream(cap)
            torch.cuda.synchronize(dev)
            dist.barrier()
            for i in range(3):
                graphs[i % nl].replay()
            torch.cuda.synchronize(dev)
            dist.barrier()
            run = lambda i: graphs[i % nl].replay()  # noqa: E731
        else:
            run = lambda i: layers[i % nl].forward(xs[i % nl])  # noqa: E731
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            run(i)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        dist.barrier()
        t = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        if mode == "capacity":
            del graphs, ys
            torch.cuda.synchronize(dev)
            stages = ep_stage_times(eops, layers[0].forward, xs[0], dev, stream, reps=10)
        else:
            samples = []
            names = {m for _, a, b in EP_STAGES for m in (a, b)}
            for i in range(3):
                eops.marks = {m: torch.cuda.Event(enable_timing=True) for m in names}
                eops.recorded = set()
                layers[0].forward(xs[0])
                torch.cuda.synchronize(dev)
                samples.append(_read_marks(eops.marks, eops.recorded))
                eops.marks = None
            stages = _stage_summary(samples, dev)
        dist.barrier()
        out[kind] = {
            "tokens_total": total, "tokens_per_gpu": T, "mode": mode, "steps": steps,
            "ms_per_step": ms, "tokens_per_s": total / (ms * 1e-3),
            "launch": "CUDA graph per weight set (kernels + NCCL)" if mode == "capacity" else
                      "eager (one host read of the row counts per call)",
            "stages_ms": stages,
        }
    return out


def prefill_lengths() -> list[int]:
    """Ragged prompt lengths of the prefill workload: 64 requests uniform in
    [16, 512] (seed 3), about 8k tokens in total."""
    import numpy as np

    return [int(v) for v in np.random.default_rng(3).integers(16, 513, size=64)]


def measure_prefill(dev, lens: list[int], steps: int, warmup: int, seed: int = 3,
                    router_bias: str | None = "zipf", cpu_seconds: float = 0.0) -> dict:
    """One FP8 MoE layer over a prefill batch (all prompts' tokens in one
    call). Expert GEMMs run on the tcgen05 grouped kernel; the roofline
    reports its tensor throughput against the FP8 dense peak (2x the measured
    bf16 GEMM peak). Two weight sets alternate between steps."""
    import numpy as np
    import torch

    from d3moe import _lib, ops, synth

    T = sum(lens)
    lib = _lib.load()
    layers = [synth.make_layer(E, I, H, seed=seed + li, device=dev, router_bias=router_bias)
              for li in range(2)]
    views = [(ops.ExpertView(l.experts), ops.ExpertView(l.shared)) for l in layers]
    ws = ops.moe_workspace(T, TOPK, E, I, H, True, dev)
    gin = torch.Generator(device=dev)
    gin.manual_seed(seed)
    xs = torch.randn((2, T, H), generator=gin, device=dev).to(torch.bfloat16)
    y = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    ids = torch.empty((T, TOPK), dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream

    def step(i, x, ids_out=None):
        lw = layers[i % 2]
        ev, sv = views[i % 2]
        bias = lw.router_bias
        _lib.call("d3_moe_layer", x.data_ptr(), x.stride(0), lw.router.data_ptr(),
                  None if bias is None else bias.data_ptr(), T, TOPK, ctypes.byref(ev.struct),
                  ctypes.byref(sv.struct), y.data_ptr(), None if ids_out is None else ids_out.data_ptr(),
                  None, ws.data_ptr(), ws.numel(), status.data_ptr(), sptr)

    stage_events = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(steps)]
    for evs in stage_events:
        for e in evs:
            e.record(stream)
    stage_arrays = [(ctypes.c_void_p * 5)(*[e._as_parameter_.value for e in evs]) for evs in stage_events]
    with ops.prefill_min_tokens(1024):
        for i in range(warmup):
            step(i, xs[i % 2])
        torch.cuda.synchronize(dev)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index or 0) as clocks:
            start.record(stream)
            for i in range(steps):
                lib.d3_set_stage_events(stage_arrays[i], 5)
                step(i, xs[i % 2], ids if i == 0 else None)
                lib.d3_set_stage_events(None, 0)
            end.record(stream)
            torch.cuda.synchronize(dev)
            ms = start.elapsed_time(end) / steps

            # end to end through the C ABI with host buffers
            hx = xs[0].cpu().pin_memory()
            hy = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
            dx = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
            for i in range(2):
                dx.copy_(hx, non_blocking=True)
                step(i, dx)
                hy.copy_(y, non_blocking=True)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(steps):
                dx.copy_(hx, non_blocking=True)
                step(i, dx)
                hy.copy_(y, non_blocking=True)
            e1.record(stream)
            torch.cuda.synchronize(dev)
            e2e_ms = e0.elapsed_time(e1) / steps
    if int(status.item()) != 0:
        raise RuntimeError(f"device status word {int(status.item())}: a bounded wait timed out")
    gate_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in stage_events)
    down_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in stage_events)
    pre_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in stage_events)
    post_ms = statistics.mean(e[3].elapsed_time(e[4]) for e in stage_events)

    R = T * TOPK + T
    gate_flops = 2.0 * R * (2 * I) * H
    down_flops = 2.0 * R * H * I
    pk = peaks()
    fp8_peak = 2.0 * pk["bf16_tflops"]
    achieved = gate_flops / (gate_ms * 1e-3) / 1e12
    counts = np.bincount(ids.cpu().numpy().reshape(-1), minlength=E)
    ragged = len(lens) > 1
    line = {
        "metric": "fp8_moe_layer_prefill_tokens_per_s",
        "value": T / (ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": 1,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp8_e4m3 x fp8_e4m3 -> f32 (tcgen05 kind::f8f6f4)",
        "data": "synthetic",
        "config": {
            "workload": (f"prefill: {len(lens)} ragged prompts uniform in [16,512] (seed {seed}), T={T} tokens"
                         if ragged else f"prefill: one batch of T={T} tokens (seed {seed})")
                        + ", one MoE layer (H=2048, E=128, I=768, top-8, shared expert)"
                        + (", Zipf(1.1) router bias" if router_bias == "zipf" else
                           ", N(0,1) router bias" if router_bias == "normal" else ", no router bias"),
            "tokens": T,
            "l2": "every step writes > 1 GB of activations/partials (8x the 126 MB L2) and alternates "
                  "two 620 MB weight sets",
            "hottest_expert_pairs": int(counts.max()), "coldest_expert_pairs": int(counts.min()),
        },
        "roofline": {
            "bound": "tensor",
            "kernel": "tc_grouped_kernel<TC_GATE_UP> (tcgen05 FP8 grouped GEMM + SiLU*mul + FP8 requant)",
            "achieved": achieved,
            "peak": fp8_peak,
            "unit": "TFLOP/s",
            "frac": achieved / fp8_peak,
            "peak_source": f"2 x the {pk['source']} bf16 cuBLAS burst peak {pk['bf16_tflops']} TFLOP/s "
                           "(FP8 dense rate = 2x bf16)",
            "traffic": None,
            "algorithmic_flops_per_launch": gate_flops,
            "avg_launch_ms": gate_ms,
            "down_kernel": {"achieved": down_flops / (down_ms * 1e-3) / 1e12, "avg_launch_ms": down_ms,
                            "algorithmic_flops_per_launch": down_flops,
                            "frac": down_flops / (down_ms * 1e-3) / 1e12 / fp8_peak},
            "expert_tflops_whole_layer": (gate_flops + down_flops) / (ms * 1e-3) / 1e12,
            "layer_frac": (gate_flops + down_flops) / (ms * 1e-3) / 1e12 / fp8_peak,
            "stage_ms": {"router_route_permute_quant": pre_ms, "gate_up": gate_ms, "down": down_ms,
                         "combine": post_ms},
        },
        "e2e": {"value": T / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2, "ms_per_step": e2e_ms},
        # router, route, permute (hist, scan, scatter), quant_scatter, gate_up, down, combine
        "gpu_launches": 9 * steps,
        "clocks": clocks.summary(),
    }
    if cpu_seconds > 0:
        line["cpu_baseline"] = cpu_prefill_baseline(layers[0], cpu_seconds)
    del layers, views, ws, xs
    torch.cuda.empty_cache()
    return line


def run_prefill(args, dev) -> None:
    """--workload prefill: the ragged 64-prompt batch (config 4) or, with
    --prefill-tokens, one flat batch."""
    lens = [args.prefill_tokens] if args.prefill_tokens > 0 else prefill_lengths()
    line = measure_prefill(dev, lens, args.steps, args.warmup, seed=3, router_bias="zipf",
                           cpu_seconds=0.0 if args.no_cpu_baseline else args.cpu_seconds)
    print(json.dumps(line), flush=True)


def measure_stack24(dev, replays: int = 1000, warmup: int = 3, T: int = 64, nlayers: int = 24,
                    seed: int = 2) -> dict:
    """a decode step through a stack of `nlayers`
    distinct layers (seed 2), each the FP8 QKV and o_proj GEMVs followed by
    the MoE layer with its fused exit (residual update + RMSNorm feeding the
    next layer), T tokens, per-expert router bias ~ N(0,1) in every layer. The
    whole step is captured in one CUDA graph and replayed `replays` times with
    a fresh N(0,1) input copied in before each replay."""
    import torch

    from d3moe import _lib, ops, synth

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    layers, dense, norms = [], [], []
    for li in range(nlayers):
        lw = synth.make_layer(E, I, H, seed=1000 * seed + li, device=dev, router_bias="normal")
        layers.append((lw, ops.ExpertView(lw.experts), ops.ExpertView(lw.shared)))
        wq, sq = synth.block_quantize(torch.randn((N_QKV, H), generator=g, device=dev) * 0.02)
        wo, so = synth.block_quantize(torch.randn((N_O, H), generator=g, device=dev) * 0.02)
        dense.append((wq, sq, wo, so))
        norms.append((torch.randn(H, generator=g, device=dev) * 0.1).to(torch.bfloat16))
    weight_bytes = sum(l[0].nbytes() for l in layers) + sum(
        t.numel() * t.element_size() for d in dense for t in d)
    lib = _lib.load()
    ws_moe = ops.moe_workspace(T, TOPK, E, I, H, True, dev)
    nb = ctypes.c_size_t()
    lib.d3_fp8_gemv_workspace_size(T, N_QKV, H, ctypes.byref(nb))
    ws_dense = torch.empty(nb.value, dtype=torch.uint8, device=dev)
    x_static = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    residual = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    hbuf = [torch.empty((T, H), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    qkv = torch.empty((T, N_QKV), dtype=torch.bfloat16, device=dev)
    o = torch.empty((T, N_O), dtype=torch.bfloat16, device=dev)
    ids = torch.empty((nlayers, T, TOPK), dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    inputs = torch.randn((8, T, H), generator=g, device=dev).to(torch.bfloat16)

    def gemv(x, wq_, sq_, n, out):
        _lib.call("d3_fp8_gemv", x.data_ptr(), x.stride(0), wq_.data_ptr(), sq_.data_ptr(), T, n, H,
                  out.data_ptr(), out.stride(0), ws_dense.data_ptr(), ws_dense.numel(),
                  status.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)

    def step():
        residual.copy_(x_static)
        h = x_static
        for li in range(nlayers):
            lw, ev, sv = layers[li]
            wq_, sq_, wo_, so_ = dense[li]
            gemv(h, wq_, sq_, N_QKV, qkv)
            gemv(qkv, wo_, so_, N_O, o)
            nxt = hbuf[li % 2]
            _lib.call("d3_moe_layer_add_norm", o.data_ptr(), o.stride(0), lw.router.data_ptr(),
                      lw.router_bias.data_ptr(), T, TOPK, ctypes.byref(ev.struct), ctypes.byref(sv.struct),
                      residual.data_ptr(), norms[li].data_ptr(), ctypes.c_float(1e-6), nxt.data_ptr(),
                      ids[li].data_ptr(), None, ws_moe.data_ptr(), ws_moe.numel(), status.data_ptr(),
                      torch.cuda.current_stream(dev).cuda_stream)
            h = nxt

    x_static.copy_(inputs[0])
    stream = torch.cuda.current_stream(dev)
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(stream)
    with torch.cuda.stream(cap):
        step()  # eager once on the capture stream (first-use attributes set outside capture)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap):
            step()
    stream.wait_stream(cap)
    for i in range(warmup):
        x_static.copy_(inputs[i % len(inputs)])
        graph.replay()
    torch.cuda.synchronize(dev)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index or 0) as clocks:
        g0.record(stream)
        for i in range(replays):
            x_static.copy_(inputs[i % len(inputs)])
            graph.replay()
        g1.record(stream)
        torch.cuda.synchronize(dev)
    ms = g0.elapsed_time(g1) / replays
    if int(status.item()) != 0:
        raise RuntimeError(f"device status word {int(status.item())}: a bounded wait timed out")
    ids_host = ids.cpu().numpy()
    per_layer = [algorithmic_bytes(ids_host[li], T) for li in range(nlayers)]
    step_bytes = sum(p["total"] for p in per_layer)
    pk = peaks()
    achieved = step_bytes / (ms * 1e-3) / 1e9
    out = {
        "config": f"BASELINE configuration 3: {nlayers} distinct layers (seed {seed}) of FP8 QKV[4096x2048] + "
                  f"o_proj[2048x2048] GEMV + MoE layer with fused residual+RMSNorm exit, T={T}, per-expert "
                  "router bias ~ N(0,1) per layer; one CUDA graph per step, replayed",
        "replays": replays,
        "ms_per_step": ms,
        "ms_per_layer": ms / nlayers,
        "tokens_per_s": T / (ms * 1e-3),
        "weight_bytes": weight_bytes,
        "step_bytes": step_bytes,
        "achieved_gbs": achieved,
        "peak_gbs": pk["hbm_gbs"],
        "frac": achieved / pk["hbm_gbs"],
        "mean_active_experts": sum(p["U"] for p in per_layer) / nlayers,
        "min_active_experts": min(p["U"] for p in per_layer),
        "gpu_launches_per_step": nlayers * 11,
        "l2": f"{weight_bytes / 1e9:.1f} GB of weights per step (> 100 x L2)",
        "clocks": clocks.summary(),
    }
    del graph, layers, dense, ws_moe, ws_dense, inputs
    torch.cuda.empty_cache()
    return out


def _load_flashinfer_moe():
    """FlashInfer's trtllm_fp8_block_scale_moe (the reference's decode MoE for
    T > 8, src/drama3/model.py:556-580). Its launcher module is JIT-compiled
    by FlashInfer; the copy prebuilt in baseline/_flashinfer (git-ignored,
    made by baseline/flashinfer_prebuild.py) is loaded, and compiling it here
    is refused (it takes tens of minutes of nvcc), so without the prebuilt
    copy the comparison reports itself unavailable."""
    pre = ROOT / "baseline" / "_flashinfer" / "aot"
    if not (pre / "fused_moe_trtllm_sm100" / "fused_moe_trtllm_sm100.so").exists():
        raise FileNotFoundError("prebuilt FlashInfer MoE launcher missing "
                                "(run baseline/flashinfer_prebuild.py)")
    os.environ["FLASHINFER_DISABLE_JIT"] = "1"
    import flashinfer.jit.env as jit_env

    jit_env.FLASHINFER_AOT_DIR = pre
    from flashinfer.fused_moe import trtllm_fp8_block_scale_moe
    return trtllm_fp8_block_scale_moe


def _moe_float64(q, qs_t, ids, w, w13, s13, w2, s2):
    """float64 value of the routed experts on the dequantised operands, with
    no intermediate quantisation: sum_j w_j * W2_e (silu(G_e x) * (U_e x)),
    W13 in [up | gate] order. The yardstick both FP8 implementations are
    measured against (each rounds its SiLU*mul output to E4M3 its own way)."""
    import torch

    def deq(wq, sc):  # e4m3 [.., N, K] with [.., N/128, K/128] block scales
        wf = wq.to(torch.float64)
        return wf * sc.to(torch.float64).repeat_interleave(128, -2).repeat_interleave(128, -1)

    T, Hh = q.shape
    x = q.to(torch.float64) * qs_t.t().to(torch.float64).repeat_interleave(128, -1)
    out = torch.zeros((T, Hh), dtype=torch.float64, device=q.device)
    for e in torch.unique(ids).tolist():
        rows, slot = (ids == e).nonzero(as_tuple=True)
        h = x[rows] @ deq(w13[e], s13[e]).t()
        up, gate = h.chunk(2, dim=1)
        a = gate / (1.0 + torch.exp(-gate)) * up
        out.index_add_(0, rows, (a @ deq(w2[e], s2[e]).t()) * w[rows, slot].to(torch.float64)[:, None])
    return out


def flashinfer_comparison(dev, sizes=(64, 1344, 8192), iters: int = 20, warmup: int = 3) -> dict:
    """Same-box comparison with the reference's own Blackwell MoE kernel:
    FlashInfer trtllm_fp8_block_scale_moe called exactly as
    src/drama3/model.py:556-580 calls it (fp32 logits, RenormalizeNaive
    routing, MajorK [up | gate] weights, pre-quantised e4m3 hidden states with
    [H/128, T] scales), against this library's drop-in with the same
    arguments (d3moe.flashinfer_compat). Both are captured in CUDA graphs and
    replayed; CUDA events on the launching stream."""
    import torch

    from d3moe import flashinfer_compat as fc, ops, synth

    try:
        fi_moe = _load_flashinfer_moe()
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"flashinfer import failed: {type(e).__name__}: {e}"[:300]}
    ex = synth.make_experts(E, I, H, seed=77, device=dev)
    gate, up = ex.w13_weight.chunk(2, dim=1)
    w13 = torch.cat((up, gate), dim=1).contiguous()
    gs, us = ex.w13_scale_inv.chunk(2, dim=1)
    s13 = torch.cat((us, gs), dim=1).contiguous()
    w2, s2 = ex.w2_weight, ex.w2_scale_inv
    del gate, up, gs, us
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    stream = torch.cuda.current_stream(dev)
    out = {"kernel": "flashinfer.fused_moe.trtllm_fp8_block_scale_moe (trtllm-gen sm100f cubins, "
                     "flashinfer 0.6.11.post2)",
           "ours": "d3moe.flashinfer_compat.trtllm_fp8_block_scale_moe (route_topk + moe_experts_fp8)",
           "what": "routed experts only (the reference's call has no shared expert), E=128 I=768 H=2048 top-8",
           "sizes": {}}

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(dev)
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap):
            with torch.cuda.graph(graph, stream=cap):
                res = fn()
        stream.wait_stream(cap)
        graph.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / iters, res.clone()

    for T in sizes:
        try:
            x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
            q, qs = ops.quant_act_fp8(x, transposed=True)
            logits = torch.randn((T, E), generator=g, device=dev)
            kw = dict(routing_logits=logits, routing_bias=None, hidden_states=q, hidden_states_scale=qs,
                      gemm1_weights=w13, gemm1_weights_scale=s13, gemm2_weights=w2,
                      gemm2_weights_scale=s2, num_experts=E, top_k=TOPK, n_group=None, topk_group=None,
                      intermediate_size=I, local_expert_offset=0, local_num_experts=E,
                      routed_scaling_factor=1.0, routing_method_type=4, use_shuffled_weight=False,
                      weight_layout=0, tune_max_num_tokens=max(4096, T), enable_pdl=None)

            def run_fi():
                r = fi_moe(**kw)
                return r[0] if isinstance(r, (list, tuple)) else r

            fi_ms, fi_y = timed(run_fi)
            our_ms, our_y = timed(lambda: fc.trtllm_fp8_block_scale_moe(**kw))
            d = (fi_y.float() - our_y.float())
            rel = float(d.norm() / our_y.float().norm().clamp_min(1e-30))
            row = {"flashinfer_ms": fi_ms, "ours_ms": our_ms, "speedup_vs_flashinfer": fi_ms / our_ms,
                   "rel_l2_between_outputs": rel}
            if T <= 1344:
                wts, ids = ops.route_topk(logits, TOPK, weights_dtype=torch.bfloat16)
                ref = _moe_float64(q, qs, ids, wts, w13, s13, w2, s2)
                nrm = ref.norm().clamp_min(1e-30)
                row["rel_l2_vs_float64"] = {"flashinfer": float((fi_y.double() - ref).norm() / nrm),
                                            "ours": float((our_y.double() - ref).norm() / nrm)}
            out["sizes"][str(T)] = row
        except Exception as e:  # noqa: BLE001
            out["sizes"][str(T)] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    del ex, w13, s13
    torch.cuda.empty_cache()
    return out


def reference_triton_comparison(dev, sizes=(1, 8), iters: int = 50, warmup: int = 3) -> dict:
    """Same-box comparison with the reference's own Triton decode kernels
    (src/drama3/kernels.py:290-357, small_batch_moe: the routed MoE for
    T <= 8 tokens, model.py:520-530), imported from the unmodified reference
    installed in baseline/_ref. They are hard-wired to the reference model's
    expert shapes (E=256, I=512, H=2048, top-8), so both sides run there. The
    reference's activation quantisers come from Fish Speech's fp8_moe module,
    which is not in this image; this library's byte-identical quantisers
    (d3_quant_act_fp8, d3_silu_mul_quant) stand in for them, and only the two
    reference Triton kernels plus those two quantisers are timed. Ours:
    d3moe.ops.moe_experts (routed experts only) on the same routing. Both are
    replayed from CUDA graphs; CUDA events on the launching stream."""
    import torch

    from d3moe import ops, synth

    ref_root = ROOT / "baseline" / "_ref"
    if not (ref_root / "drama3" / "kernels.py").exists():
        return {"unavailable": "the reference is not installed in baseline/_ref"}
    sys.path.insert(0, str(ref_root))
    try:
        from drama3 import kernels as rk
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference import failed: {type(e).__name__}: {e}"[:300]}
    Er, Ir = 256, 512
    ex = synth.make_experts(Er, Ir, H, seed=91, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(6)
    stream = torch.cuda.current_stream(dev)
    out = {"kernels": "drama3.kernels.expert_up_kernel + expert_down_kernel (Triton, the reference's "
                      "small_batch_moe), quantisers from this library",
           "ours": "d3moe.ops.moe_experts (routed experts only)",
           "shapes": f"E={Er} I={Ir} H={H} top-8 (the reference model's expert shapes)", "sizes": {}}

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(dev)
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap):
            with torch.cuda.graph(graph, stream=cap):
                res = fn()
        stream.wait_stream(cap)
        graph.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / iters, res.clone()

    for T in sizes:
        try:
            x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
            logits = torch.randn((T, Er), generator=g, device=dev).to(torch.bfloat16)
            w, ids = ops.route_topk(logits, TOPK, weights_dtype=torch.bfloat16)

            def run_ref():
                q, qs = ops.quant_act_fp8(x)
                gate_up = torch.empty((T * TOPK, 2 * Ir), dtype=x.dtype, device=dev)
                rk.expert_up_kernel[(T, TOPK, 2 * Ir // 4)](q, qs, ex.w13_weight, ex.w13_scale_inv, ids,
                                                            gate_up, 4, num_warps=4)
                a, sa = ops.silu_mul_quant(gate_up)
                y = torch.empty_like(x)
                rk.expert_down_kernel[(T, H // 4)](a, sa, ex.w2_weight, ex.w2_scale_inv, ids, w, y, 4,
                                                   num_warps=8)
                return y

            ref_ms, ref_y = timed(run_ref)
            our_ms, our_y = timed(lambda: ops.moe_experts(x, ids, w, ex)[0])
            d = ref_y.float() - our_y.float()
            out["sizes"][str(T)] = {"reference_triton_ms": ref_ms, "ours_ms": our_ms,
                                    "speedup_vs_reference": ref_ms / our_ms,
                                    "rel_l2_between_outputs": float(d.norm() / our_y.float().norm())}
        except Exception as e:  # noqa: BLE001
            out["sizes"][str(T)] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    del ex
    torch.cuda.empty_cache()
    return out


def mixed_rows(reuse: bool):
    """Rows of the mixed decode + packed-prefill call of the reference's D64/P1280
    graph (src/drama3/mixed_graph.py:33-50): 64 decode rows (the last 6 padding
    with reserved slots), then 6 prompts of 1121 rows in total and 159 rows of
    padding (the row counts of its mixed-call profile). With `reuse`, the third
    prompt starts with all 240 rows of the second and the fifth with the first
    60 rows of the fourth (300 rows removed), and the MoE runs on the row-reuse
    plan's 1088-row bucket."""
    import numpy as np
    import torch

    from d3moe import mixed

    lens = [256, 240, 300, 120, 128, 77] if reuse else [220, 190, 205, 160, 176, 170]
    assert sum(lens) == 1121
    prompts = []
    for i, n in enumerate(lens):
        p = torch.zeros((n, 11), dtype=torch.int64)
        p[:, 0] = 1 + i
        p[:, 1] = torch.arange(n)
        prompts.append(p)
    if reuse:
        prompts[2][:240] = prompts[1]
        prompts[4][:60] = prompts[3][:60]
    d, cap = 64, 1280
    dslots = list(range(58)) + [MIXED_PAD + 1 + i for i in range(6)]
    slots = mixed.packed_row_slots(dslots, lens, [100 + i for i in range(6)] + [MIXED_PAD + 100], cap)
    plan = mixed.plan_row_reuse(prompts, d, cap, (1088,)) if reuse else None
    if reuse and plan is None:
        raise RuntimeError("the reuse prompts do not fit the 1088-row bucket")
    return np.asarray(slots), plan


MIXED_PAD = 512


def run_mixed(args, dev) -> None:
    """One FP8 MoE layer over the mixed decode + packed-prefill rows (M = 1344),
    with the padding-router rule on the row slots and the layer exit (residual
    update + RMSNorm) fused, through d3_moe_layer_rows. At this M the expert
    GEMMs stream every expert's weights once, so the roofline is HBM."""
    import numpy as np
    import torch

    from d3moe import _lib, ops, synth

    Ex, Ix = args.experts, args.inter
    slots_np, plan = mixed_rows(args.row_reuse)
    M = len(slots_np)
    T = plan.compact_rows if plan is not None else M
    lib = _lib.load()
    layers = [synth.make_layer(Ex, Ix, H, seed=11 + li, device=dev, router_bias="normal")
              for li in range(args.layers)]
    views = [(ops.ExpertView(l.experts), ops.ExpertView(l.shared)) for l in layers]
    ws = ops.moe_workspace(T, TOPK, Ex, Ix, H, True, dev)
    gin = torch.Generator(device=dev)
    gin.manual_seed(5)
    xs = torch.randn((2, M, H), generator=gin, device=dev).to(torch.bfloat16)
    res = torch.randn((M, H), generator=gin, device=dev).to(torch.bfloat16)
    nw = (torch.randn(H, generator=gin, device=dev) * 0.1).to(torch.bfloat16)
    y = torch.empty((M, H), dtype=torch.bfloat16, device=dev)
    ids = torch.empty((T, TOPK), dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    slots = torch.from_numpy(slots_np).to(dev)
    keep = inverse = None
    if plan is not None:
        keep, inverse = plan.keep.to(dev), plan.inverse.to(dev)
        slots = slots.index_select(0, keep)
    rows = _lib.D3Rows(None if keep is None else keep.data_ptr(), M,
                       None if inverse is None else inverse.data_ptr(), M, slots.data_ptr(), 1,
                       MIXED_PAD)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream

    def step(i, x, r, ids_out=None):
        lw = layers[i % len(layers)]
        ev, sv = views[i % len(layers)]
        _lib.call("d3_moe_layer_rows", x.data_ptr(), x.stride(0), lw.router.data_ptr(),
                  lw.router_bias.data_ptr(), T, TOPK, ctypes.byref(ev.struct), ctypes.byref(sv.struct),
                  ctypes.byref(rows), r.data_ptr(), nw.data_ptr(), 1e-6, y.data_ptr(),
                  None if ids_out is None else ids_out.data_ptr(), None, ws.data_ptr(), ws.numel(),
                  status.data_ptr(), sptr)

    stage_events = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    for evs in stage_events:
        for e in evs:
            e.record(stream)
    stage_arrays = [(ctypes.c_void_p * 5)(*[e._as_parameter_.value for e in evs]) for evs in stage_events]
    prev = lib.d3_set_prefill_min_tokens(args.prefill_min) if args.prefill_min > 0 else None
    for i in range(args.warmup):
        step(i, xs[i % 2], res)
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index or 0) as clocks:
        start.record(stream)
        for i in range(args.steps):
            lib.d3_set_stage_events(stage_arrays[i], 5)
            step(i, xs[i % 2], res, ids if i == 0 else None)
            lib.d3_set_stage_events(None, 0)
        end.record(stream)
        torch.cuda.synchronize(dev)
    if int(status.item()) != 0:
        raise RuntimeError(f"device status word {int(status.item())}")
    ms = start.elapsed_time(end) / args.steps
    gate_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in stage_events)
    down_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in stage_events)
    pre_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in stage_events)
    post_ms = statistics.mean(e[3].elapsed_time(e[4]) for e in stage_events)

    # end to end with host buffers: x and the residual in, out and residual back
    hx = xs[0].cpu().pin_memory()
    hr = res.cpu().pin_memory()
    hy = torch.empty((M, H), dtype=torch.bfloat16).pin_memory()
    hr2 = torch.empty((M, H), dtype=torch.bfloat16).pin_memory()
    dx = torch.empty((M, H), dtype=torch.bfloat16, device=dev)
    dr = torch.empty((M, H), dtype=torch.bfloat16, device=dev)

    def e2e_step(i):
        dx.copy_(hx, non_blocking=True)
        dr.copy_(hr, non_blocking=True)
        step(i, dx, dr)
        hy.copy_(y, non_blocking=True)
        hr2.copy_(dr, non_blocking=True)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        e2e_step(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if prev is not None:
        lib.d3_set_prefill_min_tokens(prev)

    counts = np.bincount(ids.cpu().numpy().reshape(-1), minlength=Ex)
    active = int((counts > 0).sum())
    w13_bytes = (2 * Ix) * H + (2 * Ix // 128) * (H // 128) * 4
    w2_bytes = H * Ix + (H // 128) * (Ix // 128) * 4
    R = T * TOPK + T
    gate_bytes = (active + 1) * w13_bytes + R * (H + H // 128 * 4) + R * (Ix + Ix // 128 * 4)
    down_bytes = (active + 1) * w2_bytes + R * (Ix + Ix // 128 * 4) + R * H * 4
    pk = peaks()
    tc = T >= (args.prefill_min if args.prefill_min > 0 else 1024)
    achieved = gate_bytes / (gate_ms * 1e-3) / 1e9
    line = {
        "metric": "fp8_moe_layer_mixed_rows_per_s",
        "value": M / (ms * 1e-3),
        "unit": "rows/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp8_e4m3 x fp8_e4m3 -> f32",
        "data": "synthetic",
        "config": {
            "workload": f"mixed decode + packed prefill: 64 decode rows (6 padding) + 6 prompts of 1121 rows "
                        f"+ 159 padding rows = {M} rows"
                        + (f", row reuse onto {T} compact rows" if plan is not None else "")
                        + f", one MoE layer (H={H}, E={Ex}, I={Ix}, top-8, shared expert) with the fused "
                          "residual + RMSNorm exit, N(0,1) router bias",
            "rows": M, "moe_rows": T, "expert_path": "tcgen05 grouped" if tc else "decode engine",
            "l2": f"{args.layers} weight sets of {Ex * (w13_bytes + w2_bytes) / 1e6:.0f} MB rotated",
        },
        "roofline": {
            "bound": "hbm",
            "kernel": "gate_up (" + ("tc_grouped_kernel<TC_GATE_UP>" if tc else "expert_gemv_kernel<EPI_GATE_UP>") + ")",
            "achieved": achieved,
            "peak": pk["hbm_gbs"],
            "unit": "GB/s",
            "frac": achieved / pk["hbm_gbs"],
            "peak_source": pk["source"],
            "traffic": None,
            "algorithmic_bytes_per_launch": gate_bytes,
            "avg_launch_ms": gate_ms,
            "active_experts": active,
            "down_kernel": {"achieved": down_bytes / (down_ms * 1e-3) / 1e9, "avg_launch_ms": down_ms,
                            "algorithmic_bytes_per_launch": down_bytes},
            "stage_ms": {"router_route_permute_quant": pre_ms, "gate_up": gate_ms, "down": down_ms,
                         "exit_add_norm": post_ms},
        },
        "e2e": {"value": M / (e2e_ms * 1e-3), "unit": "rows/s", "h2d_bytes_per_step": 2 * M * H * 2,
                "d2h_bytes_per_step": 2 * M * H * 2, "ms_per_step": e2e_ms},
        # router, route, permute (hist, scan, scatter), quant_scatter, gate_up, down, exit
        "gpu_launches": 9 * args.steps,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


DENSE_SHAPES = ((9216, 2048, "QKV"), (12352, 2048, "GDN in"), (2048, 4096, "out / o_proj"),
                (4096, 2048, "bench QKV"), (2048, 2048, "bench o_proj"))


def run_dense(args, dev) -> None:
    """The weight-only FP8 GEMV at the reference model's real projection shapes
    (src/drama3/model.py:210-225) and the benchmark's, T in {1, 8, 16, 32, 64}.
    Each shape rotates enough weight copies that every call streams its weight
    from HBM (> 2x the 126 MB L2 per rotation). Roofline: weight + activation
    bytes per call over HBM copy bandwidth."""
    import torch

    from d3moe import _lib, ops

    lib = _lib.load()
    pk = peaks()
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    rows = []
    total_bytes, total_ms = 0.0, 0.0
    launches = 0
    shapes = DENSE_SHAPES
    if args.dense_shape:
        n_, k_ = (int(v) for v in args.dense_shape.split("x"))
        shapes = tuple(sh for sh in DENSE_SHAPES if sh[:2] == (n_, k_)) or ((n_, k_, "custom"),)
    t_values = (args.dense_t,) if args.dense_t else (1, 8, 16, 32, 64)
    for N, K, name in shapes:
        wbytes = N * K + (N // 128) * (K // 128) * 4
        sets = max(2, -(-260_000_000 // wbytes))
        g = torch.Generator(device=dev)
        g.manual_seed(N + K)
        ws_q, ws_s = [], []
        for _ in range(sets):
            # N need not be a multiple of 128 (GDN in: 12352): the registered
            # copy pads the last row block, the GEMV writes N columns
            q, sc = ops.fp8_quantize_weight((torch.randn((N, K), generator=g, device=dev) * 0.02)
                                            .to(torch.bfloat16))
            ws_q.append(q)
            ws_s.append(sc)
        for T in t_values:
            x = torch.randn((T, K), generator=g, device=dev).to(torch.bfloat16)
            y = torch.empty((T, N), dtype=torch.bfloat16, device=dev)
            nb = ctypes.c_size_t()
            lib.d3_fp8_gemv_workspace_size(T, N, K, ctypes.byref(nb))
            ws = torch.empty(nb.value, dtype=torch.uint8, device=dev)

            def call(i):
                _lib.call("d3_fp8_gemv", x.data_ptr(), K, ws_q[i % sets].data_ptr(), ws_s[i % sets].data_ptr(),
                          T, N, K, y.data_ptr(), N, ws.data_ptr(), nb.value, None, sptr)

            for i in range(max(args.warmup, sets)):
                call(i)
            torch.cuda.synchronize(dev)
            # the calls are captured in one CUDA graph and replayed, so the
            # time is the device's (back-to-back GEMVs, as in a captured
            # decode step) rather than the host's launch rate
            cap = torch.cuda.Stream(dev)
            cap.wait_stream(stream)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(cap):
                with torch.cuda.graph(graph, stream=cap):
                    for i in range(args.steps):
                        _lib.call("d3_fp8_gemv", x.data_ptr(), K, ws_q[i % sets].data_ptr(),
                                  ws_s[i % sets].data_ptr(), T, N, K, y.data_ptr(), N, ws.data_ptr(),
                                  nb.value, None, cap.cuda_stream)
            stream.wait_stream(cap)
            graph.replay()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            ms = e0.elapsed_time(e1) / args.steps
            del graph
            nbytes = wbytes + T * K * 2 + T * N * 2
            total_bytes += nbytes * args.steps
            total_ms += ms * args.steps
            launches += 2 * args.steps
            rows.append({"shape": f"{N}x{K} ({name})", "T": T, "us": round(ms * 1e3, 2),
                         "GBps": round(nbytes / (ms * 1e-3) / 1e9, 1),
                         "frac": round(nbytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 3)})
        del ws_q, ws_s
        torch.cuda.empty_cache()
    achieved = total_bytes / (total_ms * 1e-3) / 1e9
    line = {
        "metric": "fp8_dense_gemv_bytes_per_s",
        "value": achieved,
        "unit": "GB/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total_ms / (args.steps * len(rows)),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3 weights x bf16 activations split exactly into two e4m3 terms -> f32 "
                 "(tcgen05 kind::f8f6f4), bf16 out",
        "data": "synthetic",
        "config": {"workload": "weight-only FP8 GEMV, real Drama-3 projection shapes and the benchmark's, "
                               "T in {1,8,16,32,64}, weights rotated over > 260 MB per shape",
                   "per_shape": rows},
        "roofline": {"bound": "hbm", "kernel": "dense_tc_kernel (tcgen05 weight-only FP8 GEMV, + dense_split)",
                     "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / pk["hbm_gbs"], "peak_source": pk["source"], "traffic": None},
        "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)


def cpu_prefill_baseline(layer, seconds: float) -> dict:
    """Oracle port on the host cores over a bounded slice of the prefill batch
    (the first prompts, 512 tokens), repeated until `seconds` have passed."""
    import numpy as np
    import torch

    sys.path.insert(0, str(ROOT))
    from oracle import moe_oracle as O

    def cpu_ex(ex):
        return O.Experts(ex.w13_weight.view(torch.uint8).cpu().numpy(), ex.w13_scale_inv.cpu().numpy(),
                         ex.w2_weight.view(torch.uint8).cpu().numpy(), ex.w2_scale_inv.cpu().numpy())

    ex, sh = cpu_ex(layer.experts), cpu_ex(layer.shared)
    router = layer.router.float().cpu().numpy()
    bias = None if layer.router_bias is None else layer.router_bias.float().cpu().numpy()
    Ts = 512
    x = O.bf16_round(np.random.default_rng(3).standard_normal((Ts, H)).astype(np.float32))
    steps, t0 = 0, time.perf_counter()
    while True:
        O.moe_layer(x, router, ex, sh, TOPK, bias=bias)
        steps += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    threads = int(os.environ.get("OMP_NUM_THREADS", "0")) or os.cpu_count()
    return {"value": Ts * steps / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{steps} x MoE layer over {Ts} prefill tokens (numpy, BLAS threads={threads}), {dt:.1f} s"}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=64, help="decode tokens per GPU per step")
    ap.add_argument("--layers", type=int, default=4, help="weight sets rotated across steps")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "mixed", "dense"],
                    help="decode: the default 64-token step; prefill: ~8k ragged tokens, one GPU; "
                         "mixed: 64 decode + 1280 packed prompt rows in one call, one GPU; "
                         "dense: the FP8 GEMV at the real projection shapes, one GPU")
    ap.add_argument("--row-reuse", action="store_true", help="mixed: run the MoE on the row-reuse bucket")
    ap.add_argument("--experts", type=int, default=E, help="mixed: routed experts")
    ap.add_argument("--inter", type=int, default=I, help="mixed: expert intermediate size")
    ap.add_argument("--prefill-min", type=int, default=0,
                    help="mixed: MoE rows from which the tcgen05 path runs (0: the library default)")
    ap.add_argument("--prefill-tokens", type=int, default=0,
                    help="prefill: a flat batch of this many tokens instead of the ragged 64-prompt batch")
    ap.add_argument("--eager", action="store_true",
                    help="with N > 1: launch the step op by op instead of replaying its CUDA graph")
    ap.add_argument("--dense-shape", default="",
                    help="dense: one weight shape NxK (e.g. 4096x2048) instead of the list")
    ap.add_argument("--dense-t", type=int, default=0, help="dense: one token count instead of 1..64")
    ap.add_argument("--no-extras", action="store_true",
                    help="decode line only: skip the prefill, 24-layer stack and FlashInfer objects")
    ap.add_argument("--stack-replays", type=int, default=1000,
                    help="replays of the 24-layer stack step (BASELINE configuration 3)")
    ap.add_argument("--replicas", action="store_true",
                    help="with N > 1: independent full-layer replicas instead of expert parallelism")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
        return

    import numpy as np
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.workload == "dense":
        if world > 1:
            raise SystemExit("--workload dense runs on one GPU")
        run_dense(args, dev)
        return
    if args.workload in ("prefill", "mixed"):
        if world > 1:
            raise SystemExit(f"--workload {args.workload} runs on one GPU")
        if args.workload == "mixed":
            if args.layers == 4:
                args.layers = 2
            run_mixed(args, dev)
        else:
            run_prefill(args, dev)
        return
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        if not args.replicas:
            run_ep(args, world, rank, local, dev)
            dist.destroy_process_group()
            return

    from d3moe import _lib, ops, synth

    T = args.tokens
    lib = _lib.load()
    layers, dense = [], []
    for li in range(args.layers):
        seed = 1000 * rank + li
        layers.append(synth.make_layer(E, I, H, seed=seed, device=dev))
        g = torch.Generator(device=dev)
        g.manual_seed(seed + 77)
        wq, sq = synth.block_quantize(torch.randn((N_QKV, H), generator=g, device=dev) * 0.02)
        wo, so = synth.block_quantize(torch.randn((N_O, H), generator=g, device=dev) * 0.02)
        dense.append((wq, sq, wo, so))
    views = [(ops.ExpertView(l.experts), ops.ExpertView(l.shared)) for l in layers]
    ws_moe = ops.moe_workspace(T, TOPK, E, I, H, True, dev)
    nb = ctypes.c_size_t()
    lib.d3_fp8_gemv_workspace_size(T, N_QKV, H, ctypes.byref(nb))
    ws_dense = torch.empty(nb.value, dtype=torch.uint8, device=dev)
    nsteps_total = args.warmup + args.steps
    gin = torch.Generator(device=dev)
    gin.manual_seed(4242 + rank)
    xs = torch.randn((args.layers * 4, T, H), generator=gin, device=dev).to(torch.bfloat16)
    qkv = torch.empty((T, N_QKV), dtype=torch.bfloat16, device=dev)
    o = torch.empty((T, N_O), dtype=torch.bfloat16, device=dev)
    y = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    ids_all = torch.empty((args.steps, T, TOPK), dtype=torch.int64, device=dev)
    wts = torch.empty((T, TOPK), dtype=torch.bfloat16, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream

    def gemv(x, x_ld, wq, sq, n, out):
        _lib.call("d3_fp8_gemv", x.data_ptr(), x_ld, wq.data_ptr(), sq.data_ptr(), T, n, H,
                  out.data_ptr(), out.stride(0), ws_dense.data_ptr(), ws_dense.numel(),
                  status.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)

    def step(i: int, x: torch.Tensor, ids_buf, dense_events=None):
        li = i % args.layers
        wq, sq, wo_, so_ = dense[li]
        if dense_events:
            dense_events[0].record(stream)
        gemv(x, x.stride(0), wq, sq, N_QKV, qkv)
        if dense_events:
            dense_events[1].record(stream)
        gemv(qkv, qkv.stride(0), wo_, so_, N_O, o)  # first 2048 columns of qkv, row stride 4096
        lw = layers[li]
        ev, sv = views[li]
        _lib.call("d3_moe_layer", o.data_ptr(), o.stride(0), lw.router.data_ptr(), None, T, TOPK,
                  ctypes.byref(ev.struct), ctypes.byref(sv.struct), y.data_ptr(),
                  None if ids_buf is None else ids_buf.data_ptr(), wts.data_ptr(),
                  ws_moe.data_ptr(), ws_moe.numel(), status.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)

    # by hand, used when the captured step graph cannot be read: (activation split + tcgen05 GEMV)
    # x 2; router, route, permute + quant, gate_up, down, combine
    launches_per_step = 2 * 2 + 6

    # per-step stage events (gate_up / down engine launches) inside the timed region
    stage_events = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    for evs in stage_events:
        for e in evs:
            e.record(stream)  # materialise the cudaEvent_t handles
    stage_arrays = [(ctypes.c_void_p * 5)(*[e._as_parameter_.value for e in evs]) for evs in stage_events]
    dense_events = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]

    for i in range(args.warmup):
        step(i, xs[i % len(xs)], None)
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # one clock record over every timed region below: the eager loop, the
    # graph replays that give `value`, and the end-to-end loop
    clocks = ClockSampler(local)
    clocks.__enter__()
    start.record(stream)
    for i in range(args.steps):
        lib.d3_set_stage_events(stage_arrays[i], 5)
        step(args.warmup + i, xs[(args.warmup + i) % len(xs)], ids_all[i], dense_events[i])
        lib.d3_set_stage_events(None, 0)
    end.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    ms = start.elapsed_time(end) / args.steps
    gate_ms = [evs[1].elapsed_time(evs[2]) for evs in stage_events]
    down_ms = [evs[2].elapsed_time(evs[3]) for evs in stage_events]
    moe_ms = [evs[0].elapsed_time(evs[4]) for evs in stage_events]
    qkv_ms = [de[0].elapsed_time(de[1]) for de in dense_events]
    oproj_ms = [de[1].elapsed_time(se[0]) for de, se in zip(dense_events, stage_events)]
    pre_ms = [se[0].elapsed_time(se[1]) for se in stage_events]
    post_ms = [se[3].elapsed_time(se[4]) for se in stage_events]
    ids_host = ids_all.cpu().numpy()
    if int(status.item()) != 0:
        raise RuntimeError(f"device status word {int(status.item())}: a bounded wait timed out")
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    eager_ms = ms

    # ---- the step captured in one CUDA graph per weight set (the reference
    # captures its decode step, src/drama3/engine.py:84-92); the timed value
    # replays them. The eager loop above gives the per-kernel stage times.
    graphs, x_static = [], []
    step_kernels = None
    if not args.eager:
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            for li in range(args.layers):
                xb = xs[li % len(xs)].clone()
                g = torch.cuda.CUDAGraph(keep_graph=(li == 0))
                with torch.cuda.graph(g, stream=cap):
                    step(li, xb, None)
                graphs.append(g)
                x_static.append(xb)
        stream.wait_stream(cap)
        step_kernels = graph_kernels(graphs[0])
        # the replay must reproduce the eager step bit for bit
        step(0, x_static[0], None)
        y_eager = y.clone()
        y.zero_()
        graphs[0].replay()
        torch.cuda.synchronize(dev)
        if not torch.equal(y, y_eager):
            raise RuntimeError("CUDA graph replay differs from the eager step")
        for i in range(args.warmup):
            graphs[i % args.layers].replay()
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for i in range(args.steps):
            li = i % args.layers
            x_static[li].copy_(xs[(args.warmup + i) % len(xs)])
            graphs[li].replay()
        g1.record(stream)
        torch.cuda.synchronize(dev)
        ms = g0.elapsed_time(g1) / args.steps
        if world > 1:
            torch.distributed.barrier()
            t = torch.tensor([ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        if int(status.item()) != 0:
            raise RuntimeError(f"device status word {int(status.item())}: a bounded wait timed out")

    # ---- the MoE layer alone, captured and replayed the same way (no stage
    # events between its kernels, so their launches overlap as in the step):
    # the layer time the HBM roofline target is quoted on
    layer_graph_ms = None
    if not args.eager:
        lgraphs = []
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            for li in range(args.layers):
                g = torch.cuda.CUDAGraph()
                lw = layers[li]
                ev, sv = views[li]
                with torch.cuda.graph(g, stream=cap):
                    _lib.call("d3_moe_layer", o.data_ptr(), o.stride(0), lw.router.data_ptr(), None, T,
                              TOPK, ctypes.byref(ev.struct), ctypes.byref(sv.struct), y.data_ptr(), None,
                              wts.data_ptr(), ws_moe.data_ptr(), ws_moe.numel(), status.data_ptr(),
                              cap.cuda_stream)
                lgraphs.append(g)
        stream.wait_stream(cap)
        for i in range(args.warmup):
            lgraphs[i % args.layers].replay()
        torch.cuda.synchronize(dev)
        l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0.record(stream)
        for i in range(args.steps):
            lgraphs[i % args.layers].replay()
        l1.record(stream)
        torch.cuda.synchronize(dev)
        layer_graph_ms = l0.elapsed_time(l1) / args.steps
        del lgraphs

    # ---- end-to-end through the C ABI with host buffers (pinned H2D + D2H per step)
    hx = torch.randn((T, H)).to(torch.bfloat16).pin_memory()
    hy = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
    dx = torch.empty((T, H), dtype=torch.bfloat16, device=dev)

    def e2e_step(i):
        if graphs:
            li = i % args.layers
            x_static[li].copy_(hx, non_blocking=True)
            graphs[li].replay()
        else:
            dx.copy_(hx, non_blocking=True)
            step(i, dx, None)
        hy.copy_(y, non_blocking=True)

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        e2e_step(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / args.steps
    clocks.__exit__(None, None, None)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())

    pk = peaks()
    per_step = [algorithmic_bytes(ids_host[i], T) for i in range(args.steps)]
    gate_bytes = statistics.mean(p["gate_up"] for p in per_step)
    down_bytes = statistics.mean(p["down"] for p in per_step)
    total_bytes = statistics.mean(p["total"] for p in per_step)
    gate_avg = statistics.mean(gate_ms)
    down_avg = statistics.mean(down_ms)
    achieved = gate_bytes / (gate_avg * 1e-3) / 1e9
    line = {
        "metric": "fp8_moe_layer_decode_tokens_per_s",
        "value": T * world / (ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp8_e4m3 x fp8_e4m3 -> f32 (experts); fp8 weights x bf16 (dense)",
        "data": "synthetic",
        "config": {
            "workload": f"decode T={T}/GPU: FP8 QKV[4096x2048] + o_proj[2048x2048] weight-only GEMV + "
                        "MoE layer (H=2048, E=128, I=768, top-8, shared expert), 128x128 fp32 block scales",
            "tokens_per_gpu": T, "weight_sets_rotated": args.layers,
            "l2": f"inputs larger than L2: {args.layers} weight sets x "
                  f"{layers[0].nbytes() / 1e6:.0f} MB rotated per step",
            "parallelism": "replicas" if world > 1 else "single",
            "launch": "one CUDA graph per weight set, replayed" if graphs else "eager",
            "eager_ms_per_step": eager_ms,
        },
        "roofline": {
            "bound": "hbm",
            "kernel": "expert_gemv_kernel<EPI_GATE_UP> (gate_up + SiLU*mul + FP8 requant)",
            "achieved": achieved,
            "peak": pk["hbm_gbs"],
            "unit": "GB/s",
            "frac": achieved / pk["hbm_gbs"],
            "peak_source": pk["source"],
            # not measured in this run: dram__bytes_read.sum + dram__bytes_write.sum
            # of one gate_up launch from the ncu capture named in traffic_source
            "traffic": GATE_UP_TRAFFIC_BYTES,
            "traffic_source": GATE_UP_TRAFFIC_SOURCE,
            "algorithmic_bytes_per_launch": gate_bytes,
            "avg_launch_ms": gate_avg,
            "down_kernel": {"achieved": down_bytes / (down_avg * 1e-3) / 1e9, "avg_launch_ms": down_avg,
                            "algorithmic_bytes_per_launch": down_bytes},
            "moe_layer_ms": statistics.mean(moe_ms),
            "moe_layer_graph_ms": layer_graph_ms,
            "moe_layer_frac": (None if layer_graph_ms is None else
                               (gate_bytes + down_bytes) / (layer_graph_ms * 1e-3) / 1e9 / pk["hbm_gbs"]),
            "stage_ms": {"qkv_gemv": statistics.mean(qkv_ms), "o_proj_gemv": statistics.mean(oproj_ms),
                         "router_route_permute_quant": statistics.mean(pre_ms),
                         "gate_up": gate_avg, "down": down_avg, "combine": statistics.mean(post_ms)},
            "step_bytes": total_bytes,
            "step_achieved_gbs": total_bytes / (ms * 1e-3) / 1e9,
            "mean_active_experts": statistics.mean(p["U"] for p in per_step),
        },
        "e2e": {"value": T * world / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": hx.numel() * 2, "d2h_bytes_per_step": hy.numel() * 2,
                "ms_per_step": e2e_ms},
        "gpu_launches": (step_kernels["ours"] if step_kernels else launches_per_step) * args.steps,
        "graph_kernels_per_step": step_kernels,
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, str(ROOT))
        from oracle import moe_oracle as O

        def cpu_ex(ex):
            return O.Experts(ex.w13_weight.view(torch.uint8).cpu().numpy(), ex.w13_scale_inv.cpu().numpy(),
                             ex.w2_weight.view(torch.uint8).cpu().numpy(), ex.w2_scale_inv.cpu().numpy())

        wq, sq, wo_, so_ = dense[0]
        weights_cpu = (wq.view(torch.uint8).cpu().numpy(), sq.cpu().numpy(), wo_.view(torch.uint8).cpu().numpy(),
                       so_.cpu().numpy(), layers[0].router.float().cpu().numpy(), cpu_ex(layers[0].experts),
                       cpu_ex(layers[0].shared))
        line["cpu_baseline"] = cpu_baseline(T, args.cpu_seconds, weights_cpu)
    if world == 1 and not args.no_extras:
        # the metric's prefill half, BASELINE configuration 3 and the same-box
        # comparison with the reference's FlashInfer kernel, on this GPU
        del graphs, layers, dense, views, ws_moe, xs
        torch.cuda.empty_cache()
        line["prefill"] = {
            "T8192": measure_prefill(dev, [8192], 10, 3, seed=4, router_bias=None,
                                     cpu_seconds=0.0 if args.no_cpu_baseline else 6.0),
            "config4": measure_prefill(dev, prefill_lengths(), 10, 3, seed=3, router_bias="zipf"),
        }
        line["stack24"] = measure_stack24(dev, replays=args.stack_replays)
        line["vs_flashinfer"] = flashinfer_comparison(dev)
        line["vs_reference_triton"] = reference_triton_comparison(dev)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
