#!/usr/bin/env python
"""NVFP4 MoE layer benchmark on B200 (BASELINE metric: NVFP4 MoE layer tokens/s + HBM GB/s).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ftb|reference]

N=1 workload: BASELINE config 1 decode at T=64 tokens (H=4096, I=1536, 256 routed experts,
top-8, one shared expert; the largest decode batch of config 1). A step = one layer forward:
softmax top-k routing of the step's logits -> sort -> gate_up GEMV + SwiGLU -> down GEMV ->
combine + shared expert, through the C-ABI library. Four layers with distinct weights
(4 x 2.7 GB > L2) are rotated so no step reads weights another step left in L2.
N>1 (torchrun): BASELINE config 3, expert-parallel decode, T=64 tokens per rank, experts
sharded contiguously; tokens and outputs move over NVLink peer memory inside the layer's own
kernels (--ep-transport p2p, default) or by NCCL all_to_all (--ep-transport nccl, the
collective-library baseline); value = tokens/s of the whole box.
Timed steps replay one CUDA graph per layer (--no-graphs: eager launches).
The line's "prefill" object is BASELINE config 2 on one GPU: a T=4096 prefill chunk through
the tcgen05 grouped GEMMs (ftb.moe_prefill), with its own tensor-pipe roofline (--no-prefill
skips it).

Prints one JSON line (rank 0). `--impl reference` times the reference's CPU MoE executor
semantics (the C++ restatement in oracle/, the reference's own executor being unbuildable)
on the host cores for the same metric and config.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "freetoken-ox-boost_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

H, I, E, TOPK = 4096, 1536, 256, 8
METRIC = "NVFP4 MoE layer tokens/s (decode, BASELINE config 1/3)"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ftb", "reference"], default="ftb")
    ap.add_argument("--tokens", type=int, default=64, help="tokens per step (per rank)")
    ap.add_argument("--layers", type=int, default=4, help="distinct layer banks rotated")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the T=1/4/16 decode sweep")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the config 2 prefill measurement (T=--prefill-tokens)")
    ap.add_argument("--prefill-tokens", type=int, default=4096)
    ap.add_argument("--no-graphs", dest="graphs", action="store_false",
                    help="time eager launches instead of CUDA-graph replay")
    ap.add_argument("--ep-transport", choices=["p2p", "nccl"], default="p2p",
                    help="expert-parallel transport for --gpus > 1")
    ap.add_argument("--stack", type=int, default=0,
                    help="BASELINE config 4 (--gpus > 1): a step runs this many distinct stacked "
                         "layers (60 in the config) back to back, --tokens per GPU")
    ap.add_argument("--routing", choices=["flat", "zipf"], default="flat",
                    help="config 4 routing: flat N(0,1) logits, or + log Zipf(1.1) popularity")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback (6.65 TB/s, earlier measurement on this pool)"


def measured_tensor_peaks():
    """(burst, sustained) dense bf16 TFLOP/s and where they come from."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return (float(d["bf16_tflops"]), float(d["bf16_tflops_sustained"]),
                "measured (MEASURED_PEAKS.json bf16_tflops / bf16_tflops_sustained, cuBLAS)")
    except (OSError, KeyError, ValueError):
        return 1590.0, 1400.0, "fallback (1.59 / 1.4 PFLOP/s, earlier measurement on this pool)"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled every 10 ms through NVML while the
    timed region runs (the data nvidia-smi's clocks/clocks_event_reasons query reports).
    The GPU is addressed by the UUID of the CUDA device, so device renumbering is harmless."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, torch, device: int = 0):
        self.samples, self.reasons, self.err = [], set(), None
        self.stop_flag = False
        self.thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            if not uuid.startswith("GPU-"):
                uuid = "GPU-" + uuid
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001 - report, never fail the bench
            self.nvml, self.err = None, f"nvml unavailable: {e}"

    def _run(self):
        import threading  # noqa: F401

        while not self.stop_flag:
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h,
                                                                    self.nvml.NVML_CLOCK_SM))
                r = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception as e:  # noqa: BLE001
                self.err = str(e)
                return
            time.sleep(0.01)

    def start(self):
        import threading

        if self.nvml is None:
            return
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()
        time.sleep(0.02)

    def stop(self) -> dict:
        if self.nvml is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": self.err}
        self.stop_flag = True
        self.thread.join(timeout=2)
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None,
               "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
               "samples": len(self.samples), "source": "NVML, 10 ms, during the timed region"}
        if self.err:
            out["note"] = self.err
        return out


def gate_up_bytes_per_expert(h=H, i=I):
    return 2 * i * (h // 2 + h // 16 + 2)


def workload_config(args, world: int) -> dict:
    """The workload this run measures, printed identically by both arms (ftb and reference)."""
    if world > 1:
        work = (f"config 3 expert-parallel decode: T={args.tokens} tokens per GPU x {world} GPUs, "
                f"H{H} I{I} E{E} top{TOPK} +1 shared expert, softmax-renorm router, "
                f"{E // world} experts per GPU")
    else:
        work = (f"config 1 decode T={args.tokens}: H{H} I{I} E{E} top{TOPK} +1 shared expert, "
                f"softmax-renorm router")
    return {"workload": work, "tokens_per_step": args.tokens * world, "hidden": H,
            "inter": I, "experts": E, "top_k": TOPK, "shared_experts": 1,
            "l2": "inputs larger than L2: distinct 2.7 GB layer banks rotated across steps "
                  "(GPU arm); the CPU arm streams its banks from DRAM"}


def host_cpu() -> dict:
    """CPU model, logical CPUs usable by this process and physical cores (from /proc/cpuinfo)."""
    model, cores = None, set()
    phys = core = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                k, _, v = line.partition(":")
                k, v = k.strip(), v.strip()
                if k == "model name" and model is None:
                    model = v
                elif k == "physical id":
                    phys = v
                elif k == "core id":
                    core = v
                elif not k and phys is not None:
                    cores.add((phys, core))
                    phys = core = None
        if phys is not None:
            cores.add((phys, core))
    except OSError:
        pass
    logical = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return {"cpu_model": model, "logical_cpus": logical,
            "physical_cores": len(cores) or None}


class Layers:
    """L distinct synthetic layers on the GPU plus per-layer step inputs."""

    def __init__(self, torch, ftb, synth, n_layers: int, tokens: int, experts, device, seed0=0):
        self.torch, self.ftb = torch, ftb
        self.T = tokens
        self.banks, self.shared, self.inputs, self.outs = [], [], [], []
        for l in range(n_layers):
            bank = synth.make_bank(E, H, I, seed=seed0 + l, device=device)
            if experts is not None:  # this rank's contiguous expert shard
                bank = bank.select(experts)
            self.banks.append(bank)
            self.shared.append(synth.make_shared(H, I, seed=seed0 + l, device=device))
            self.inputs.append(synth.make_inputs(tokens, H, E, seed=1000 + seed0 + l,
                                                 device=device))
            self.outs.append(torch.empty(tokens, H, dtype=torch.bfloat16, device=device))
        self.routes = [ftb.fused_topk(None, inp.logits, TOPK, True) for inp in self.inputs]
        self.uniq = [int(torch.unique(r[1]).numel()) for r in self.routes]

    def step(self, i: int):
        l = i % len(self.banks)
        inp = self.inputs[l]
        w, ids = self.ftb.fused_topk(None, inp.logits, TOPK, True)
        self.ftb.moe_decode(inp.x, self.banks[l], w, ids, shared=self.shared[l], out=self.outs[l])


def time_steps(torch, fn, steps: int) -> float:
    """Device time of `steps` calls (CUDA events on the current stream), ms per step. The
    host time spent issuing them is kept in time_steps.host_ms (ms per step)."""
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    t0 = time.perf_counter()
    for i in range(steps):
        fn(i)
    time_steps.host_ms = (time.perf_counter() - t0) * 1e3 / steps
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


time_steps.host_ms = None


def graph_steps(torch, fn, n: int):
    """Captures fn(0) .. fn(n-1) (one step per distinct layer, after eager warm-up) into CUDA
    graphs and returns a step function that replays graph i % n: the same launches with the
    host's per-launch work removed."""
    graphs = []
    torch.cuda.synchronize()
    for l in range(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn(l)
        graphs.append(g)
    torch.cuda.synchronize()

    def step(i):
        graphs[i % n].replay()

    step.graphs = graphs
    return step


def kernel_times(ftb_lib, torch, fn, steps: int, launches_per_step: int = 64):
    """Per-launch durations of the library's kernels over `steps` calls (CUDA events on the
    launching stream, recorded by the library around each launch)."""
    import ctypes

    lib = ftb_lib.load()
    torch.cuda.synchronize()
    lib.ftb_profile_begin()
    for i in range(steps):
        fn(i)
    torch.cuda.synchronize()
    cap = launches_per_step * steps + 64
    ids = (ctypes.c_int32 * cap)()
    ms = (ctypes.c_float * cap)()
    n = lib.ftb_profile_end(ids, ms, cap)
    if n < 0:
        raise RuntimeError(f"ftb_profile_end failed ({n})")
    out = {}
    for k in range(min(n, cap)):
        out.setdefault(ftb_lib.KERNEL_NAMES.get(ids[k], str(ids[k])), []).append(ms[k])
    return out


def e2e_steps(torch, ftb, layers: "Layers", steps: int):
    """End to end through the public API with host buffers: each step copies its x and logits
    from pinned host memory, runs routing + the layer, and reads the output back to host."""
    T = layers.T
    hx = [inp.x.cpu().pin_memory() for inp in layers.inputs]
    hl = [inp.logits.cpu().pin_memory() for inp in layers.inputs]
    hout = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    dx = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    dl = torch.empty(T, E, dtype=torch.float32, device="cuda")
    dout = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")

    def one(i):
        l = i % len(layers.banks)
        dx.copy_(hx[l], non_blocking=True)
        dl.copy_(hl[l], non_blocking=True)
        w, ids = ftb.fused_topk(dx, dl, TOPK, True)
        ftb.moe_decode(dx, layers.banks[l], w, ids, shared=layers.shared[l], out=dout)
        hout.copy_(dout, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(3):
        one(i)
    t0 = time.perf_counter()
    for i in range(steps):
        one(i)
    dt = (time.perf_counter() - t0) / steps
    return dt, T * H * 2 + T * E * 4, T * H * 2


def cpu_baseline(torch, layers: "Layers", budget_s: float):
    """The C++ CPU restatement of the layer (oracle/cpu_moe.cpp) on all host threads, on a
    bounded sample: whole T-token steps of layer 0 until ~budget_s of CPU time."""
    from oracle import cpu_moe

    bank = layers.banks[0].numpy()
    shared = layers.shared[0].numpy()
    inp = layers.inputs[0]
    x_bits = inp.x.cpu().contiguous().view(torch.int16).numpy().view("uint16")
    w, ids = layers.routes[0]
    w, ids = w.cpu().numpy(), ids.cpu().numpy()
    threads = cpu_moe.max_threads()
    cpu_moe.moe_layer(x_bits, bank, w, ids, shared, nthreads=threads)  # warm (page in)
    times = []
    t_start = time.perf_counter()
    while not times or (time.perf_counter() - t_start < budget_s and len(times) < 20):
        t0 = time.perf_counter()
        cpu_moe.moe_layer(x_bits, bank, w, ids, shared, nthreads=threads)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": layers.T / t, "unit": "tokens/s", "cores": threads,
            "kind": "port", **host_cpu(),
            "sample": f"{len(times)} full T={layers.T} layer steps (config 1 shape, layer 0, "
                      f"{layers.uniq[0]} routed experts + shared), median {t * 1e3:.0f} ms; "
                      f"avx512={cpu_moe.has_avx512()}"}


def roofline_entry(kt: dict, layers: "Layers", steps: int):
    """Dominant kernel (gate_up GEMV): algorithmic bytes per launch = (distinct routed experts
    + shared) x gate_up bytes per expert; achieved = total bytes / total event time."""
    peak, peak_src = measured_peaks()
    gu = kt.get("gate_up_gemv", [])
    n = len(gu)
    if n == 0:
        return None
    byts = sum((layers.uniq[i % len(layers.uniq)] + 1) * gate_up_bytes_per_expert()
               for i in range(n))
    achieved = byts / (sum(gu) * 1e-3) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "decode_gate_up_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            d = json.load(f)
        # ncu dram bytes per streamed expert, scaled to this workload's experts per launch
        per_unit = d.get("dram_bytes_per_expert")
        if per_unit:
            traffic = per_unit * (sum(layers.uniq) / len(layers.uniq) + 1)
    return {"kernel": "gate_up_gemv (k_gemv_tma<0>)", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": peak_src,
            "traffic": traffic, "algorithmic_bytes_per_launch": byts / n,
            "launches": n, "avg_launch_ms": sum(gu) / n}


def run_ftb_single(args, torch):
    import ftb
    from ftb import _lib, synth

    torch.cuda.set_device(0)
    layers = Layers(torch, ftb, synth, args.layers, args.tokens, None, "cuda")
    for i in range(max(3, args.warmup)):
        layers.step(i)
    torch.cuda.synchronize()
    timed = graph_steps(torch, layers.step, args.layers) if args.graphs else layers.step
    for i in range(max(3, args.warmup)):
        timed(i)
    torch.cuda.synchronize()
    clocks = ClockSampler(torch, 0)
    clocks.start()
    ms = time_steps(torch, timed, args.steps)
    host_ms = time_steps.host_ms
    clk = clocks.stop()
    kt = kernel_times(_lib, torch, layers.step, min(args.steps, 64))
    e2e_dt, h2d, d2h = e2e_steps(torch, ftb, layers, min(args.steps, 64))
    value = args.tokens * 1e3 / ms
    per_exp = ftb.bank_bytes_per_expert(H, I)
    layer_bytes = statistics.mean((u + 1) * per_exp for u in layers.uniq) + 2 * args.tokens * H * 2
    out = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "nvfp4 (e2m1+e4m3) x bf16 -> fp32 accumulate, bf16 out",
        "data": "synthetic: seeded NVFP4 banks and N(0,1) logits/activations per BASELINE config 1",
        "config": workload_config(args, 1),
        "run": {"layers_rotated": args.layers,
                "routed_experts_per_step": round(statistics.mean(layers.uniq), 1),
                "launch": "CUDA graph per layer (route + layer), replayed" if args.graphs
                          else "eager launches",
                "host_issue_ms_per_step": round(host_ms, 4)},
        "layer_hbm_gbs": round(layer_bytes / (ms * 1e-3) / 1e9, 1),
        "roofline": roofline_entry(kt, layers, args.steps),
        "kernels_ms": {k: round(statistics.mean(v), 4) for k, v in kt.items()},
        "e2e": {"value": round(args.tokens / e2e_dt, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": 5 * args.steps,  # route_topk, sort_stage, gate_up, down, combine
        "clocks": clk,
    }
    if not args.no_sweep:
        out["decode_sweep"] = sweep_decode(torch, ftb, layers, args)
    if not args.no_prefill:
        out["prefill"] = bench_prefill(torch, ftb, layers, args)
        out["prefill_fp4"] = bench_prefill_fp4(torch, ftb, layers, args)
    if not args.no_sweep:
        out["ds_fp4_decode"] = bench_ds_fp4(torch, ftb, args)
    if not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(torch, layers, args.cpu_seconds)
    return out


def sweep_decode(torch, ftb, layers: "Layers", args):
    """Tokens/s at T = 1, 4, 16 on the same layer banks (fresh routing per T), with each
    kernel's eager CUDA-event time."""
    from ftb import _lib, synth

    res = {}
    for T in (1, 4, 16):
        inps = [synth.make_inputs(T, H, E, seed=2000 + T * 10 + l, device="cuda")
                for l in range(len(layers.banks))]
        outs = [torch.empty(T, H, dtype=torch.bfloat16, device="cuda") for _ in inps]

        def step(i, inps=inps, outs=outs):
            l = i % len(inps)
            w, ids = ftb.fused_topk(None, inps[l].logits, TOPK, True)
            ftb.moe_decode(inps[l].x, layers.banks[l], w, ids, shared=layers.shared[l],
                           out=outs[l])

        for i in range(3):
            step(i)
        timed = graph_steps(torch, step, len(inps)) if args.graphs else step
        for i in range(3):
            timed(i)
        ms = time_steps(torch, timed, min(max(8, args.steps), 200))
        host_ms = time_steps.host_ms
        kt = kernel_times(_lib, torch, step, 16)
        res[f"T={T}"] = {"tokens_per_s": round(T * 1e3 / ms, 1), "ms_per_step": round(ms, 4),
                         "host_issue_ms_per_step": round(host_ms, 4),
                         "kernels_ms": {k: round(statistics.mean(v), 4) for k, v in kt.items()}}
    return res


def bench_prefill(torch, ftb, layers: "Layers", args):
    """one prefill chunk of T tokens (flat N(0,1) router logits) through
    ftb.moe_prefill on the same rotated layer banks, eager launches (route, sort, permute,
    gate_up, down, combine). The tensor roofline is taken per GEMM: useful FLOPs per launch =
    2 x rows x (output rows) x K with rows = T x (top_k + 1) (routed + shared routes)."""
    from ftb import _lib, synth

    T = args.prefill_tokens
    nl = len(layers.banks)
    inps = [synth.make_inputs(T, H, E, seed=3000 + l, device="cuda") for l in range(nl)]
    outs = [torch.empty(T, H, dtype=torch.bfloat16, device="cuda") for _ in range(nl)]

    def step(i):
        l = i % nl
        w, ids = ftb.fused_topk(None, inps[l].logits, TOPK, True)
        ftb.moe_prefill(inps[l].x, layers.banks[l], w, ids, shared=layers.shared[l],
                        out=outs[l])

    for i in range(max(3, args.warmup)):
        step(i)
    steps = min(max(8, args.steps // 4), 60)
    clocks = ClockSampler(torch, 0)
    clocks.start()
    ms = time_steps(torch, step, steps)
    clk = clocks.stop()
    kt = kernel_times(_lib, torch, step, 8)
    rows = T * (TOPK + 1)
    flops = {"gate_up_gemv": 2.0 * rows * 2 * I * H, "down_gemv": 2.0 * rows * H * I}
    burst, sustained, src = measured_tensor_peaks()
    gemms = {}
    for k, f in flops.items():
        t = statistics.mean(kt[k])
        ach = f / (t * 1e-3) / 1e12
        gemms[k] = {"avg_launch_ms": round(t, 4), "tflops": round(ach, 1),
                    "frac_burst": round(ach / burst, 4), "frac_sustained": round(ach / sustained, 4)}
    gemm_ms = sum(statistics.mean(kt[k]) for k in flops)
    ach = sum(flops.values()) / (gemm_ms * 1e-3) / 1e12
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "prefill_gemm_traffic.json")
    if os.path.exists(tpath) and T == 4096:
        # ncu DRAM bytes of one gate_up and one down launch at this workload
        with open(tpath) as f:
            d = json.load(f)
        traffic = d["gate_up_dram_bytes_per_launch"] + d["down_dram_bytes_per_launch"]
    hx = [inp.x.cpu().pin_memory() for inp in inps]
    hl = [inp.logits.cpu().pin_memory() for inp in inps]
    hout = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    dx = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    dl = torch.empty(T, E, dtype=torch.float32, device="cuda")
    dout = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")

    def e2e_one(i):
        l = i % nl
        dx.copy_(hx[l], non_blocking=True)
        dl.copy_(hl[l], non_blocking=True)
        w, ids = ftb.fused_topk(dx, dl, TOPK, True)
        ftb.moe_prefill(dx, layers.banks[l], w, ids, shared=layers.shared[l], out=dout)
        hout.copy_(dout, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(3):
        e2e_one(i)
    n_e2e = min(steps, 20)
    t0 = time.perf_counter()
    for i in range(n_e2e):
        e2e_one(i)
    e2e_dt = (time.perf_counter() - t0) / n_e2e
    return {
        "workload": f"config 2 prefill T={T}: H{H} I{I} E{E} top{TOPK} +1 shared expert, "
                    "flat N(0,1) router logits, layers rotated",
        "tokens_per_s": round(T * 1e3 / ms, 1), "ms_per_step": round(ms, 4), "steps": steps,
        "layer_tflops": round(sum(flops.values()) / (ms * 1e-3) / 1e12, 1),
        "kernels_ms": {k: round(statistics.mean(v), 4) for k, v in kt.items()},
        "roofline": {"kernel": "gate_up + down (k_prefill_gemm<0>, <1>), tcgen05 kind::f16",
                     "bound": "tensor", "achieved": round(ach, 1), "peak": burst,
                     "unit": "TFLOP/s", "frac": round(ach / burst, 4),
                     "frac_sustained": round(ach / sustained, 4), "peak_source": src,
                     "flops_per_step": sum(flops.values()), "traffic": traffic,
                     "per_gemm": gemms},
        "e2e": {"value": round(T / e2e_dt, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": T * H * 2 + T * E * 4, "d2h_bytes_per_step": T * H * 2},
        "gpu_launches_per_step": 6,  # route_topk, sort, permute, gate_up, down, combine
        "clocks": clk,
    }


FP4_DENSE_PEAK_TFLOPS = 9000.0  # nominal dense FP4 per B200 (NVIDIA's 18 PF figure is 2:4 sparse)


def bench_prefill_fp4(torch, ftb, layers: "Layers", args):
    """The opt-in FP4 prefill (ftb.moe_prefill_fp4: x and h quantised to NVFP4, both GEMMs on
    tcgen05 kind::mxf4nvf4) on the config 2 workload, beside the parity path. Not a parity
    number: its distance from the bf16-activation result on the same inputs is reported. Two
    bounds apply: FP4 tensor rate (nominal 9 PFLOP/s dense; no measured FP4 figure exists for
    this pool) and HBM (the weights every step streams, at the measured copy rate)."""
    from ftb import _lib, synth

    T = args.prefill_tokens
    nl = len(layers.banks)
    inps = [synth.make_inputs(T, H, E, seed=3000 + l, device="cuda") for l in range(nl)]
    outs = [torch.empty(T, H, dtype=torch.bfloat16, device="cuda") for _ in range(nl)]
    routes = [ftb.fused_topk(None, inp.logits, TOPK, True) for inp in inps]

    def step(i):
        l = i % nl
        w, ids = ftb.fused_topk(None, inps[l].logits, TOPK, True)
        ftb.moe_prefill_fp4(inps[l].x, layers.banks[l], w, ids, shared=layers.shared[l],
                            out=outs[l])

    for i in range(max(3, args.warmup)):
        step(i)
    steps = min(max(8, args.steps // 4), 60)
    clocks = ClockSampler(torch, 0)
    clocks.start()
    ms = time_steps(torch, step, steps)
    clk = clocks.stop()
    kt = kernel_times(_lib, torch, step, 8)
    rows = T * (TOPK + 1)
    flops = {"gate_up_gemv": 2.0 * rows * 2 * I * H, "down_gemv": 2.0 * rows * H * I}
    gemm_ms = sum(statistics.mean(kt[k]) for k in flops)
    ach = sum(flops.values()) / (gemm_ms * 1e-3) / 1e12
    hbm, hbm_src = measured_peaks()
    w_bytes = (statistics.mean(
        int(torch.unique(r[1]).numel()) for r in routes) + 1) * ftb.bank_bytes_per_expert(H, I)
    hbm_ms = w_bytes / (hbm * 1e9) * 1e3
    # error against the parity path (bf16 activations) on layer 0's inputs
    w0, ids0 = routes[0]
    ref = ftb.moe_prefill(inps[0].x, layers.banks[0], w0, ids0, shared=layers.shared[0])
    got = ftb.moe_prefill_fp4(inps[0].x, layers.banks[0], w0, ids0, shared=layers.shared[0])
    err = float((got.float() - ref.float()).abs().max() / ref.float().abs().max())
    return {
        "workload": f"config 2 prefill T={T} as 'prefill', opt-in NVFP4 activations",
        "parity": "not parity-preserving (activations quantised to NVFP4)",
        "max_abs_rel_vs_parity_path": round(err, 4),
        "tokens_per_s": round(T * 1e3 / ms, 1), "ms_per_step": round(ms, 4), "steps": steps,
        "kernels_ms": {k: round(statistics.mean(v), 4) for k, v in kt.items()},
        "roofline": {"kernel": "gate_up + down (k_prefill_fp4<0>, <1>), tcgen05 kind::mxf4nvf4",
                     "bound": "tensor", "achieved": round(ach, 1), "peak": FP4_DENSE_PEAK_TFLOPS,
                     "unit": "TFLOP/s", "frac": round(ach / FP4_DENSE_PEAK_TFLOPS, 4),
                     "peak_source": "nominal dense FP4 (9 PFLOP/s per B200), not measured here",
                     "hbm_bound_ms": round(hbm_ms, 4),
                     "frac_of_hbm_bound": round(hbm_ms / gemm_ms, 4),
                     "hbm_peak_source": hbm_src},
        "gpu_launches_per_step": 7,  # route, sort, quant x, gate_up, quant h, down, combine
        "clocks": clk,
    }


def bench_ds_fp4(torch, ftb, args, T: int = 64, n_layers: int = 2):
    """ds_fp4 decode (ftb.fused_experts_ds_fp4) at the reference's DSV4-Flash GEMV geometry
    (gate_up K = 4096, down K = 2048: K_BYTES 2048 / 1024 in patches/moe_fused_ds_fp4.patch:
    14-21), 256 experts, top-8, no shared expert, T tokens: seeded ds_fp4 banks (e8m0 per 32)
    converted once to the NVFP4 bank, FP8 round trip of h. HBM roofline of the layer: bytes of
    the converted experts hit + activations, at the measured copy rate."""
    from ftb import _lib, synth
    from ftb.ds_fp4 import nvfp4_from_ds_fp4

    Hd, Id = 4096, 2048
    banks, inps = [], []
    for l in range(n_layers):
        banks.append(nvfp4_from_ds_fp4(synth.make_ds_fp4_bank(E, Hd, Id, seed=500 + l,
                                                             device="cuda"))[0])
        inps.append(synth.make_inputs(T, Hd, E, seed=600 + l, device="cuda"))
    routes = [ftb.fused_topk(None, inp.logits, TOPK, True) for inp in inps]
    outs = [torch.empty(T, Hd, dtype=torch.bfloat16, device="cuda") for _ in range(n_layers)]

    def step(i):
        l = i % n_layers
        w, ids = ftb.fused_topk(None, inps[l].logits, TOPK, True)
        ftb.fused_experts_ds_fp4(inps[l].x, banks[l], w, ids, 0.0, out=outs[l], prefill=False)

    for i in range(3):
        step(i)
    timed = graph_steps(torch, step, n_layers) if args.graphs else step
    for i in range(3):
        timed(i)
    ms = time_steps(torch, timed, min(max(8, args.steps), 200))
    kt = kernel_times(_lib, torch, step, 16)
    hbm, hbm_src = measured_peaks()
    uniq = statistics.mean(int(torch.unique(r[1]).numel()) for r in routes)
    layer_bytes = uniq * ftb.bank_bytes_per_expert(Hd, Id) + 2 * T * Hd * 2
    gbs = layer_bytes / (ms * 1e-3) / 1e9
    return {
        "workload": f"ds_fp4 decode T={T}: H{Hd} I{Id} E{E} top{TOPK}, no shared expert, "
                    "e8m0/32 banks converted to NVFP4, FP8 round trip of h",
        "tokens_per_s": round(T * 1e3 / ms, 1), "ms_per_step": round(ms, 4),
        "experts_hit_per_step": round(uniq, 1),
        "kernels_ms": {k: round(statistics.mean(v), 4) for k, v in kt.items()},
        "layer_hbm_gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4),
        "hbm_peak_source": hbm_src,
        "gpu_launches_per_step": 6,  # route, sort_stage, gate_up, h round trip, down, combine
    }


def run_reference(args, torch, world: int = 1):
    """The reference arm: the reference's CPU MoE executor semantics (C++ restatement in
    oracle/cpu_moe.cpp; the reference's cpu_moe_ext.cpp is absent and unbuildable) on all host
    threads, same metric and config; each step = one layer over the whole job's tokens
    (T per GPU x GPUs). Everything is built on the host: seeded inputs, the oracle's softmax
    top-k, and NVFP4 banks for the routed experts only (the executor reads nothing else); no
    GPU and no product code is involved."""
    import numpy as np

    from ftb import synth  # seeded generator only (pure torch on the CPU)
    from oracle import cpu_moe
    from oracle import moe_oracle as m

    T = args.tokens * world
    inp = synth.make_inputs(T, H, E, seed=1000, device="cpu")
    w, ids = m.topk_softmax(inp.logits.numpy(), TOPK, True)
    used = np.unique(ids)
    remap = np.full(E, -1, np.int32)
    remap[used] = np.arange(used.size, dtype=np.int32)
    bank = synth.make_bank(int(used.size), H, I, seed=0, device="cpu").numpy()
    shared = synth.make_shared(H, I, seed=0, device="cpu").numpy()
    x_bits = inp.x.contiguous().view(torch.int16).numpy().view("uint16")
    cids = remap[ids]
    threads = cpu_moe.max_threads()
    for _ in range(max(1, args.warmup)):
        cpu_moe.moe_layer(x_bits, bank, w, cids, shared, nthreads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_moe.moe_layer(x_bits, bank, w, cids, shared, nthreads=threads)
    dt = (time.perf_counter() - t0) / args.steps
    value = T / dt
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "nvfp4 x bf16 -> fp32 (CPU)",
        "data": "synthetic: seeded NVFP4 banks and N(0,1) logits/activations per BASELINE config "
                f"{3 if world > 1 else 1} (generated on the host)",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": threads,
                         "kind": "port", **host_cpu(),
                         "sample": f"{args.steps} full T={T} layer steps ({used.size} routed "
                                   "experts + shared; C++ restatement of the reference CPU "
                                   "executor semantics, all host threads)"},
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_ep(args, torch, rank: int, world: int, local: int):
    """expert-parallel decode, T tokens per rank, 256 experts sharded
    contiguously over the ranks. value = tokens/s of the whole box = world * T / (max over
    ranks of the per-step device time). Transport "p2p" (default): the layer's own kernels
    move tokens and outputs over NVLink peer memory; "nccl": all_to_all_single dispatch and
    combine (the collective-library baseline)."""
    import datetime

    import torch.distributed as dist

    import ftb
    from ftb import _lib, synth
    from ftb.ep import EpGroup, ExpertParallelMoE, shard_range

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    transport = args.ep_transport
    e0, e1 = shard_range(E, rank, world)
    group = EpGroup(args.tokens, H, I, E, TOPK, True, rank, world) if transport == "p2p" else None
    layers, hits = [], []
    for l in range(args.layers):
        full = synth.make_bank(E, H, I, seed=l, device=dev)
        bank = full.select(slice(e0, e1))
        del full
        torch.cuda.empty_cache()
        shared = synth.make_shared(H, I, seed=l, device=dev)
        inp = synth.make_inputs(args.tokens, H, E, seed=1000 + l, stream=rank, device=dev)
        layers.append((ExpertParallelMoE(bank, shared, E, TOPK, rank, world,
                                         transport=transport, ep_group=group), inp))
        # owned experts hit by every rank's routes of this layer (the bytes this rank streams)
        ids = torch.cat([ftb.fused_topk(r.x, r.logits, TOPK, True)[1].flatten() for r in
                         (synth.make_inputs(args.tokens, H, E, seed=1000 + l, stream=q, device=dev)
                          for q in range(world))])
        hits.append(int(torch.unique(ids[(ids >= e0) & (ids < e1)]).numel()))

    def step(i):
        ep, inp = layers[i % len(layers)]
        return ep.forward(inp.x, inp.logits)

    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    dist.barrier()
    # the NCCL transport reads receive counts on the host every step: not capturable
    use_graphs = args.graphs and transport == "p2p"
    timed = graph_steps(torch, step, len(layers)) if use_graphs else step
    for i in range(max(3, args.warmup)):
        timed(i)
    # the sampler starts (NVML set-up, first sample) before the barrier: started after it,
    # rank 0 would enter the timed loop tens of ms after the others, whose first step then
    # waits for it and whose timed region absorbs the skew
    clocks = ClockSampler(torch, local) if rank == 0 else None
    if clocks:
        clocks.start()
    torch.cuda.synchronize()
    dist.barrier()
    ms = time_steps(torch, timed, args.steps)
    host_ms = time_steps.host_ms
    dist.barrier()
    clk = clocks.stop() if clocks else None
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())

    # end to end through the public API: pinned host x/logits in, host output back, per step
    hx = [inp.x.cpu().pin_memory() for _, inp in layers]
    hl = [inp.logits.cpu().pin_memory() for _, inp in layers]
    hout = torch.empty(args.tokens, H, dtype=torch.bfloat16).pin_memory()
    dx = torch.empty(args.tokens, H, dtype=torch.bfloat16, device=dev)
    dl = torch.empty(args.tokens, E, dtype=torch.float32, device=dev)

    def e2e_one(i):
        l = i % len(layers)
        dx.copy_(hx[l], non_blocking=True)
        dl.copy_(hl[l], non_blocking=True)
        hout.copy_(layers[l][0].forward(dx, dl), non_blocking=True)
        torch.cuda.current_stream().synchronize()

    n_e2e = min(args.steps, 64)
    for i in range(3):
        e2e_one(i)
    dist.barrier()
    t0 = time.perf_counter()
    for i in range(n_e2e):
        e2e_one(i)
    e2e_dt = torch.tensor([(time.perf_counter() - t0) / n_e2e], dtype=torch.float64, device=dev)
    dist.all_reduce(e2e_dt, op=dist.ReduceOp.MAX)
    e2e_s = float(e2e_dt.item())

    # kernel events on every rank (same steps), gate_up roofline from rank 0's launches
    nprof = min(args.steps, 32)
    kt = kernel_times(_lib, torch, step, nprof)
    local_experts = [layers[i % len(layers)][0].last_local_experts for i in range(nprof)]
    phases = ep_phase_trace(torch, dist, group, step, world, dev) if group is not None else None
    status = group.status() if group is not None else 0
    dist.barrier()
    if group is not None:
        group.close()
    dist.destroy_process_group()
    if status:
        raise RuntimeError(f"EP device status word {status:#x} on rank {rank}")
    if rank != 0:
        return None
    peak, peak_src = measured_peaks()
    gu = kt.get("gate_up_gemv", [])
    if transport == "p2p":
        # one gate_up launch per step: owned experts hit + the shared expert
        routed = gu
        byts = sum((hits[i % len(hits)] + 1) * gate_up_bytes_per_expert()
                   for i in range(len(routed)))
        launches = 6  # route, publish, front (sort+stage), gate_up, down, combine
    else:
        # launches alternate: routed experts (received routes), then the shared expert
        routed = gu[0::2]
        byts = sum(local_experts[i % len(local_experts)] * gate_up_bytes_per_expert()
                   for i in range(len(routed)))
        launches = 10  # route, 4 for received routes, 4 for the shared expert, combine
    achieved = byts / (sum(routed) * 1e-3) / 1e9 if routed else None
    value = world * args.tokens * 1e3 / ms_max
    return {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "nvfp4 (e2m1+e4m3) x bf16 -> fp32 accumulate, bf16 out",
        "data": "synthetic: seeded NVFP4 banks and N(0,1) logits/activations per BASELINE config 3",
        "config": workload_config(args, world),
        "run": {"transport": transport, "layers_rotated": args.layers,
                "owned_experts_hit_per_layer_rank0": hits,
                "launch": "CUDA graph per layer (route + layer), replayed" if use_graphs
                          else "eager launches",
                "host_issue_ms_per_step_rank0": round(host_ms, 4),
                "timing": "per-rank CUDA events, max over ranks"},
        "e2e": {"value": round(world * args.tokens / e2e_s, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": args.tokens * (H * 2 + E * 4),
                "d2h_bytes_per_step": args.tokens * H * 2,
                "note": "per rank: pinned x+logits H2D, route + layer, output D2H, host sync; "
                        "max over ranks"},
        "roofline": None if achieved is None else {
            "kernel": "gate_up_gemv (k_gemv_tma<0>), rank 0", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": peak_src, "traffic": None},
        "kernels_ms": {k: round(statistics.mean(v), 4) for k, v in kt.items()},
        "ep_phases_us": phases,
        "gpu_launches": launches * args.steps,
        "clocks": clk,
    }


def ep_phase_trace(torch, dist, group, step, world: int, dev, n: int = 16):
    """Per-phase device timestamps (%globaltimer, ftb_ep_set_trace) of n eager steps on every
    rank: publish, front wait/work, gate_up, down, combine wait/work. Returns, per phase, the
    mean over steps of the max over ranks and every rank's mean, plus the step span."""
    from ftb.ep import EP_TRACE_PHASES, trace_phases_us, trace_reset

    buf = torch.empty(8, dtype=torch.int64, device=dev)
    group.set_trace(buf)
    rows = []
    for i in range(n):
        trace_reset(buf)
        step(i)
        torch.cuda.synchronize()
        rows.append(buf.clone())
    group.set_trace(None)
    mine = torch.stack(rows)  # [n, 8]
    every = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(every, mine)
    names = list(EP_TRACE_PHASES) + ["step"]
    per = [[trace_phases_us(r.tolist()) for r in e.cpu()] for e in every]  # [rank][step]
    out = {"steps": n, "max_over_ranks": {}, "per_rank_mean": {}}
    for name in names:
        out["max_over_ranks"][name] = round(
            statistics.mean(max(per[q][i][name] for q in range(world)) for i in range(n)), 2)
        out["per_rank_mean"][name] = [round(statistics.mean(per[q][i][name] for i in range(n)), 2)
                                      for q in range(world)]
    out["note"] = ("eager steps, trace on; phase i = slot i+1 - slot i of one rank's trace; "
                   "front_wait/combine_wait end when the last peer flag is seen. Each GPU's "
                   "globaltimer has its own offset (seconds apart on this box), so only "
                   "differences within one rank are reported")
    return out


def run_ep_stack(args, torch, rank: int, world: int, local: int):
    """--stack distinct layers of the config 1 shape resident and sharded
    expert-parallel (experts [r E/W, (r+1) E/W) of every layer on rank r, the shared expert
    replicated), run back to back in one step over the peer-memory transport, --tokens per
    GPU, flat or Zipf(1.1)-skewed routing. Each layer takes its own seeded input rows (the
    layers are timed as a stack; no norm or attention sits between them). value = tokens/s
    of the whole box through the stack = W T / (max over ranks of the step's device time)."""
    import datetime

    import torch.distributed as dist

    import ftb
    from ftb import _lib, synth
    from ftb.ep import EpGroup, ExpertParallelMoE, shard_range

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    per_gpu_bytes = args.stack * (E // world + 1) * ftb.bank_bytes_per_expert(H, I)
    free, _ = torch.cuda.mem_get_info(dev)
    if per_gpu_bytes > 0.8 * free:
        raise SystemExit(f"config 4 needs {per_gpu_bytes / 1e9:.1f} GB per GPU at {world} GPUs; "
                         f"{free / 1e9:.1f} GB free")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    e0, e1 = shard_range(E, rank, world)
    zipf = 1.1 if args.routing == "zipf" else None
    group = EpGroup(args.tokens, H, I, E, TOPK, True, rank, world)
    layers, hits = [], []
    for l in range(args.stack):
        # this rank's shard only, drawn directly (the values do not enter the timing)
        bank = synth.make_bank(e1 - e0, H, I, seed=100000 + 1000 * l + rank, device=dev)
        shared = synth.make_shared(H, I, seed=200000 + l, device=dev)
        inp = synth.make_inputs(args.tokens, H, E, seed=3000 + l, stream=rank, device=dev,
                                zipf_s=zipf)
        layers.append((ExpertParallelMoE(bank, shared, E, TOPK, rank, world,
                                         transport="p2p", ep_group=group), inp))
        ids = torch.cat([ftb.fused_topk(r.x, r.logits, TOPK, True)[1].flatten() for r in
                         (synth.make_inputs(args.tokens, H, E, seed=3000 + l, stream=q,
                                            device=dev, zipf_s=zipf) for q in range(world))])
        hits.append(int(torch.unique(ids[(ids >= e0) & (ids < e1)]).numel()))
    # busiest rank: max over ranks of the owned experts hit, summed over the stack
    t_hits = torch.tensor([sum(hits)], dtype=torch.float64, device=dev)
    dist.all_reduce(t_hits, op=dist.ReduceOp.MAX)

    def stack_step(i):
        for ep, inp in layers:
            ep.forward(inp.x, inp.logits)

    for i in range(max(2, min(args.warmup, 3))):
        stack_step(i)
    torch.cuda.synchronize()
    dist.barrier()
    timed = graph_steps(torch, stack_step, 1) if args.graphs else stack_step
    for i in range(2):
        timed(i)
    clocks = ClockSampler(torch, local) if rank == 0 else None  # before the barrier, as above
    if clocks:
        clocks.start()
    torch.cuda.synchronize()
    dist.barrier()
    steps = max(3, min(args.steps, 20))
    ms = time_steps(torch, timed, steps)
    dist.barrier()
    clk = clocks.stop() if clocks else None
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    kt = kernel_times(_lib, torch, stack_step, 1, launches_per_step=8 * args.stack)
    status = group.status()
    if args.graphs:
        del timed
    dist.barrier()
    group.close()
    dist.destroy_process_group()
    if status:
        raise RuntimeError(f"EP device status word {status:#x} on rank {rank}")
    if rank != 0:
        return None
    peak, peak_src = measured_peaks()
    # rank 0's weight bytes per step: its owned experts hit plus the shared expert, per layer
    r0_bytes = sum((h + 1) * ftb.bank_bytes_per_expert(H, I) for h in hits)
    return {
        "metric": METRIC, "value": round(world * args.tokens * 1e3 / ms_max, 1),
        "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": 2,
        "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "nvfp4 (e2m1+e4m3) x bf16 -> fp32 accumulate, bf16 out",
        "data": "synthetic: seeded NVFP4 banks and N(0,1) logits/activations per BASELINE "
                f"config 4 ({args.routing} routing)",
        "config": {"workload": f"config 4 stacked MoE: {args.stack} layers of H{H} I{I} E{E} "
                               f"top{TOPK} +1 shared, T={args.tokens} tokens per GPU per step, "
                               f"{E // world} experts per GPU per layer, {args.routing} routing",
                   "routing": args.routing, "layers": args.stack,
                   "tokens_per_step_per_gpu": args.tokens,
                   "resident_expert_bytes_per_gpu": per_gpu_bytes,
                   "resident_expert_bytes_total": args.stack * (E + world) *
                                                  ftb.bank_bytes_per_expert(H, I),
                   "owned_experts_hit_rank0": sum(hits),
                   "owned_experts_hit_busiest_rank": int(t_hits.item()),
                   "launch": "one CUDA graph per step" if args.graphs else "eager launches",
                   "timing": "per-rank CUDA events, max over ranks"},
        "layer_ms": round(ms_max / args.stack, 4),
        "rank0_weight_gbs": round(r0_bytes / (ms * 1e-3) / 1e9, 1), "peak_gbs": peak,
        "peak_source": peak_src,
        "kernels_ms": {k: round(statistics.mean(v), 4) for k, v in kt.items()},
        "gpu_launches": 6 * args.stack * steps,
        "clocks": clk,
    }


def main():
    args = parse_args()
    rank, world, local = dist_env()
    import torch

    if args.impl == "reference":
        if rank != 0:
            return 0  # the reference arm runs on rank 0 only
        print(json.dumps(run_reference(args, torch, world)), flush=True)
        return 0
    if args.stack > 0:
        out = run_ep_stack(args, torch, rank, world, local)
        if rank == 0:
            print(json.dumps(out), flush=True)
        return 0
    if world > 1:
        out = run_ep(args, torch, rank, world, local)
        if rank == 0:
            print(json.dumps(out), flush=True)
        return 0
    print(json.dumps(run_ftb_single(args, torch)), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
