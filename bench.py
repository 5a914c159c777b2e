#!/usr/bin/env python
"""Benchmark of the B200 DeepSeek-V3/R1 FP8 MoE forward (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload at N=1: benchmark configuration 2 (T=4096 tokens, 32 local experts of 256,
local_expert_offset 0; the prefill case the headline tokens/s is quoted on). Each step is one
full moe_forward: route -> gather -> GEMM1+SwiGLU -> GEMM2 -> combine. The
1.41 GB of FP8 expert weights exceed the 126 MB L2, so no flush is needed between steps.
The decode case (configuration 1, T=64) is reported alongside as microseconds per layer.

Under torchrun (N > 1) the layer runs expert-parallel (15642_moe_b200/ep.py): rank r owns
experts 32r..32r+31, the 4096 tokens are split over the ranks, token rows travel to their
experts' owners and partial results back as peer stores over NVLink issued by the kernels.
Per-GPU work stays that of configuration 2 ("weak" scaling); the value counts each token once
per 32-expert slice it passes through, over the max-over-ranks device time.

--impl reference times the CPU restatement of reference/moe_ref.py (oracle/) on the host
cores, on the same configuration (rank 0 only).
"""
from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "MoE fwd tokens/s @T=4096 (1-8 B200 EP); µs/layer @T=64; %HBM / %FP8 TC peak"
W13_EXPERT_BYTES = 4096 * 7168
W2_EXPERT_BYTES = 7168 * 2048
W13_SCALE_BYTES = 32 * 56 * 4
W2_SCALE_BYTES = 56 * 16 * 4
FLOPS_G1_PER_ROUTE = 2 * 7168 * 4096
FLOPS_G2_PER_ROUTE = 2 * 2048 * 7168
STAGES = ["route", "gather", "gemm1_swiglu", "gemm2_weighted", "combine"]


def load_peaks() -> dict:
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return dict(hbm_gbs=float(p["hbm_gbs"]), bf16_tflops=float(p["bf16_tflops"]), source="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, source="fallback")


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms in the background."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        busy = [s for s, p in zip(sm, power) if p > 0.5 * max(power)] or sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm), "samples_under_load": len(busy),
                "power_w_max": max(power)}


def routing_stats(pkg, inp) -> dict:
    idx, _ = pkg.route(inp["routing_logits"], inp["routing_bias"], inp["routed_scaling_factor"])
    idx = idx.cpu().numpy()
    off, E = inp["local_expert_offset"], inp["gemm1_weights"].shape[0]
    local = (idx >= off) & (idx < off + E)
    counts = np.bincount((idx[local] - off).ravel(), minlength=E)
    return dict(routes=int(local.sum()), active=int((counts > 0).sum()),
                max_per_expert=int(counts.max()), tiles=int(((counts + 127) // 128).sum()))


def kernel_work(rs: dict, T: int) -> dict:
    """Algorithmic bytes and FLOPs per launch of each kernel (what it must move / compute)."""
    r, a = rs["routes"], rs["active"]
    return {
        "gemm1_swiglu": dict(bytes=a * (W13_EXPERT_BYTES + W13_SCALE_BYTES) + r * (7168 + 56 * 4)
                             + r * (2 * 2048 + 16 * 4), flops=r * FLOPS_G1_PER_ROUTE),
        "gemm2_weighted": dict(bytes=a * (W2_EXPERT_BYTES + W2_SCALE_BYTES) + r * (2 * 2048 + 16 * 4)
                               + r * 7168 * 4, flops=2 * r * FLOPS_G2_PER_ROUTE),
        "combine": dict(bytes=r * 7168 * 4 + T * 7168 * 2, flops=0),
        "route": dict(bytes=T * 256 * 4 + T * 8 * 8, flops=0),
        "gather": dict(bytes=r * (7168 + 56 * 4) * 2, flops=0),
    }


class Step:
    """One moe_forward of a fixed workload with resident packed weights and buffers."""

    def __init__(self, pkg, inp, device, packed=None):
        self.pkg, self.inp, self.dev = pkg, inp, device
        self.lib = pkg._native.cuda_lib()
        self.T = inp["hidden_states"].shape[0]
        self.E = inp["gemm1_weights"].shape[0]
        if packed is None:
            packed = (pkg.pack_w13(inp["gemm1_weights"]), pkg.pack_w2(inp["gemm2_weights"]))
        self.w13p, self.w2p = packed
        self.hs = inp["hidden_states_scale"].float().contiguous()
        self.s13 = inp["gemm1_weights_scale"].float().contiguous()
        self.s2 = inp["gemm2_weights_scale"].float().contiguous()
        self.lg = inp["routing_logits"].float().contiguous()
        self.b = inp["routing_bias"].float().reshape(-1).contiguous()
        self.out = torch.empty((self.T, 7168), dtype=torch.bfloat16, device=device)
        self.ws = torch.empty(pkg.workspace_bytes(self.T, self.E), dtype=torch.uint8, device=device)
        self.stream = torch.cuda.current_stream(device).cuda_stream
        self.args = (inp["hidden_states"].data_ptr(), self.hs.data_ptr(), self.w13p.data_ptr(),
                     self.s13.data_ptr(), self.w2p.data_ptr(), self.s2.data_ptr(), self.lg.data_ptr(),
                     self.b.data_ptr(), float(inp["routed_scaling_factor"]),
                     int(inp["local_expert_offset"]), self.T, self.E, self.out.data_ptr(),
                     self.ws.data_ptr(), self.ws.numel(), self.stream)

    def __call__(self):
        self.pkg._native.check(self.lib.moe_forward(*self.args))

    def profiled(self, events):
        arr = (ctypes.c_void_p * (len(STAGES) + 1))(*[e.cuda_event for e in events])
        self.pkg._native.check(self.lib.moe_forward_profiled(*self.args, arr))


def time_steps(fn, steps: int) -> float:
    """Device time in ms of `steps` calls, CUDA events on the launching stream."""
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e)


def stage_times(step: Step, reps: int) -> dict:
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(STAGES) + 1)] for _ in range(reps)]
    for row in evs:          # torch creates the CUDA event on first record
        for ev in row:
            ev.record()
    torch.cuda.synchronize()
    for r in range(reps):
        step.profiled(evs[r])
    torch.cuda.synchronize()
    out = {}
    for i, name in enumerate(STAGES):
        out[name] = statistics.mean(evs[r][i].elapsed_time(evs[r][i + 1]) for r in range(reps))
    return out


def roofline(stage_ms: dict, work: dict, peaks: dict, traffic: dict | None) -> dict:
    dom = max(("gemm1_swiglu", "gemm2_weighted"), key=lambda k: stage_ms[k])
    w, ms = work[dom], stage_ms[dom]
    fp8_tflops = 2.0 * peaks["bf16_tflops"]          # dense FP8 issues at twice the bf16 rate
    t_hbm = w["bytes"] / (peaks["hbm_gbs"] * 1e9)
    t_tc = w["flops"] / (fp8_tflops * 1e12)
    bound = "hbm" if t_hbm >= t_tc else "tensor"
    if bound == "hbm":
        achieved, peak, unit = w["bytes"] / (ms * 1e-3) / 1e9, peaks["hbm_gbs"], "GB/s"
    else:
        achieved, peak, unit = w["flops"] / (ms * 1e-3) / 1e12, fp8_tflops, "TFLOP/s"
    tr = None
    if traffic and dom in traffic:
        tr = traffic[dom]
    return {"kernel": dom, "bound": bound, "achieved": round(achieved, 1), "peak": peak,
            "unit": unit, "frac": round(achieved / peak, 4), "traffic": tr,
            "algorithmic_bytes": int(w["bytes"]), "algorithmic_flops": int(w["flops"]),
            "kernel_us": round(ms * 1e3, 2), "peak_source": peaks["source"],
            "tensor_frac_fp8": round(w["flops"] / (ms * 1e-3) / 1e12 / fp8_tflops, 4),
            "hbm_frac": round(w["bytes"] / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)}


def load_traffic(workload: str) -> dict | None:
    path = os.path.join(REPO, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        return json.load(f).get(workload)


def e2e_run(pkg, inp, device, steps: int, warmup: int, forward=None) -> dict:
    """End to end through the public serving API (pkg.HostPipeline): every step copies its
    activations in from pinned host memory, runs the layer with resident packed weights and
    copies its bf16 result back to pinned host memory; neighbouring steps' copies overlap the
    forward on separate streams. `forward(h, s, logits, out)` replaces the single-GPU layer (the
    expert-parallel bench passes its context's forward). Timed with CUDA events from before the
    first copy in to after the last copy out."""
    T = int(inp["hidden_states"].shape[0])
    if forward is None:
        pipe = pkg.HostPipeline.for_layer(
            pkg.pack_w13(inp["gemm1_weights"]), inp["gemm1_weights_scale"].float().contiguous(),
            pkg.pack_w2(inp["gemm2_weights"]), inp["gemm2_weights_scale"].float().contiguous(),
            inp["routing_bias"], float(inp["routed_scaling_factor"]), int(inp["local_expert_offset"]), T)
    else:
        pipe = pkg.HostPipeline(forward, T, device)
    hidden = inp["hidden_states"].cpu().pin_memory()
    scale = inp["hidden_states_scale"].float().cpu().pin_memory()
    logits = inp["routing_logits"].float().cpu().pin_memory()
    out_host = torch.empty((T, 7168), dtype=torch.bfloat16).pin_memory()
    for _ in range(max(warmup, 3)):
        pipe.submit(hidden, scale, logits, out_host)
    pipe.synchronize()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(pipe.h2d_stream)
    for _ in range(steps):
        pipe.submit(hidden, scale, logits, out_host)
    end.record(pipe.d2h_stream)
    torch.cuda.synchronize()
    h2d = sum(t.numel() * t.element_size() for t in (hidden, scale, logits))
    return {"ms_per_step": start.elapsed_time(end) / steps, "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(out_host.numel() * out_host.element_size()),
            "api": "HostPipeline (3 streams, double-buffered device slots)"}


def cpu_oracle_time(pkg, inp, max_seconds: float, experts=None) -> tuple[float, str, int]:
    """Seconds of one oracle layer (or of an expert sample scaled to the layer)."""
    from oracle import moe_oracle as O
    npi = O.to_numpy_inputs(inp)
    rs_idx, _ = O.route(npi["routing_logits"], npi["routing_bias"], npi["routed_scaling_factor"])
    off, E = npi["local_expert_offset"], npi["gemm1_weights"].shape[0]
    active = [e for e in range(E) if (rs_idx == off + e).any()]
    sample = active if experts is None else experts
    O.moe_forward(**npi, experts=sample)        # first call pays the page faults; discarded
    t0 = time.perf_counter()
    O.moe_forward(**npi, experts=sample)
    dt = time.perf_counter() - t0
    scale = len(active) / max(1, len(sample))
    desc = (f"full layer ({len(active)} active local experts)" if len(sample) == len(active)
            else f"{len(sample)} of {len(active)} active local experts, time scaled x{scale:.2f}")
    return dt * scale, desc, len(active)


def ref_cuda_leg(cases: dict) -> dict:
    """The reference's own CUDA extension (kernels/moe.cu, built unchanged for sm_100 by
    oracle/build_ref.py into oracle/_ref) timed on the same GPU and the same device inputs as this
    package: the GPU baseline. ``cases`` maps a name to (inputs, our us/layer, our bf16 output)."""
    from oracle import build_ref
    if not os.path.exists(build_ref.so_path()):
        return {"unavailable": "oracle/_ref/moe_fused_ref.so not built (python -m oracle.build_ref)"}
    from oracle import ref_cuda
    from oracle import moe_oracle as O
    mod = build_ref.load()
    res = {"what": "reference kernels/moe.cu (mma.sync e4m3, fp32 atomicAdd combine) built for sm_100 "
                   "with its own flags, run_custom's call sequence, CUDA events, same device inputs"}
    for name, (inp, ours_us, ours_out) in cases.items():
        rc = ref_cuda.RefCuda(inp, mod)
        us = rc.time_us(steps=10, warmup=3)
        ref_out = rc()
        torch.cuda.synchronize()
        a = ours_out.view(torch.int16).cpu().numpy().view(np.uint16)
        b = ref_out.view(torch.int16).cpu().numpy().view(np.uint16)
        diff = O.check_tolerance(a, b)
        res[name] = {"ref_us_per_layer": round(us, 2), "ours_us_per_layer": round(ours_us, 2),
                     "speedup": round(us / ours_us, 2),
                     "ref_vs_ours": {"max_abs_diff": round(diff["max_abs_err"], 5),
                                     "elements_outside_ref_tolerance": diff["bad"]}}
        del rc, ref_out
        torch.cuda.empty_cache()
    return res


# Configuration 2 of the benchmark description: the workload the N = 1 line is quoted on.
CFG2 = dict(T=4096, E_local=32, local_expert_offset=0, seed=0, routed_scaling_factor=2.5)
LAYER_FLOPS_PER_ROUTE = FLOPS_G1_PER_ROUTE + FLOPS_G2_PER_ROUTE   # 88,080,384 (reference bench)


def config_1gpu() -> dict:
    """The `config` object of the N = 1 line (both arms print exactly this)."""
    return {"workload": "config2_prefill_t4096", "T": CFG2["T"], "E_local": CFG2["E_local"],
            "experts_total": 256, "local_expert_offset": CFG2["local_expert_offset"],
            "routed_scaling_factor": CFG2["routed_scaling_factor"], "seed": CFG2["seed"],
            "parallelism": "1 GPU", "l2": "inputs larger than L2 (1.41 GB FP8 expert weights per step)"}


def config_ep(world: int) -> dict:
    """The `config` object of an N > 1 line (both arms print exactly this)."""
    return {"workload": "ep_weak_config2_t4096", "T_global": CFG2["T"], "experts_per_rank": 32,
            "experts_instantiated": 32 * world, "experts_total": 256,
            "routed_scaling_factor": CFG2["routed_scaling_factor"], "seed": CFG2["seed"],
            "parallelism": f"ep{world}: dispatch/combine as peer stores over NVLink",
            "placement": "experts 0..32N-1 balanced over the ranks by the route counts of a calibration "
                         "batch (seed-1 tokens routed with this layer's bias)",
            "token_count": "each token counted once per 32-expert slice it passes through "
                           f"({CFG2['T']} x {world} per step); N=8 is the full 256-expert layer",
            "l2": "inputs larger than L2 (1.41 GB FP8 expert weights per rank per step)"}


def layer_work(rs: dict, T: int) -> dict:
    """Algorithmic HBM bytes and FLOPs of one layer call: every active expert's FP8 weights and
    scales once, the token rows, scales and logits in, the bf16 output out; FLOPs = local routes
    x 88,080,384 (the reference benchmark's count, bench/bench_moe.py:32)."""
    per_expert = W13_EXPERT_BYTES + W2_EXPERT_BYTES + W13_SCALE_BYTES + W2_SCALE_BYTES
    return dict(bytes=rs["active"] * per_expert + T * (7168 + 224 + 1024) + 512 + T * 14336,
                flops=rs["routes"] * LAYER_FLOPS_PER_ROUTE)


SWEEP_T = [1, 4, 32, 64, 256, 2048, 4096, 8192, 16384]   # reference bench/bench_moe.py:20


def t_sweep(pkg, base_inp, packed, device, peaks) -> list:
    """One GPU, experts 0-31 of configuration 2's weights, T over the reference benchmark's list.
    Tokens from seed 0, except T = 1, whose seed-0 token routes to no local expert: the probe uses
    seed 1 (two local routes) so the latency includes the expert GEMMs."""
    fp8 = 2.0 * peaks["bf16_tflops"]
    out = []
    for T in SWEEP_T:
        seed = 1 if T == 1 else 0
        act = pkg.make_inputs(pkg.CONFIGS[2].with_(T=T, seed=seed, E_local=1), device)
        inp = dict(act, **{k: base_inp[k] for k in ("gemm1_weights", "gemm1_weights_scale",
                                                    "gemm2_weights", "gemm2_weights_scale")})
        step = Step(pkg, inp, device, packed=packed)
        rs = routing_stats(pkg, inp)
        for _ in range(3):
            step()
        n = 20 if T <= 4096 else 10
        us = time_steps(step, n) / n * 1e3
        w = layer_work(rs, T)
        out.append({"T": T, "seed": seed, "us_per_layer": round(us, 2),
                    "tokens_per_s": round(T / (us * 1e-6), 1), "routes": rs["routes"],
                    "active_experts": rs["active"], "bytes": int(w["bytes"]), "flops": int(w["flops"]),
                    "hbm_frac": round(w["bytes"] / (us * 1e-6) / 1e9 / peaks["hbm_gbs"], 4),
                    "fp8_tc_frac": round(w["flops"] / (us * 1e-6) / 1e12 / fp8, 4)})
        del step, inp, act
    torch.cuda.empty_cache()
    return out


def slice_spread(pkg, device, peaks, steps: int = 10) -> list:
    """Configuration 2's tokens (T = 4096, seed 0) on each 32-expert slice of the 256-expert layer
    (local_expert_offset 0, 32, ..., 224): the headline instance is slice 0."""
    act = pkg.make_inputs(pkg.CONFIGS[2].with_(E_local=1), device)
    out = []
    for off in range(0, 256, 32):
        cfg = pkg.CONFIGS[2].with_(local_expert_offset=off)
        inp = dict(act, **pkg.make_weights(cfg, range(off, off + 32), device), local_expert_offset=off)
        step = Step(pkg, inp, device)
        rs = routing_stats(pkg, inp)
        for _ in range(3):
            step()
        us = time_steps(step, steps) / steps * 1e3
        w = layer_work(rs, cfg.T)
        out.append({"local_expert_offset": off, "routes": rs["routes"], "active_experts": rs["active"],
                    "max_routes_per_expert": rs["max_per_expert"], "us_per_layer": round(us, 2),
                    "tokens_per_s": round(cfg.T / (us * 1e-6), 1),
                    "hbm_frac": round(w["bytes"] / (us * 1e-6) / 1e9 / peaks["hbm_gbs"], 4)})
        del step, inp
        torch.cuda.empty_cache()
    return out


def make_workload(pkg, name: str, rank: int, device):
    base = pkg.CONFIGS[2] if name == "prefill" else pkg.CONFIGS[1]
    cfg = base.with_(local_expert_offset=32 * (rank % 8))
    return cfg, pkg.make_inputs(cfg, device)


def bench_ours(args, rank, world, local_rank, dist):
    pkg = importlib.import_module("15642_moe_b200")
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    peaks = load_peaks()

    cfg, inp = make_workload(pkg, "prefill", rank, device)
    step = Step(pkg, inp, device)
    rs = routing_stats(pkg, inp)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # Burn-in (untimed) so clocks settle and the sampler sees the GPU under this load.
    sampler = ClockSampler(local_rank)
    sampler.start()
    t_end = time.time() + args.burn_in
    while time.time() < t_end:
        for _ in range(20):
            step()
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ms = time_steps(step, args.steps)
    if dist is not None:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    clocks = sampler.stop()
    status = pkg.device_status(reset=True)

    stages = stage_times(step, min(args.steps, 50))
    work = kernel_work(rs, cfg.T)
    roof = roofline(stages, work, peaks, load_traffic("prefill_t4096"))

    # Decode shape: microseconds per layer at T=64 (configuration 1).
    dcfg, dinp = make_workload(pkg, "decode", rank, device)
    dstep = Step(pkg, dinp, device)
    drs = routing_stats(pkg, dinp)
    for _ in range(max(args.warmup, 3)):
        dstep()
    dms = time_steps(dstep, max(args.steps, 20)) / max(args.steps, 20)
    dstages = stage_times(dstep, 20)
    droof = roofline(dstages, kernel_work(drs, dcfg.T), peaks, load_traffic("decode_t64"))
    layer_bytes = drs["active"] * (W13_EXPERT_BYTES + W2_EXPERT_BYTES + W13_SCALE_BYTES + W2_SCALE_BYTES)

    # FP8 activation quantiser (the step before the path), T = 16384: 352 MB moved per call,
    # more than L2, so repeated calls stream from HBM.
    TQ = 16384
    xq = torch.randn((TQ, 7168), device=device).to(torch.bfloat16)
    qo = torch.empty((TQ, 7168), dtype=torch.float8_e4m3fn, device=device)
    qs = torch.empty((56, TQ), dtype=torch.float32, device=device)
    for _ in range(3):
        pkg.quantize_hidden(xq, qo, qs)
    q_ms = time_steps(lambda: pkg.quantize_hidden(xq, qo, qs), 20) / 20
    q_bytes = TQ * (7168 * 2 + 7168 + 56 * 4)
    # Gate GEMM fused with the quantiser on the same rows: logits + codes + scales in one pass.
    wg = (0.02 * torch.randn((256, 7168), device=device)).to(torch.bfloat16)
    gp = pkg.pack_gate(wg)
    gl = torch.empty((TQ, 256), dtype=torch.float32, device=device)
    for _ in range(3):
        pkg.gate_quantize(xq, gp, gl, qo, qs)
    g_ms = time_steps(lambda: pkg.gate_quantize(xq, gp, gl, qo, qs), 20) / 20
    g_bytes = q_bytes + TQ * 256 * 4 + 256 * 7168 * 2
    g_flops = 2.0 * TQ * 256 * 7168
    del xq, qo, qs, wg, gp, gl

    e2e = e2e_run(pkg, inp, device, args.steps, args.warmup)
    if dist is not None:
        t = torch.tensor([e2e["ms_per_step"]], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e["ms_per_step"] = float(t.item())

    # The reference benchmark's T list on one GPU, and configuration 2's tokens on every slice.
    sweep = t_sweep(pkg, inp, (step.w13p, step.w2p), device, peaks)
    spread = slice_spread(pkg, device, peaks)
    # Configurations 3 and 4 as one GPU's layer (all 256 experts local): the N = 1 points of the
    # expert-parallel strong-scaling curves reported by the N > 1 lines.
    config3 = layer_1gpu(pkg, device, pkg.CONFIGS[3])
    config4 = layer_1gpu(pkg, device, pkg.CONFIGS[4], steps=5)

    if rank != 0:
        return None
    tokens = cfg.T * world
    line = {
        "metric": METRIC,
        "value": round(tokens * args.steps / (ms * 1e-3), 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3 (fp32 accumulate)",
        "data": "synthetic: seeded N(0,1) logits/hidden, N(0,0.1) bias, N(0,0.02) weights, "
                "e4m3 with amax/448 128-block scales",
        "config": config_1gpu(),
        "routing": {"routes": rs["routes"], "active_experts": rs["active"],
                    "max_routes_per_expert": rs["max_per_expert"], "tiles": rs["tiles"]},
        "roofline": roof,
        "layer_roofline": (lambda w: {"bytes": int(w["bytes"]), "flops": int(w["flops"]),
                                      "hbm_frac": round(w["bytes"] / (ms / args.steps * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                                      "fp8_tc_frac": round(w["flops"] / (ms / args.steps * 1e-3) / 1e12 / (2.0 * peaks["bf16_tflops"]), 4),
                                      "fp8_peak": "derived: 2 x measured bf16 burst"})(layer_work(rs, cfg.T)),
        "stage_us": {k: round(v * 1e3, 2) for k, v in stages.items()},
        "decode_t64": {"us_per_layer": round(dms * 1e3, 2), "routes": drs["routes"],
                       "active_experts": drs["active"],
                       "weight_bytes": int(layer_bytes),
                       "hbm_frac_layer": round(layer_bytes / (dms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                       "roofline": droof, "stage_us": {k: round(v * 1e3, 2) for k, v in dstages.items()}},
        "config3_layer": config3,
        "config4_skew": config4,
        "t_sweep": sweep,
        "t1_probe": next(x for x in sweep if x["T"] == 1),
        "slices_t4096": spread,
        "quantize": {"T": TQ, "us": round(q_ms * 1e3, 2), "bytes": q_bytes,
                     "achieved_gbs": round(q_bytes / (q_ms * 1e-3) / 1e9, 1),
                     "hbm_frac": round(q_bytes / (q_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                     "kernel": "quantize_hidden_kernel: bf16 [T,7168] -> e4m3 + [56,T] scales"},
        "gate_quantize": {"T": TQ, "us": round(g_ms * 1e3, 2), "bytes": g_bytes,
                          "achieved_gbs": round(g_bytes / (g_ms * 1e-3) / 1e9, 1),
                          "hbm_frac": round(g_bytes / (g_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                          "tflops": round(g_flops / (g_ms * 1e-3) / 1e12, 1),
                          "kernel": "gate_quantize_kernel: bf16 [T,7168] -> fp32 logits [T,256] "
                                    "(tcgen05 bf16) + e4m3 + [56,T] scales, one read of the rows"},
        "e2e": {"value": round(cfg.T * world / (e2e["ms_per_step"] * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": e2e["h2d_bytes_per_step"],
                "d2h_bytes_per_step": e2e["d2h_bytes_per_step"],
                "ms_per_step": round(e2e["ms_per_step"], 4), "api": e2e["api"]},
        "gpu_launches": len(STAGES) * args.steps,
        "clocks": clocks,
        "device_status": status,
    }
    if world == 1:
        out_p, out_d = torch.empty_like(step.out), torch.empty_like(dstep.out)
        step()
        out_p.copy_(step.out)
        dstep()
        out_d.copy_(dstep.out)
        line["ref_cuda"] = ref_cuda_leg({"config2_t4096": (inp, ms * 1e3 / args.steps, out_p),
                                         "config1_t64": (dinp, dms * 1e3, out_d)})
    if world == 1 and not args.no_cpu_baseline:
        secs, desc, _ = cpu_oracle_time(pkg, {k: (v.cpu() if isinstance(v, torch.Tensor) else v)
                                              for k, v in inp.items()}, 30.0)
        line["cpu_baseline"] = {"value": round(cfg.T / secs, 2), "unit": "tokens/s",
                                "cores": os.cpu_count(), "kind": "port",
                                "sample": f"oracle/moe_oracle.py (numpy restatement of "
                                          f"reference/moe_ref.py), T={cfg.T}, {desc}, "
                                          f"1 warm call after 1 discarded call"}
    return line


def ep_routing_stats(pkg, inp, experts) -> dict:
    """Routes and active experts a rank owning `experts` receives (their picks over all tokens)."""
    idx, _ = pkg.route(inp["routing_logits"], inp["routing_bias"], inp["routed_scaling_factor"])
    per = np.bincount(idx.cpu().numpy().ravel(), minlength=256)[list(experts)]
    return dict(routes=int(per.sum()), active=int((per > 0).sum()),
                max_per_expert=int(per.max()), tiles=int(((per + 127) // 128).sum()))


class EpCase:
    """One expert-parallel layer instance on this rank: `T_global` tokens of `cfg` split evenly
    over the ranks, the experts `pool` placed e_rank per rank by expected load (route counts of a
    calibration batch: seed+1 tokens routed with this layer's bias), packed weights of this
    rank's experts, and an ExpertParallel context. Collective (every rank builds it)."""

    def __init__(self, pkg, epm, rank, world, device, cfg, T_global, e_rank, pool):
        self.pkg, self.epm, self.rank, self.world, self.dev = pkg, epm, rank, world, device
        self.cfg, self.T_global, self.e_rank = cfg, T_global, e_rank
        act = pkg.make_inputs(cfg.with_(T=T_global, E_local=1), device)
        cal = pkg.make_inputs(cfg.with_(T=T_global, seed=cfg.seed + 1, E_local=1), device)["routing_logits"]
        cidx, _ = pkg.route(cal, act["routing_bias"], cfg.routed_scaling_factor)
        loads = torch.bincount(cidx.flatten().long(), minlength=256).cpu().numpy()
        self.placement = epm.balanced_placement(loads, world, e_rank, experts=pool)
        w = pkg.make_weights(cfg, self.placement[rank], device)
        idx, _ = pkg.route(act["routing_logits"], act["routing_bias"], cfg.routed_scaling_factor)
        per = np.bincount(idx.cpu().numpy().ravel(), minlength=256)[list(self.placement[rank])]
        self.routes, self.active = int(per.sum()), int((per > 0).sum())
        self.lo, self.hi = epm.token_range(T_global, world, rank)
        lo, hi = self.lo, self.hi
        self.k = dict(hidden=act["hidden_states"][lo:hi].contiguous(),
                      hs=act["hidden_states_scale"][:, lo:hi].float().contiguous(),
                      lg=act["routing_logits"][lo:hi].float().contiguous(),
                      b=act["routing_bias"].float().reshape(-1).contiguous(),
                      s13=w["gemm1_weights_scale"].float().contiguous(),
                      s2=w["gemm2_weights_scale"].float().contiguous())
        self.w13p, self.w2p = pkg.pack_w13(w["gemm1_weights"]), pkg.pack_w2(w["gemm2_weights"])
        del w, cal, act
        self.out = torch.empty((hi - lo, 7168), dtype=torch.bfloat16, device=device)
        self.ctx = epm.ExpertParallel(t_rank_max=max(1, hi - lo), e_rank=e_rank, device=device,
                                      placement=self.placement)

    def __call__(self, events=None, out=None):
        k = self.k
        return self.ctx.forward(k["hidden"], k["hs"], self.w13p, k["s13"], self.w2p, k["s2"], k["lg"], k["b"],
                                float(self.cfg.routed_scaling_factor), out=self.out if out is None else out,
                                events=events)

    def close(self):
        self.ctx.close()

    def time_ms(self, dist, steps: int, warmup: int) -> float:
        """Max over ranks of the device time of one forward, from `steps` timed after `warmup`."""
        for _ in range(warmup):
            self()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        ms = time_steps(self, steps)
        t = torch.tensor([ms], device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item()) / steps

    def parity(self, dist, oracle_rows: int = 8) -> dict:
        """This rank's output against (1) the same layer composed from single-expert forwards on
        this GPU - per owner d ascending, the fp32 chain over d's experts in ascending order of
        moe_forward(..., fp32_out=True) with that one expert, then the fp32 chain over owners,
        rounded once - bit for bit; (2) on rank 0, the CPU oracle (single rounding over all the
        token's experts, reference tolerance) on a few rows. Collective."""
        pkg, k = self.pkg, self.k
        got = self().clone()
        torch.cuda.synchronize()
        status = pkg.device_status(reset=True)
        T_r = self.hi - self.lo
        acc = torch.zeros((T_r, 7168), dtype=torch.float32, device=self.dev)
        for d in range(self.world):
            part = torch.zeros_like(acc)
            for g in sorted(self.placement[d]):
                w = pkg.make_weights(self.cfg, [g], self.dev)
                if T_r:
                    part += pkg.moe_forward(k["hidden"], k["hs"], pkg.pack_w13(w["gemm1_weights"]),
                                            w["gemm1_weights_scale"].float().contiguous(),
                                            pkg.pack_w2(w["gemm2_weights"]),
                                            w["gemm2_weights_scale"].float().contiguous(), k["lg"], k["b"],
                                            float(self.cfg.routed_scaling_factor), g, fp32_out=True)
            acc += part
        ref = acc.to(torch.bfloat16)
        differ = int((got.view(torch.int16) != ref.view(torch.int16)).sum().item())
        res = {"rows": T_r, "bf16_values_differing_from_composition": differ, "device_status": status}
        if self.rank == 0 and T_r:
            res["oracle"] = self._oracle_rows(got, oracle_rows)
        flags = torch.tensor([float(differ != 0 or status != 0), float(res.get("oracle", {}).get("bad", 0) > 0)],
                             device=self.dev)
        dist.all_reduce(flags, op=dist.ReduceOp.MAX)
        res["all_ranks_bit_exact"] = bool(flags[0].item() == 0)
        res["ok"] = bool(flags[0].item() == 0 and flags[1].item() == 0)
        return res

    def _oracle_rows(self, got, n: int) -> dict:
        from oracle import moe_oracle as O
        pkg, k, cfg = self.pkg, self.k, self.cfg
        lg = k["lg"].cpu().numpy()
        idx, _ = O.route(lg, k["b"].cpu().numpy(), cfg.routed_scaling_factor)
        pool = {int(g) for p in self.placement for g in p}
        rows = [t for t in range(idx.shape[0]) if any(int(g) in pool for g in idx[t])][:n]
        sub = dict(routing_logits=lg[rows], routing_bias=k["b"].cpu().numpy(),
                   hidden_states=k["hidden"][rows].view(torch.uint8).cpu().numpy(),
                   hidden_states_scale=np.ascontiguousarray(k["hs"][:, rows].cpu().numpy()),
                   local_expert_offset=0, routed_scaling_factor=cfg.routed_scaling_factor)
        out = np.zeros((len(rows), 7168), np.float32)
        for g in sorted({int(g) for t in rows for g in idx[t]} & pool):
            w = pkg.make_weights(cfg, [g], self.dev)
            one = dict(sub, local_expert_offset=g,
                       gemm1_weights=w["gemm1_weights"].view(torch.uint8).cpu().numpy(),
                       gemm1_weights_scale=w["gemm1_weights_scale"].cpu().numpy(),
                       gemm2_weights=w["gemm2_weights"].view(torch.uint8).cpu().numpy(),
                       gemm2_weights_scale=w["gemm2_weights_scale"].cpu().numpy())
            out = O.moe_forward(**one, accumulate=out, return_fp32=True)
        ref = O.f32_to_bf16_bits(out)
        r = O.check_tolerance(ref, got[rows].view(torch.int16).cpu().numpy().view(np.uint16))
        r["rows"] = len(rows)
        return r


def ep_layer_measure(pkg, epm, dist, rank, world, device, cfg, T_global, e_rank, pool, steps, warmup,
                     what: str) -> dict:
    """Layer tokens/s of one expert-parallel configuration (max over ranks), with its parity."""
    case = EpCase(pkg, epm, rank, world, device, cfg, T_global, e_rank, pool)
    try:
        par = case.parity(dist, oracle_rows=4)
        ms = case.time_ms(dist, steps, warmup)
        rt = torch.tensor([case.routes], device=device, dtype=torch.float64)
        parts = [torch.empty_like(rt) for _ in range(world)]
        dist.all_gather(parts, rt)
    finally:
        case.close()
    return {"what": what, "T_global": T_global, "experts_per_rank": e_rank, "experts": len(pool),
            "us_per_layer": round(ms * 1e3, 2), "layer_tokens_per_s": round(T_global / (ms * 1e-3), 1),
            "routes_per_rank": [int(p.item()) for p in parts], "parity": par, "steps": steps}


def layer_1gpu(pkg, device, cfg, steps: int = 10) -> dict:
    """Configuration 3 (or 4) on one GPU: the full 256-expert layer (moe_forward with all 256
    experts local; the N = 1 point of the expert-parallel strong-scaling curve)."""
    inp = pkg.make_inputs(cfg, device)
    step = Step(pkg, inp, device)
    rs = routing_stats(pkg, inp)
    del inp["gemm1_weights"], inp["gemm2_weights"]
    for _ in range(2):
        step()
    us = time_steps(step, steps) / steps * 1e3
    del step
    torch.cuda.empty_cache()
    return {"what": f"{cfg.name}: full 256-expert layer, T={cfg.T}, one GPU (all experts local)",
            "T_global": cfg.T, "experts_per_rank": 256, "experts": 256, "us_per_layer": round(us, 2),
            "layer_tokens_per_s": round(cfg.T / (us * 1e-6), 1), "routes_per_rank": [rs["routes"]],
            "steps": steps}


def bench_ep(args, rank, world, local_rank, dist):
    """Expert-parallel layer over `world` GPUs (weak scaling of configuration 2's per-GPU work).

    Every rank owns 32 experts (N ranks hold experts 0..32N-1 of the 256, spread by expected load
    over the ranks; N = 8 is the full layer); the T = 4096 tokens of configuration 2 are split
    evenly over the ranks. Each rank therefore streams the weights of 32 experts and receives, in
    expectation, the routes of 4096 token-slices, as the one GPU of configuration 2 does.
    `value` counts each token once per 32-expert slice it passes through (4096 * N per step),
    the unit configuration 2 is measured in at N = 1; `layer_tokens_per_s` is 4096 per step.
    """
    pkg = importlib.import_module("15642_moe_b200")
    epm = importlib.import_module("15642_moe_b200.ep")
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    peaks = load_peaks()
    e_rank, T_global = 32, pkg.CONFIGS[2].T
    cfg = pkg.CONFIGS[2]
    case = EpCase(pkg, epm, rank, world, device, cfg, T_global, e_rank, range(e_rank * world))
    placement, ctx, k, w13p, w2p, out = case.placement, case.ctx, case.k, case.w13p, case.w2p, case.out
    rs = {"routes": case.routes, "active": case.active, "max_per_expert": 0, "tiles": 0}
    lo, hi = case.lo, case.hi
    T_r = hi - lo
    mine = {"hidden_states": k["hidden"], "hidden_states_scale": k["hs"], "routing_logits": k["lg"]}
    # Output parity of this very configuration before anything is timed.
    parity = case.parity(dist)

    def step(events=None):
        case(events=events)

    try:
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        sampler = ClockSampler(local_rank)
        sampler.start()
        t_end = time.time() + args.burn_in
        n_burn = torch.zeros(1, device=device)
        while True:                   # every rank runs the same number of steps
            go = torch.tensor([1.0 if time.time() < t_end else 0.0], device=device)
            dist.all_reduce(go, op=dist.ReduceOp.MIN)
            if go.item() == 0.0:
                break
            for _ in range(20):
                step()
            torch.cuda.synchronize()
            n_burn += 20
        dist.barrier()
        torch.cuda.synchronize()
        ms = time_steps(step, args.steps)
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        clocks = sampler.stop()
        status = pkg.device_status(reset=True)

        reps = min(args.steps, 30)
        names = epm.EP_EVENTS
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)] for _ in range(reps)]
        for row in evs:
            for ev in row:
                ev.record()
        torch.cuda.synchronize()
        dist.barrier()
        for r in range(reps):
            step(evs[r])
        torch.cuda.synchronize()
        stages = {n: statistics.mean(evs[r][i].elapsed_time(evs[r][i + 1]) for r in range(reps))
                  for i, n in enumerate(names)}
        work = kernel_work(rs, T_r)
        # No ncu capture of these per-rank workloads exists, so no traffic figure is reported.
        roof = roofline(stages, work, peaks, None)

        # Every rank's load and stage times (the slowest rank sets the step).
        names_all = list(stages)
        mine_t = torch.tensor([rs["routes"], rs["active"]] + [stages[n] for n in names_all],
                              dtype=torch.float64, device=device)
        parts = [torch.empty_like(mine_t) for _ in range(world)]
        dist.all_gather(parts, mine_t)
        per_rank = [p.tolist() for p in parts]

        def ep_layer(h, sc, lg, o):       # the same layer as `step`, on the pipeline's buffers
            ctx.forward(h, sc, w13p, k["s13"], w2p, k["s2"], lg, k["b"], float(cfg.routed_scaling_factor), out=o)

        dist.barrier()
        e2e = e2e_run(pkg, mine, device, args.steps, args.warmup, forward=ep_layer)
        t = torch.tensor([e2e["ms_per_step"]], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e["ms_per_step"] = float(t.item())
        routes_all = torch.tensor([rs["routes"]], device=device, dtype=torch.float64)
        dist.all_reduce(routes_all)
    finally:
        ctx.close()
    # The model's layer at this N (strong scaling): configuration 3, and configuration 4's skewed
    # routing; each checked for parity like the headline case before it is timed.
    del case
    torch.cuda.empty_cache()
    c3, c4 = pkg.CONFIGS[3], pkg.CONFIGS[4]
    config3 = ep_layer_measure(pkg, epm, dist, rank, world, device, c3, c3.T, 256 // world, range(256), 10, 3,
                               "config 3: full 256-expert layer, T=8192 split evenly over the ranks, 256/N "
                               "experts per rank (placement balanced by a calibration batch)")
    torch.cuda.empty_cache()
    config4 = ep_layer_measure(pkg, epm, dist, rank, world, device, c4, c4.T, 256 // world, range(256), 5, 2,
                               "config 4: skewed routing (bias +1.5 on 2 experts per group), T=16384 split "
                               "evenly, 256/N experts per rank (placement balanced by a calibration batch)")
    if rank != 0:
        return None
    slices = T_global * world
    return {
        "metric": METRIC,
        "value": round(slices * args.steps / (ms * 1e-3), 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3 (fp32 accumulate)",
        "data": "synthetic: seeded N(0,1) logits/hidden, N(0,0.1) bias, N(0,0.02) weights, "
                "e4m3 with amax/448 128-block scales",
        "config": config_ep(world),
        "routing": {"T_per_rank": T_r, "routes_all_ranks": int(routes_all.item()), "routes_rank0": rs["routes"],
                    "active_experts_rank0": rs["active"]},
        "layer_tokens_per_s": round(T_global * args.steps / (ms * 1e-3), 1),
        "parity": parity,
        "config3_layer": config3,
        "config4_skew": config4,
        "roofline": roof,
        "stage_us_rank0": {kk: round(v * 1e3, 2) for kk, v in stages.items()},
        "routes_per_rank": [int(p[0]) for p in per_rank],
        "stage_us_slowest_rank": (lambda p: {"rank": per_rank.index(p), **{n: round(v * 1e3, 2) for n, v in
                                                                             zip(names_all, p[2:])}})(
            max(per_rank, key=lambda p: p[2 + names_all.index("gemm1_swiglu")] + p[2 + names_all.index("gemm2_weighted")])),
        "e2e": {"value": round(slices / (e2e["ms_per_step"] * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": e2e["h2d_bytes_per_step"],
                "d2h_bytes_per_step": e2e["d2h_bytes_per_step"],
                "ms_per_step": round(e2e["ms_per_step"], 4), "per": "rank 0 (max over ranks)",
                "api": e2e["api"]},
        "gpu_launches": 10 * args.steps,
        "clocks": clocks,
        "device_status": status,
    }


def bench_reference(args, rank, world):
    """The reference's algorithm on the host CPU cores (oracle/moe_oracle.py, the numpy
    restatement of reference/moe_ref.py; the reference itself is Python and cannot travel), on
    the same configuration, metric and unit as this package's arm at the same N. Inputs come from
    oracle/synth_oracle.py (numpy restatement of the package's generator, same bytes), so this
    arm loads none of the package's compiled code.

    Unit of work: one 32-expert slice of the layer over configuration 2's 4096 tokens (a
    moe_ref.run call; local_expert_offset = 32 r), all of its active experts. At N = 1 that is
    the whole workload and every step times it. At N > 1 the workload is N slices and the unit
    (token-slices) adds over slices, so step i times slice i mod N and the value is
    4096 N / (sum over slices of their mean step time). Rank 0 alone runs; the others exit."""
    if rank != 0:
        return None
    from oracle import moe_oracle as O
    from oracle import synth_oracle as S
    T, seed, rsf = CFG2["T"], CFG2["seed"], CFG2["routed_scaling_factor"]
    logits = S.logits(seed, T)
    bias = (S.bias_bits(seed, 0.1, (), 1.5).astype(np.uint32) << 16).view(np.float32)
    hid, hsc = S.hidden(seed, T)
    idx, _ = O.route(logits, bias, rsf)
    slices, stats = [], []
    for r in range(world):
        off = 32 * r
        sel = idx[(idx >= off) & (idx < off + 32)] - off
        counts = np.bincount(sel.ravel(), minlength=32)
        active = [e for e in range(32) if counts[e] > 0]
        w13 = np.zeros((32, 4096, 7168), np.uint8)
        s13 = np.zeros((32, 32, 56), np.float32)
        w2 = np.zeros((32, 7168, 2048), np.uint8)
        s2 = np.zeros((32, 56, 16), np.float32)
        if active:
            a, b, c, d = S.weights(seed, [off + e for e in active])
            w13[active], s13[active], w2[active], s2[active] = a, b, c, d
        npi = dict(routing_logits=logits, routing_bias=bias, hidden_states=hid, hidden_states_scale=hsc,
                   gemm1_weights=w13, gemm1_weights_scale=s13, gemm2_weights=w2, gemm2_weights_scale=s2,
                   local_expert_offset=off, routed_scaling_factor=rsf)
        O.moe_forward(**npi, experts=active)      # first call pays the page faults; discarded
        slices.append((npi, active))
        stats.append({"local_expert_offset": off, "routes": int(counts.sum()), "active_experts": len(active)})
    times = [[] for _ in range(world)]
    for i in range(args.warmup + args.steps):
        r = i % world
        npi, active = slices[r]
        t0 = time.perf_counter()
        O.moe_forward(**npi, experts=active)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times[r].append(dt)
    timed = [statistics.mean(t) for t in times if t]
    secs = statistics.mean(timed) * world      # CPU seconds of the whole workload of one step
    value = T * world / secs
    cores = os.cpu_count()
    sample = (f"oracle/moe_oracle.py (numpy restatement of reference/moe_ref.py), T={T}, "
              + ("the full layer (all active local experts) every step" if world == 1 else
                 f"step i = 32-expert slice i mod {world} with all its active experts; "
                 f"{sum(1 for t in times if t)} of {world} slices timed")
              + f"; numpy/BLAS on {cores} host threads")
    return {"metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(secs * 1e3, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (same generator and seed, restated in numpy: oracle/synth_oracle.py)",
            "config": config_1gpu() if world == 1 else config_ep(world),
            "routing_slices": stats,
            "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": cores,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def profile_forwards(T: int, n: int = 4) -> None:
    """n forwards of configuration 2's experts on T tokens: input synthesis (5 launches), weight
    packing (2), then 5 kernels per forward."""
    pkg = importlib.import_module("15642_moe_b200")
    inp = pkg.make_inputs(pkg.CONFIGS[2].with_(T=T), "cuda")
    step = Step(pkg, inp, torch.device("cuda"))
    for _ in range(n):
        step()
    torch.cuda.synchronize()
    print("profile_forwards", T, "device status", pkg.device_status(reset=True), file=sys.stderr)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--burn-in", type=float, default=2.0, help="untimed seconds before timing")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-forwards", type=int, default=0, metavar="T",
                    help="profiling driver: run 4 forwards of configuration 2's weights with T tokens "
                         "(seed 0) and exit without timing (for ncu launch lists and captures)")
    args = ap.parse_args()
    if args.profile_forwards:
        profile_forwards(args.profile_forwards)
        return
    args.warmup = max(args.warmup, 3)
    # Standard output carries the one JSON line only: keep a handle on it, then send whatever
    # else writes to file descriptor 1 (NCCL's version banner, library prints) to stderr.
    sys.stdout.flush()
    result_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = bench_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), file=result_out, flush=True)
        return

    dist = None
    if world > 1:
        import datetime
        import torch.distributed as tdist
        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                 device_id=torch.device("cuda", local_rank))
        dist = tdist
    try:
        line = (bench_ours if world == 1 else bench_ep)(args, rank, world, local_rank, dist)
        if line is not None:
            print(json.dumps(line), file=result_out, flush=True)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
