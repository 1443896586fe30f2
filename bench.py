#!/usr/bin/env python
"""Selective-scan fwd+bwd throughput on B200 — the benchmark contract of this repository.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mamba_b200|reference] [--workload W]
    torchrun --nproc-per-node N bench.py --gpus N ...          (N > 1, one rank per GPU)

A step is one forward + backward of the selective scan (public operator
``mamba_b200.selective_scan_fn`` and autograd) over one batch of synthetic inputs at the
north-star point of BASELINE.json: per GPU batch 8, d_inner 1536, seqlen 2048, d_state 16,
bf16 u / delta / z / B / C, fp32 A / D / delta_bias, softplus on, SiLU(z) gate.  Inputs per
step (u, delta, z, dout: 4 x 50 MB) exceed the 126 MB L2, so no flush is needed between
steps.  N GPUs run N batch shards of a global batch 8N (weak scaling; the scan has no
exchange, so no collective runs inside the timed region).  Other scan workloads:
``scan-c0`` (config 0: fp32 forward + final state, batch 2), ``scan-c1`` (config 1: bf16
fwd+bwd, batch 2), ``scan-c2`` (config 2: bf16 forward + final state, batch 1, d_inner 5120,
seqlen 32768) — per-GPU batch fixed; ``scan-c4`` (config 4: d_inner 5120, a global batch of
64 split over the N GPUs: strong scaling).  Workloads whose inputs fit in L2 (configs 0 and
1) flush it between timed steps.

Rank 0 prints one JSON line.  ``value`` is tokens/s of the whole job (inputs resident in
HBM); ``e2e`` is the same metric with pinned-host inputs copied in and all results copied
out every step; ``roofline`` covers the dominant kernel with algorithmic bytes;
``cpu_baseline`` is the CPU oracle port (oracle/ss_oracle.c, fp32, all host threads) on a
bounded sample; ``reference_ext`` (N = 1) times the reference's own CUDA extension against
this library at the same shape in the extension's only mode (fp32, no gate); ``verification``
(N > 1) reports the NCCL all-gather of the shards and their oracle check, done after the
timed regions.  ``--impl reference`` times the CPU port alone: the reference
(nmquan1503/Mamba) has no CPU implementation of its own, and its CUDA extension has no bf16
or z support.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "selective-scan fwd+bwd tokens/s and HBM GB/s (% of ~8 TB/s peak) at 1/2/4/8 B200"
# scan workloads: "scan" is the north-star point (per-GPU batch fixed, weak scaling); "scan-c0",
# "scan-c1" and "scan-c2" are BASELINE configs 0 (fp32 forward + last state), 1 (bf16 fwd+bwd at
# batch 2) and 2 (long-sequence bf16 forward + last state), per-GPU batch fixed; "scan-c4" is
# BASELINE config 4, a Mamba-2.8B-shaped layer whose global batch of 64 is split over the GPUs
# (strong scaling).  dtype: I/O dtype of u / delta / z / B / C (A, D, delta_bias are fp32);
# passes: "fwd+bwd" (autograd step) or "fwd" (forward only); z: SiLU(z) gate; last: the forward
# also returns the final state.
SCAN_WORKLOADS = {
    "scan": dict(b=8, d=1536, L=2048, n=16, scaling="weak", dtype="bf16", passes="fwd+bwd", z=True, last=False,
                 label="selective_scan fwd+bwd, batch 8 per GPU, d_inner 1536, seqlen 2048, d_state 16, "
                       "bf16 I/O + fp32 state, z gate, softplus (north-star point)"),
    "scan-c0": dict(b=2, d=1536, L=2048, n=16, scaling="weak", dtype="f32", passes="fwd", z=False, last=True,
                    label="selective_scan forward + last state, batch 2 per GPU, d_inner 1536, seqlen 2048, "
                          "d_state 16, fp32 I/O, no gate, softplus (config 0)"),
    "scan-c1": dict(b=2, d=1536, L=2048, n=16, scaling="weak", dtype="bf16", passes="fwd+bwd", z=True, last=False,
                    label="selective_scan fwd+bwd, batch 2 per GPU, d_inner 1536, seqlen 2048, d_state 16, "
                          "bf16 I/O + fp32 state, z gate, softplus (config 1)"),
    "scan-c2": dict(b=1, d=5120, L=32768, n=16, scaling="weak", dtype="bf16", passes="fwd", z=True, last=True,
                    label="selective_scan forward + last state, batch 1 per GPU, d_inner 5120, seqlen 32768, "
                          "d_state 16, bf16 I/O + fp32 state, z gate, softplus (config 2, long sequence)"),
    "scan-c4": dict(b=64, d=5120, L=2048, n=16, scaling="strong", dtype="bf16", passes="fwd+bwd", z=True,
                    last=False,
                    label="selective_scan fwd+bwd, global batch 64 split over the GPUs, d_inner 5120, seqlen 2048, "
                          "d_state 16, bf16 I/O + fp32 state, z gate, softplus (config 4, Mamba-2.8B-shaped layer)"),
}
PER_GPU = {k: SCAN_WORKLOADS["scan"][k] for k in ("b", "d", "L", "n")}
ES = {"bf16": 2, "f32": 4}


def scan_shape(workload, world):
    """Per-GPU batch b, the job's global batch, d, L, n and the scaling kind of a scan workload."""
    s = dict(SCAN_WORKLOADS[workload])
    if s["scaling"] == "weak":
        s["global_b"] = s["b"] * world
    else:
        if s["b"] % world:
            raise SystemExit(f"{workload}: the global batch {s['b']} does not split over {world} GPUs")
        s["global_b"], s["b"] = s["b"], s["b"] // world
    return s


def args_():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mamba_b200", choices=["mamba_b200", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=50,
                    help="pipelined end-to-end steps (the loop's fill and drain are spread over them)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU-baseline sample budget")
    ap.add_argument("--no-reference-ext", action="store_true",
                    help="skip the reference extension comparison (N = 1 scan workloads)")
    ap.add_argument("--workload", default="scan",
                    choices=["scan", "scan-c0", "scan-c1", "scan-c2", "scan-c4", "block", "decode", "norm", "model"],
                    help="scan: the north-star selective scan (default); scan-c0 / scan-c1 / scan-c2: BASELINE "
                         "configs 0 (fp32 forward), 1 (bf16 fwd+bwd, batch 2), 2 (bf16 forward, L 32768); "
                         "scan-c4: the scan at config 4 "
                         "(global batch 64 over the GPUs, d_inner 5120); block: one MambaSimple block "
                         "(d_model 768) fwd+bwd, fused mamba_inner_fn against the reference's op sequence; "
                         "decode: a 24-layer CausalLM (d_model 768) decoding 256 tokens after a 128-token prompt "
                         "at batch 64; norm: residual add + RMSNorm fwd+bwd over 16384 x 768 bf16 rows; "
                         "model: one training step (fwd+bwd, cross-entropy) of the 24-layer CausalLM")
    ap.add_argument("--decode-tokens", type=int, default=256, help="decode workload: new tokens per sequence")
    ap.add_argument("--decode-no-cache-tokens", type=int, default=8,
                    help="decode workload: tokens timed for the no-cache alternative (0 skips it)")
    ap.add_argument("--model-path", default="both", choices=["both", "fused", "reference"],
                    help="model workload: time both paths, or only one (for a launch list of one path)")
    ap.add_argument("--block-path", default="both", choices=["both", "fused", "unfused"],
                    help="block workload: time both paths, or only one (for a launch list of one path)")
    return ap.parse_args()


def algorithmic_bytes(b, d, L, n, es=2, z=True, last=False):
    """Bytes the path must move (I/O element size es, variable B / C, fp32 dB / dC).
    fwd: read u, delta (, z); write out          -> (3 + z) es per element; B, C -> 2 n es per
         token; the final state, when returned, 4 n per (batch, channel)
    bwd: read u, delta, dout (, z); write du, ddelta (, dz) -> (5 + 2 z) es per element;
         read B, C (2 n es) and write dB, dC fp32 (2 n 4) per token."""
    elems, tokens = b * d * L, b * L
    fwd = elems * (3 + int(z)) * es + tokens * 2 * n * es + (b * d * n * 4 if last else 0)
    bwd = elems * (5 + 2 * int(z)) * es + tokens * (2 * n * es + 2 * n * 4)
    return fwd, bwd


# warp instructions per warp-step (one lane per channel, 4 states, one time step) of the whole-row
# scan kernels with 2-byte I/O, a gate and dstate 16, from ncu's smsp__inst_executed.sum at the
# north-star point divided by its 3,145,728 warp-steps (profiles/ss_fwd_kernel_north_star.md,
# profiles/ss_bwd_kernel_north_star.md)
INST_PER_WARP_STEP = {"fwd": 124773888 / 3145728, "bwd": 267692544 / 3145728}


def compute_floor(b, d, L, n, ms_step, sm_mhz, z=True, backward=True, io_bytes=2):
    """The step's MUFU (ex2 / lg2 / rcp) work, counted from the kernels' arithmetic, against the
    B200's 148 SMs x 16 MUFU lanes per clock at the sampled SM clock: the compute floor that
    keeps this path far from its HBM roofline.  Per element: forward 1 ex2 per state + 2
    (softplus: ex2, lg2) + 2 with a gate (SiLU: ex2, rcp); backward 2 ex2 per state (the tile's
    forward recompute and the reverse step) + 3 (softplus and its slope: ex2, lg2, rcp) + 2 with
    a gate."""
    elems = b * d * L
    g = 2 if z else 0
    mufu = elems * ((n + 2 + g) + ((2 * n + 3 + g) if backward else 0))
    mhz = sm_mhz or 1965.0
    peak = 148 * 16 * mhz * 1e6
    floor_ms = mufu / peak * 1e3
    out = {"mufu_ops_per_step": mufu, "mufu_peak_ops_per_s": peak, "mufu_floor_ms": floor_ms,
           "mufu_frac": floor_ms / ms_step,
           "note": "MUFU floor of the step at the sampled SM clock; the scan kernels issue at ~45 % of "
                   "peak with latency stalls on shared-memory and MUFU results (ncu summaries)"}
    if z and n == 16 and io_bytes == 2:
        # issue floor: the kernels' measured instruction counts at one warp instruction per
        # scheduler per clock (148 SMs x 4 schedulers); the time-chunk summary passes are not
        # counted, so for a time-chunked step this is a lower bound of the floor
        warp_steps = b * L * (-(-d // 32)) * (n // 4)
        inst = warp_steps * (INST_PER_WARP_STEP["fwd"] + (INST_PER_WARP_STEP["bwd"] if backward else 0.0))
        issue_ms = inst / (148 * 4 * mhz * 1e6) * 1e3
        out.update({"issue_warp_inst_per_step": inst, "issue_floor_ms": issue_ms, "issue_frac": issue_ms / ms_step})
    return out


def load_peaks():
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(workload, kernel):
    """dram bytes (read + write) of one launch of `kernel` at `workload`, from the committed ncu
    table profiles/scan_kernels_dram_traffic.txt (lines "workload kernel bytes"), if present."""
    p = os.path.join(HERE, "profiles", "scan_kernels_dram_traffic.txt")
    try:
        for line in open(p):
            f = line.split()
            if len(f) == 3 and not line.startswith("#") and f[0] == workload and f[1] == kernel:
                return float(f[2])
    except OSError:
        pass
    return None


def count_own_launches(fn):
    """Kernels of this library (C++ namespace ssb) that one call of fn launches, counted by the
    torch profiler outside every timed region: (count, None), or (None, why) if the profiler failed."""
    try:
        import torch
        from torch.profiler import ProfilerActivity, profile

        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        return sum(1 for e in prof.events() if e.device_type.name == "CUDA" and "ssb::" in e.name), None
    except Exception as e:
        return None, repr(e)[:200]


def launches_per_step(d, n, backward):
    """This library's kernels per step: the forward scan, the backward scan with it, and a
    finishing pass after each when the states run in groups (dstate > 16)."""
    per_pass = 2 if n > 16 else 1
    return per_pass * (2 if backward else 1)


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event reasons of this process's GPU, polled through NVML from a
    thread every ~10 ms while the timed region runs, with one sample at each end, so even a
    short region is covered (every rank polls its own GPU: a faster poll adds driver queries
    that contend with the ranks' launches on a shared host).  The GPU is found by UUID (then PCI
    bus id), never by index, because CUDA_VISIBLE_DEVICES may renumber devices."""
    PERIOD_S = 0.010

    def __init__(self, device_index):
        self.dev = device_index
        self.rows, self.h, self.err = [], None, None

    def _handle(self):
        import pynvml as N
        import torch

        N.nvmlInit()
        pr = torch.cuda.get_device_properties(self.dev)
        try:
            return N.nvmlDeviceGetHandleByUUID("GPU-" + str(pr.uuid))
        except Exception:
            return N.nvmlDeviceGetHandleByPciBusId(f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0")

    def _sample(self):
        import pynvml as N

        self.rows.append((N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM),
                          N.nvmlDeviceGetCurrentClocksEventReasons(self.h)))

    def _loop(self):
        while not self.stop.wait(self.PERIOD_S):
            try:
                self._sample()
            except Exception as e:  # keep the samples taken so far
                self.err = repr(e)
                return

    def __enter__(self):
        import threading

        try:
            import pynvml as N

            self.h = self._handle()
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
            self._sample()
        except Exception as e:
            self.h, self.err = None, repr(e)
            return self
        self.stop = threading.Event()
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *exc):
        if self.h is not None:
            self.stop.set()
            self.thread.join(timeout=5)
            try:
                self._sample()
            except Exception as e:
                self.err = repr(e)
        return False

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "error": self.err}
        import pynvml as N

        bits = {"hw_slowdown": N.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": N.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": N.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": N.nvmlClocksEventReasonSwPowerCap}
        reasons = sorted({k for _, r in self.rows for k, bit in bits.items() if r & bit})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.rows), "source": "NVML, 10 ms poll"}


# ----------------------------------------------------------------------------- inputs
def make_inputs(b, d, L, n, seed, device="cpu", dtype="bf16", z=True, dout=True):
    """Seeded inputs with the configs' distributions, generated on `device` (the CPU for the
    north-star point; the GPU for the large configs, whose 168M- to 671M-element tensors take
    minutes to draw on one host thread).  u, delta, z, B, C, dout in `dtype`; A, D, delta_bias
    fp32; z / dout left out when not wanted."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=g, dtype=torch.float32, device=device)
    dt = torch.exp(torch.rand(d, generator=g, device=device) * (math.log(0.1) - math.log(1e-3))
                   + math.log(1e-3)).clamp(min=1e-4)
    io = torch.bfloat16 if dtype == "bf16" else torch.float32
    cv = lambda t: t.to(io)
    x = dict(u=cv(rn(b, d, L)), delta=cv(0.5 * rn(b, d, L)))
    if z:
        x["z"] = cv(rn(b, d, L))
    x.update(B=cv(rn(b, 1, n, L)), C=cv(rn(b, 1, n, L)))
    if dout:
        x["dout"] = cv(rn(b, d, L))
    x.update(A=-torch.arange(1, n + 1, dtype=torch.float32, device=device).repeat(d, 1),
             D=torch.ones(d, device=device), delta_bias=dt + torch.log(-torch.expm1(-dt)))
    return x


# ----------------------------------------------------------------------------- cpu legs
def cpu_sample_rate(n_full_elems, tokens_full, budget_s, seed=0, shape=None):
    """Time the fp32 CPU oracle port (fwd + bwd, all host threads) on a slice of the
    workload sized to ~budget_s, and extrapolate to tokens/s of the full workload."""
    import torch
    from oracle import oracle as O

    shape = shape or SCAN_WORKLOADS["scan"]
    d_full, L, n = shape["d"], shape["L"], shape["n"]
    with_z, bwd, last = shape.get("z", True), shape.get("passes", "fwd+bwd") == "fwd+bwd", shape.get("last", False)

    def run(rows):
        bsl, dsl = (1, rows) if rows <= d_full else (rows // d_full, d_full)
        h = make_inputs(bsl, dsl, L, n, seed, "cpu", dtype="f32", z=with_z, dout=bwd)
        zz = h.get("z")
        t = time.perf_counter()
        O.selective_scan_ref(h["u"], h["delta"], h["A"], h["B"], h["C"], h["D"], zz, h["delta_bias"], True,
                             return_last_state=last, precision="f32", nthreads=threads)
        if bwd:
            O.selective_scan_ref_bwd(h["u"], h["delta"], h["A"], h["B"], h["C"], h["D"], zz, h["delta_bias"], True,
                                     h["dout"], precision="f32", nthreads=threads)
        return time.perf_counter() - t

    # every host thread this process may use (a launcher such as torchrun sets OMP_NUM_THREADS=1
    # for its ranks; the baseline runs on rank 0 alone and takes them all)
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    # calibrate on a slice that keeps every thread busy, then grow the slice (channels first,
    # then whole batch rows) towards ~budget_s, never past the per-GPU workload
    cal = max(8, 8 * threads)
    t_cal = run(cal)
    rows = int(min(n_full_elems // L, shape["b"] * d_full, max(cal, cal * budget_s / max(t_cal, 1e-3))))
    rows = max(8, rows - rows % 8) if rows <= d_full else rows - rows % d_full
    t, reps = run(rows), 1
    while t < budget_s and reps < 64:  # the whole slice was fast: repeat it to fill the budget
        t += run(rows)
        reps += 1
    bsl, dsl = (1, rows) if rows <= d_full else (rows // d_full, d_full)
    rate_elems = reps * rows * L / t
    value = tokens_full / (n_full_elems / rate_elems)
    return value, threads, (f"{reps} x batch {bsl} x {dsl} channels x {L} steps ({'fwd+bwd' if bwd else 'fwd'}, "
                            f"fp32 port) "
                            f"in {t:.2f} s"), t


def reference_arm(a, world, rank):
    if rank != 0:
        return 0
    shape = scan_shape(a.workload if a.workload in SCAN_WORKLOADS else "scan", world)
    b, d, L, n = shape["global_b"], shape["d"], shape["L"], shape["n"]
    elems, tokens = b * d * L, b * L
    per_step_budget = max(1.0, 120.0 / max(1, a.steps + a.warmup))
    vals = []
    sample = threads = None
    for i in range(a.warmup + a.steps):
        v, threads, sample, _ = cpu_sample_rate(elems, tokens, per_step_budget, seed=i, shape=shape)
        if i >= a.warmup:
            vals.append(v)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * tokens / value, "higher_is_better": True,
        "scaling": shape["scaling"], "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(world, shape),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"per step: {sample}; extrapolated to the workload's elements"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference has no CPU implementation; this is the CPU restatement of its "
                "algorithm (oracle/ss_oracle.c) with OpenMP over channels",
    }
    print(json.dumps(line), flush=True)
    return 0


L2_BYTES = 126 * 1024 * 1024


def step_input_bytes(shape):
    """Bytes of the per-element tensors a step reads (u, delta, z, dout) on one GPU."""
    b, d, L = shape["b"], shape["d"], shape["L"]
    k = 2 + int(shape["z"]) + int(shape["passes"] == "fwd+bwd")
    return k * b * d * L * ES[shape["dtype"]]


def flushes_l2(shape):
    """Workloads whose step inputs fit in the L2 get the L2 flushed between timed steps; the others
    read more than the L2 holds every step."""
    return step_input_bytes(shape) <= L2_BYTES


def parallelism(world, shape):
    if world == 1:
        return "x1, no collective"
    if shape["passes"] == "fwd+bwd":
        return (f"batch-sharded x{world}; per step one NCCL all-reduce of the partial dA / dD / "
                f"ddelta_bias (mamba_b200.sharding.reduce_param_grads) inside the step")
    return f"batch-sharded x{world}, forward only: no exchange in the step"


def config_dict(world, shape):
    b, d, L = shape["b"], shape["d"], shape["L"]
    mb = step_input_bytes(shape) / 1e6
    l2 = (f"L2 flushed between timed steps (a 256 MiB buffer written outside the per-step events; "
          f"{mb:.0f} MB of per-element inputs per GPU per step)" if flushes_l2(shape) else
          f"inputs larger than L2 ({mb:.0f} MB of per-element inputs per GPU per step)")
    return {"workload": shape["label"],
            "global_batch": shape["global_b"], "per_gpu_batch": b, "d_inner": d, "seq_len": L,
            "d_state": shape["n"], "parallelism": parallelism(world, shape),
            "l2": l2}


# ----------------------------------------------------------------------------- baselines / checks
REF_SO = os.path.join(HERE, "oracle", "_ref", "selective_scan.so")


def gpu_lead(ms=50.0):
    """Enqueue ~ms of idle GPU work (a spin kernel) so the host gets ahead of the device before a
    timed region: the CUDA events that bracket each step then measure the device's time for the
    step, not the host's launch latency (which matters for the sub-millisecond small-batch steps)
    nor a host-side hiccup shorter than the lead.  The lead itself lies before the first event of
    the region."""
    import torch

    torch.cuda._sleep(int(ms * 1e-3 * 2.0e9))


class quiet_host:
    """No Python garbage collection inside a timed region (one full collection just before it),
    as timeit does: a collector pause on the host would otherwise stall the launches."""

    def __enter__(self):
        import gc

        self.was = gc.isenabled()
        gc.collect()
        gc.disable()
        return self

    def __exit__(self, *exc):
        import gc

        if self.was:
            gc.enable()


def _timed_calls(fn, iters, warmup=3, scrub=None):
    """Mean ms of fn() over `iters` calls on the current stream (CUDA events per call, the host
    ahead of the device; the L2 is flushed before each call when `scrub` is given, outside the
    call's events)."""
    import torch

    for _ in range(warmup):
        if scrub is not None:
            scrub.zero_()  # its kernel loads here, not inside the timed calls
        fn()
    torch.cuda.synchronize()
    evs = []
    with quiet_host():
        gpu_lead()
        for _ in range(iters):
            if scrub is not None:
                scrub.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            evs.append((e0, e1))
        torch.cuda.synchronize()
    return statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)


def host_link(dev, pin, dbuf, names, outs_host, s_in, s_out, e2e_ms, step_ms, reps=3):
    """The host link alone, outside every timed region: one step's input bytes host -> device,
    its result bytes device -> host, and both at once (the pipelined end-to-end step moves both
    concurrently), each the best of `reps` CUDA-event timings on the end-to-end loop's streams.
    floor_ms = max(both at once, the device step): what a perfectly overlapped end-to-end step
    would take; frac = floor_ms / the measured end-to-end step."""
    import torch

    dres = [torch.empty(h.shape, dtype=h.dtype, device=dev) for h in outs_host]
    h2d = sum(pin[k].numel() * pin[k].element_size() for k in names)
    d2h = sum(h.numel() * h.element_size() for h in outs_host)

    def timed(do_in, do_out):
        best = None
        for _ in range(reps):
            cur = torch.cuda.current_stream(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record(cur)
            for st in (s_in, s_out):
                st.wait_stream(cur)
            if do_in:
                with torch.cuda.stream(s_in):
                    for k in names:
                        dbuf[k].copy_(pin[k], non_blocking=True)
            if do_out:
                with torch.cuda.stream(s_out):
                    for hb, db in zip(outs_host, dres):
                        hb.copy_(db, non_blocking=True)
            for st in (s_in, s_out):
                cur.wait_stream(st)
            e1.record(cur)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        return best

    ms_in, ms_out, ms_both = timed(True, False), timed(False, True), timed(True, True)
    floor = max(ms_both, step_ms)
    return {"h2d_gbs": h2d / ms_in / 1e6, "d2h_gbs": d2h / ms_out / 1e6, "both_ms": ms_both,
            "floor_ms": floor, "frac": floor / e2e_ms}


def reference_ext_compare(shape, dev, backward, iters=5):
    """The reference's own CUDA extension (csrc/selective_scan/*, compiled unmodified from its
    sources into oracle/_ref/ by oracle/build_ref.py) against this library on the same GPU, at
    this workload's shape in the only mode the extension supports: fp32 I/O, no gate.  Both run
    through the same positional entry points (selective_scan.cpp:331-334 of the reference;
    mamba_b200.selective_scan_ext here), on identical seeded inputs; outputs are compared as a
    sanity check.  A baseline measurement beside the bench line, not part of the timed step."""
    import importlib.util

    import torch

    import mamba_b200.selective_scan_ext as ours

    if not os.path.exists(REF_SO):
        return {"unavailable": "reference extension not built (oracle/build_ref.py needs the reference sources)"}
    spec = importlib.util.spec_from_file_location("selective_scan", REF_SO)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    b, d, L, n = shape["b"], shape["d"], shape["L"], shape["n"]
    x = make_inputs(b, d, L, n, seed=7, device=dev, dtype="f32", z=False, dout=backward)
    args = (x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["delta_bias"])
    scrub = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev) if flushes_l2(
        dict(shape, dtype="f32", z=False)) else None
    r_out, r_x = ref.forward(*args, True)
    o_out, o_x = ours.forward(*args, True)
    torch.cuda.synchronize()
    diff = (o_out - r_out).abs()
    excess = float((diff / (1e-5 + 1e-4 * r_out.abs())).max())
    del diff
    res = {"mode": "fp32 I/O, no gate (the reference extension's only mode), same shape, GPU and inputs",
           "out_max_excess_fp32_tol": excess}
    for tag, mod, xs in (("reference_ext", ref, r_x), ("mamba_b200", ours, o_x)):
        if backward:
            ms = _timed_calls(lambda: mod.backward(*args, x["dout"], mod.forward(*args, True)[1], True), iters,
                              scrub=scrub)
        else:
            ms = _timed_calls(lambda: mod.forward(*args, True), iters, scrub=scrub)
        res[f"{tag}_ms"] = ms
        res[f"{tag}_tokens_per_s"] = b * L / (ms / 1e3)
    res["pass"] = "fwd+bwd" if backward else "fwd"
    res["speedup"] = res["reference_ext_ms"] / res["mamba_b200_ms"]
    return res


def verify_shards(x, host, shape, rank, world, dev, step, backward):
    """Verification of a sharded run (outside every timed region), through
    mamba_b200.sharding.verify: every rank recomputes its shard, the shards' outputs are
    all-gathered over NCCL with their owners' checksums, and each rank checks three sampled
    (batch row, channel) rows of its shard — out and, with a backward, du / ddelta / dz —
    against the CPU oracle (rows are independent, so a row's inputs alone determine them)."""
    import numpy as np
    import torch

    from mamba_b200 import sharding
    from oracle import oracle as O

    b, d, L, n = shape["b"], shape["d"], shape["L"], shape["n"]
    if backward:
        for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias"):
            if k in x:
                x[k].grad = None
        out, _ = step(x)
        out.backward(x["dout"])
    else:
        with torch.no_grad():
            out, _ = step(x)
    torch.cuda.synchronize()
    rtol, atol = (1e-4, 1e-5) if shape["dtype"] == "f32" else (2e-2, 5e-2)
    br, chans = rank % b, sorted({0, d // 2 + 1, d - 1})
    sl = lambda t: t[br:br + 1, chans].float()
    hz = host.get("z")
    args = (sl(host["u"]), sl(host["delta"]), host["A"][chans], host["B"][br:br + 1].float(),
            host["C"][br:br + 1].float(), host["D"][chans], None if hz is None else sl(hz),
            host["delta_bias"][chans], True)
    got, want = [out.detach()[br:br + 1, chans]], [O.selective_scan_ref(*args)]
    if backward:
        g = O.selective_scan_ref_bwd(*args, sl(host["dout"]))
        got += [x["u"].grad[br:br + 1, chans], x["delta"].grad[br:br + 1, chans]]
        want += [g["du"], g["ddelta"]]
        if hz is not None:
            got.append(x["z"].grad[br:br + 1, chans])
            want.append(g["dz"])
    got_rows = torch.cat([t.float().reshape(-1).cpu() for t in got])
    want_rows = np.concatenate([np.asarray(w, np.float64).reshape(-1) for w in want])
    s = sharding.plan(b * world, d, world, rank)
    rep = sharding.verify(out.detach(), s, got_rows, want_rows, rtol, atol)
    res = {"shards": world, "collective": "NCCL all_gather of every shard's output (mamba_b200.sharding.verify)",
           "gathered_bytes": int(rep["gathered"].numel() * rep["gathered"].element_size()),
           "checksum_bad_ranks": rep["checksum_bad_ranks"], "rows_checked_per_shard": len(chans),
           "max_row_excess": max(rep["row_excess"]), "bad_ranks": rep["bad_ranks"],
           "tolerance": f"rtol {rtol}, atol {atol} against the CPU oracle", "pass": rep["ok"]}
    del rep
    if rank == 0:
        print(f"[bench] shard verification: {json.dumps(res)}", file=sys.stderr, flush=True)
    return res


# ----------------------------------------------------------------------------- gpu arm
# ----------------------------------------------------------------------------- block / decode workloads
def _mamba_block(dm, n=16, K=4):
    """A block with MambaSimple's parameter names, shapes and initial values
    (modules/mamba_simple.py:9-85; expansion 2, dt_rank ceil(dm / 16), no biases)."""
    import torch
    import torch.nn as nn

    d, R = 2 * dm, math.ceil(dm / 16)
    blk = nn.Module()
    blk.input_proj = nn.Linear(dm, 2 * d, bias=False)
    blk.short_conv = nn.Conv1d(d, d, K, padding=K - 1, groups=d, bias=False)
    blk.ssm_param_proj = nn.Linear(d, R + 2 * n, bias=False)
    blk.delta_proj = nn.Linear(R, d, bias=True)
    nn.init.uniform_(blk.delta_proj.weight, -R ** -0.5, R ** -0.5)
    dt = torch.exp(torch.rand(d) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3)).clamp(min=1e-4)
    with torch.no_grad():
        blk.delta_proj.bias.copy_(dt + torch.log(-torch.expm1(-dt)))
    blk.log_A = nn.Parameter(torch.log(torch.arange(1, n + 1, dtype=torch.float32)).repeat(d, 1))
    blk.D = nn.Parameter(torch.ones(d))
    blk.output_proj = nn.Linear(d, dm, bias=False)
    return blk


# Mamba-130M-shaped CausalLM (24 layers, d_model 768, vocab 50280 with tied
# embeddings, RMSNorm eps 1e-5)
LM_VOCAB, LM_EPS = 50280, 1e-5


def _causal_lm(vocab, dm, layers, n=16, K=4, eps=LM_EPS):
    """A model with the reference CausalLM's module tree (models/causal_lm.py:20-58): embedding,
    layers of (RMSNorm, MambaSimple block), final RMSNorm, lm_head tied to the embedding."""
    import torch
    import torch.nn as nn

    class RMSNorm(nn.Module):  # modules/rms_norm.py:4-30
        def __init__(self, dim, eps):
            super().__init__()
            self.eps, self.weight = eps, nn.Parameter(torch.zeros(dim))

        def forward(self, x):
            xf = x.float()
            return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * (1.0 + self.weight.float())
                    ).type_as(x)

    m = nn.Module()
    m.embedding = nn.Embedding(vocab, dm)
    m.layers = nn.ModuleList()
    for _ in range(layers):
        layer = nn.Module()
        layer.norm, layer.mamba = RMSNorm(dm, eps), _mamba_block(dm, n, K)
        m.layers.append(layer)
    m.norm = RMSNorm(dm, eps)
    m.lm_head = nn.Linear(dm, vocab, bias=False)
    m.lm_head.weight = m.embedding.weight
    return m


def decode_bench(a):
    """Decoding with a 24-layer CausalLM-shaped model (d_model 768, d_inner 1536, N 16, vocab
    50280; the decode of the 24-layer model config): batch 64, a 128-token prompt, then 256 new
    tokens (greedy), bf16.  Reports new tokens per second over the decode loop (prompt prefill
    timed separately) for the CUDA-graph step and the eager step, and — as the reference's
    alternative, since its generate() is a stub and MambaSimple has no step — the cost of one
    full forward over the sequence per new token (fused path, no cache), timed on 8 tokens."""
    import torch

    from mamba_b200 import mamba_simple_forward
    from mamba_b200.decode import Decoder

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    vocab, dm, layers, b, L0, T = LM_VOCAB, 768, 24, 64, 128, a.decode_tokens
    torch.manual_seed(0)
    model = _causal_lm(vocab, dm, layers).to(dev, torch.bfloat16).eval()
    prompt = torch.randint(0, vocab, (b, L0), generator=torch.Generator().manual_seed(1)).to(dev)

    def ev():
        return torch.cuda.Event(enable_timing=True)

    def run(cuda_graph):
        dec = Decoder(model, b, cuda_graph=cuda_graph)
        logits = dec.prefill(prompt)
        tok = logits.argmax(-1)
        for _ in range(a.warmup):  # warm-up steps (the graph is captured on the first)
            tok = dec.step(tok).argmax(-1)
        torch.cuda.synchronize()  # the timed run reuses this decoder: prefill overwrites its states
        e0, e1, e2 = ev(), ev(), ev()
        with ClockSampler(dev.index) as clk:
            e0.record()
            logits = dec.prefill(prompt)
            e1.record()
            tok = logits.argmax(-1)
            for _ in range(T):
                tok = dec.step(tok).argmax(-1)
            e2.record()
            torch.cuda.synchronize()
        return e0.elapsed_time(e1), e1.elapsed_time(e2), clk.summary()

    with torch.no_grad():
        pre_g, dec_g, clocks = run(True)
        _, dec_e, _ = run(False)
        nc = a.decode_no_cache_tokens
        naive_ms = float("nan")
        if nc > 0:
            ids = torch.cat([prompt, prompt[:, :nc]], 1)
            fwd = lambda L: model.lm_head(_lm_hidden(model, ids[:, :L], mamba_simple_forward)[:, -1])
            for _ in range(2):
                fwd(L0 + 1)
            torch.cuda.synchronize()
            e0, e1 = ev(), ev()
            e0.record()
            for i in range(nc):
                fwd(L0 + 1 + i).argmax(-1)
            e1.record()
            torch.cuda.synchronize()
            naive_ms = e0.elapsed_time(e1) / nc
    n_params = sum(p.numel() for p in model.parameters())
    d, n = 2 * dm, 16
    step_bytes = 2 * n_params + layers * b * d * (n + 3) * 4 * 2  # weights once + SSM / conv states in and out
    step_ms = dec_g / T
    line = {
        "workload": "decode", "metric": "CausalLM decode tokens/s (24 layers, d_model 768, batch 64)",
        "value": b * T / (dec_g / 1e3), "unit": "tokens/s", "ms_per_token_step": step_ms,
        "eager_value": b * T / (dec_e / 1e3), "eager_ms_per_token_step": dec_e / T,
        "no_cache_value": b / (naive_ms / 1e3), "no_cache_ms_per_token_step": naive_ms,
        "prefill_ms": pre_g, "prompt_tokens_per_s": b * L0 / (pre_g / 1e3),
        "roofline": {"bound": "hbm", "bytes_per_step": step_bytes, "achieved": step_bytes / (step_ms / 1e3) / 1e9,
                     "peak": load_peaks()[0], "unit": "GB/s",
                     "frac": step_bytes / (step_ms / 1e3) / 1e9 / load_peaks()[0]},
        "n_gpus": 1, "higher_is_better": True, "dtype": "bf16", "data": "synthetic (random weights, random prompt)",
        "config": {"workload": "24-layer CausalLM, d_model 768, d_inner 1536, d_state 16, vocab 50280, batch 64, "
                               "prompt 128, 256 new tokens, greedy", "params": n_params},
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    return 0


def norm_bench(a):
    """Residual add + RMSNorm (the reference's Block add, models/causal_lm.py:37, and RMSNorm,
    modules/rms_norm.py:21-30) over the rows of one training step of the 24-layer config
    (batch 8 x seqlen 2048 = 16384 rows of d_model 768, bf16), forward + backward: the fused
    kernels against the reference's PyTorch ops.  Algorithmic bytes per row: forward reads x and
    the residual and writes y and the sum (4 x 2 B x 768); backward reads the sum, dy and the
    incoming residual gradient and writes dh (4 x 2 B x 768)."""
    import torch

    from mamba_b200.norm import rms_norm_fn

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rows, dim = 16384, 768
    g = torch.Generator().manual_seed(0)
    x = torch.randn(rows, dim, generator=g).to(dev, torch.bfloat16).requires_grad_()
    r = torch.randn(rows, dim, generator=g).to(dev, torch.bfloat16).requires_grad_()
    w = (0.1 * torch.randn(dim, generator=g)).to(dev).requires_grad_()
    dy = torch.randn(rows, dim, generator=g).to(dev, torch.bfloat16)
    dh = torch.randn(rows, dim, generator=g).to(dev, torch.bfloat16)

    def clear():  # fresh .grad every step: no accumulation kernels in either path
        x.grad = r.grad = w.grad = None

    def ref():
        clear()
        h = x + r
        hf = h.float()
        y = (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-6) * (1.0 + w.float())).type_as(h)
        torch.autograd.backward([y, h], [dy, dh])

    def fused():
        clear()
        y, h = rms_norm_fn(x, w, r, 1e-6, True, True)
        torch.autograd.backward([y, h], [dy, dh])

    def timed(fn):
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / a.steps

    def graphed(fn):
        # the same step captured in a CUDA graph and replayed: the GPU's time for it, without the
        # host-side Python / autograd overhead that bounds an eager step of this size (inside a
        # training step the GPU, not the host, sets the pace)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        for _ in range(a.warmup):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / a.steps

    ms_ref, ms_f = timed(ref), timed(fused)
    gms_ref, gms_f = graphed(ref), graphed(fused)
    nbytes = rows * dim * 2 * 8
    peak = load_peaks()[0]
    line = {"workload": "norm", "metric": "residual add + RMSNorm fwd+bwd rows/s (16384 x 768, bf16)",
            "value": rows / (gms_f / 1e3), "unit": "rows/s", "ms_per_step": gms_f,
            "reference_ops_ms_per_step": gms_ref, "speedup_vs_reference_ops": gms_ref / gms_f,
            "timing": "CUDA-graph replay of each path's fwd + bwd step (GPU time)",
            "eager_ms_per_step": ms_f, "eager_reference_ops_ms_per_step": ms_ref,
            "roofline": {"bound": "hbm", "algorithmic_bytes": nbytes, "achieved": nbytes / (gms_f / 1e3) / 1e9,
                         "peak": peak, "unit": "GB/s", "frac": nbytes / (gms_f / 1e3) / 1e9 / peak,
                         "note": "fwd + bwd kernels and the small kernels of the autograd glue, replayed "
                                 "together"},
            "n_gpus": 1, "higher_is_better": True, "dtype": "bf16", "data": "synthetic"}
    print(json.dumps(line), flush=True)
    return 0


def model_bench(a):
    """One training step (forward, cross-entropy over the vocabulary, backward; no optimizer)
    of the 24-layer CausalLM config (d_model 768, d_inner 1536, N 16, vocab 50280) at batch 8 x
    seqlen 2048, bf16 parameters, two ways on the same model and tokens:
      fused:     mamba_b200.causal_lm_forward (fused blocks; residual add fused with RMSNorm);
      reference: the reference CausalLM's own forward structure (models/causal_lm.py:30-58: torch
                 RMSNorm, MambaSimple's op sequence with its permute copies,
                 modules/mamba_simple.py:87-151) with mamba_b200's scan as its SelectiveScanFn —
                 what the reference runs after the drop-in alone."""
    import torch
    import torch.nn.functional as F

    import mamba_b200
    from mamba_b200 import causal_lm_forward

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    vocab, dm, layers, b, L = LM_VOCAB, 768, 24, 8, 2048
    d, n, K = 2 * dm, 16, 4
    R = math.ceil(dm / 16)
    torch.manual_seed(0)
    model = _causal_lm(vocab, dm, layers).to(dev, torch.bfloat16).train()
    ids = torch.randint(0, vocab, (b, L + 1), generator=torch.Generator().manual_seed(1)).to(dev)
    inp, tgt = ids[:, :-1], ids[:, 1:]

    def mamba_ref(blk, x):  # modules/mamba_simple.py:87-151
        xs, zs = torch.chunk(blk.input_proj(x).permute(0, 2, 1).contiguous(), 2, dim=1)
        xs = F.silu(blk.short_conv(xs)[..., :L])
        dbl = blk.ssm_param_proj(xs.permute(0, 2, 1).contiguous().view(b * L, d))
        dr, B, C = torch.split(dbl, [R, n, n], dim=-1)
        delta = (blk.delta_proj.weight @ dr.t()).view(d, b, L).permute(1, 0, 2).contiguous()
        B = B.view(b, L, n).permute(0, 2, 1).contiguous().unsqueeze(1)
        C = C.view(b, L, n).permute(0, 2, 1).contiguous().unsqueeze(1)
        y = mamba_b200.selective_scan_fn(xs, delta, -torch.exp(blk.log_A.float()), B, C, blk.D.float(), None,
                                         blk.delta_proj.bias.float(), True)
        hs = y.permute(0, 2, 1).contiguous()
        hs = hs * F.silu(zs.permute(0, 2, 1).contiguous())
        return blk.output_proj(hs)

    def ref_forward(x_ids):  # models/causal_lm.py:30-58
        h = model.embedding(x_ids)
        for layer in model.layers:
            r = h
            h = mamba_ref(layer.mamba, layer.norm(h)) + r
        return model.lm_head(model.norm(h))

    def timed(fwd):
        def step():
            loss = F.cross_entropy(fwd(inp).float().view(-1, vocab), tgt.reshape(-1))
            loss.backward()
            for p_ in model.parameters():
                p_.grad = None
        for _ in range(a.warmup):
            step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index) as clk:
            e0.record()
            for _ in range(a.steps):
                step()
            e1.record()
            torch.cuda.synchronize()
        return e0.elapsed_time(e1) / a.steps, clk.summary()

    ms_ref = ms_f = float("nan")
    clocks = None
    if a.model_path in ("both", "reference"):
        ms_ref, clocks = timed(ref_forward)
    if a.model_path in ("both", "fused"):
        ms_f, clocks = timed(lambda x: causal_lm_forward(model, x))
    tokens = b * L
    line = {"workload": "model", "metric": "24-layer CausalLM training step tokens/s (fwd + bwd, batch 8 x 2048)",
            "value": tokens / (ms_f / 1e3), "unit": "tokens/s", "ms_per_step": ms_f,
            "reference_structure_value": tokens / (ms_ref / 1e3), "reference_structure_ms_per_step": ms_ref,
            "speedup_vs_reference_structure": ms_ref / ms_f, "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
            "higher_is_better": True, "dtype": "bf16", "data": "synthetic (random weights and tokens)",
            "config": {"workload": "CausalLM 24 layers, d_model 768, d_inner 1536, d_state 16, vocab 50280 (tied), RMSNorm eps 1e-5, "
                                   "batch 8, seqlen 2048, bf16 parameters, cross-entropy loss, no optimizer step",
                       "params": sum(p_.numel() for p_ in model.parameters())},
            "clocks": clocks}
    print(json.dumps(line), flush=True)
    return 0


def _lm_hidden(model, ids, block_forward):
    h = model.embedding(ids)
    for layer in model.layers:
        h = h + block_forward(layer.mamba, layer.norm(h))
    return model.norm(h)
def block_bench(a):
    """One MambaSimple block (d_model 768 -> d_inner 1536, N 16, conv width 4; the layer of the
    24-layer model config) fwd+bwd at batch 8 x seqlen 2048, bf16, through
      fused:   mamba_b200.mamba_simple_forward (conv+SiLU kernel, GEMMs on transposed views,
               scan with the gate fused, no permute copies), and
      unfused: the reference's own op sequence (modules/mamba_simple.py:87-151: permute +
               contiguous copies, cuDNN depthwise conv, SiLU, the gate as separate kernels)
               with mamba_b200.selective_scan_fn as its SelectiveScanFn — what a user of the
               reference gets from the drop-in scan alone.
    Same parameters, inputs and output gradient for both."""
    import torch
    import torch.nn as nn
    import torch.nn.functional as F

    import mamba_b200

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dm, d, n, K, b, L = 768, 1536, 16, 4, 8, 2048
    R = math.ceil(dm / 16)
    torch.manual_seed(0)
    blk = _mamba_block(dm, n, K).to(dev, torch.bfloat16)
    g = torch.Generator().manual_seed(1)
    h = torch.randn(b, L, dm, generator=g).to(dev, torch.bfloat16).requires_grad_()
    dy = torch.randn(b, L, dm, generator=g).to(dev, torch.bfloat16)

    def unfused(x):
        xs, zs = torch.chunk(blk.input_proj(x).permute(0, 2, 1).contiguous(), 2, dim=1)
        xs = F.silu(blk.short_conv(xs)[..., :L])
        dbl = blk.ssm_param_proj(xs.permute(0, 2, 1).contiguous().view(b * L, d))
        dr, B, C = torch.split(dbl, [R, n, n], dim=-1)
        delta = (blk.delta_proj.weight @ dr.t()).view(d, b, L).permute(1, 0, 2).contiguous()
        B = B.view(b, L, n).permute(0, 2, 1).contiguous().unsqueeze(1)
        C = C.view(b, L, n).permute(0, 2, 1).contiguous().unsqueeze(1)
        A = -torch.exp(blk.log_A.float())
        y = mamba_b200.selective_scan_fn(xs, delta, A, B, C, blk.D.float(), None, blk.delta_proj.bias.float(), True)
        hs = y.permute(0, 2, 1).contiguous()
        hs = hs * F.silu(zs.permute(0, 2, 1).contiguous())
        return blk.output_proj(hs)

    def fused(x):
        return mamba_b200.mamba_simple_forward(blk, x)

    def timed(fn):
        def step():
            out = fn(h)
            out.backward(dy)
            h.grad = None
            for p_ in blk.parameters():
                p_.grad = None
        for _ in range(a.warmup):
            step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index) as clk:
            e0.record()
            for _ in range(a.steps):
                step()
            e1.record()
            torch.cuda.synchronize()
        return e0.elapsed_time(e1) / a.steps, clk.summary()

    ms_u = ms_f = float("nan")
    clocks = None
    if a.block_path in ("both", "unfused"):
        ms_u, clocks = timed(unfused)
    if a.block_path in ("both", "fused"):
        ms_f, clocks = timed(fused)
    tokens = b * L
    line = {
        "workload": "block", "metric": "Mamba block (MambaSimple, d_model 768) fwd+bwd tokens/s",
        "value": tokens / (ms_f / 1e3), "unit": "tokens/s", "ms_per_step": ms_f,
        "unfused_value": tokens / (ms_u / 1e3), "unfused_ms_per_step": ms_u, "speedup_vs_unfused": ms_u / ms_f,
        "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "one MambaSimple block fwd+bwd, batch 8, seqlen 2048, d_model 768, d_inner 1536, "
                               "d_state 16, conv width 4, dt_rank 48, bf16 parameters and activations",
                   "global_batch": b, "seq_len": L, "l2": "activations larger than L2"},
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    a = args_()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        return reference_arm(a, world, rank)
    if a.warmup < 3:
        a.warmup = 3
    if a.workload == "block":
        return block_bench(a) if rank == 0 else 0
    if a.workload == "decode":
        return decode_bench(a) if rank == 0 else 0
    if a.workload == "norm":
        return norm_bench(a) if rank == 0 else 0
    if a.workload == "model":
        return model_bench(a) if rank == 0 else 0

    import torch
    import torch.distributed as dist

    import mamba_b200

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        # NCCL prints its version line on stdout when its communicator starts: send it to stderr,
        # so rank 0's stdout stays one JSON line
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=180))
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)

    shape = scan_shape(a.workload, world)
    b, d, L, n = shape["b"], shape["d"], shape["L"], shape["n"]
    with_z, backward, last = shape["z"], shape["passes"] == "fwd+bwd", shape["last"]
    mk = dict(dtype=shape["dtype"], z=with_z, dout=backward)
    if b * d * L <= 32 * 1024 * 1024:  # small configs: drawn on the host, like the tests
        host = make_inputs(b, d, L, n, seed=1000 + rank, device="cpu", **mk)
        x = {k: v.to(dev) for k, v in host.items()}
    else:
        x = make_inputs(b, d, L, n, seed=1000 + rank, device=dev, **mk)
        host = {k: v.cpu() for k, v in x.items()}
    leaves = [k for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias") if k in x]

    def step(t):
        r = mamba_b200.selective_scan_fn(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t.get("z"),
                                         t["delta_bias"], True, return_last_state=last)
        return r if last else (r, None)

    from mamba_b200 import sharding

    shard = sharding.plan(b * world, d, world, rank)
    exchange = world > 1 and backward

    def reduce_grads(t):
        """The sharded training step's one exchange: the batch shards' partial dA / dD /
        ddelta_bias summed over the ranks (one NCCL all-reduce, inside the step)."""
        sharding.reduce_param_grads({"dA": t["A"].grad, "dD": t["D"].grad if t.get("D") is not None else None,
                                     "ddelta_bias": t["delta_bias"].grad if t.get("delta_bias") is not None else None},
                                    shard)

    def scan_step(t):
        """One step of this rank's shard; returns (out, last_state | None).  Forward-only
        workloads run without autograd."""
        if backward:
            out, ls = step(t)
            out.backward(t["dout"])
            return out, ls
        with torch.no_grad():
            return step(t)

    def run_step(t):
        r = scan_step(t)
        if exchange:
            reduce_grads(t)
        return r

    def clear(t):
        for k in leaves:
            t[k].grad = None

    def barrier():
        if world > 1:
            dist.barrier()

    if backward:
        for k in leaves:
            x[k].requires_grad_(True)
    K = a.steps
    flush = flushes_l2(shape)
    scrub = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev) if flush else None
    for _ in range(a.warmup):
        if flush:
            scrub.zero_()  # its kernel loads here, not inside the timed region
        run_step(x)
        one_span = exchange and sharding._adjacent_span(
            [x[k].grad for k in ("A", "D", "delta_bias") if x.get(k) is not None]) is not None
        clear(x)
    torch.cuda.synchronize()

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clk, quiet_host():
        gpu_lead()  # outside the region: the host runs ahead of the device through it
        t0.record()
        for i in range(K):
            if flush:
                scrub.zero_()  # evicts the previous step's tensors from L2 (outside the step's events)
            ev[i][0].record()
            if backward:
                out, _ = step(x)
                ev[i][1].record()
                out.backward(x["dout"])
                if exchange:
                    reduce_grads(x)
            else:
                with torch.no_grad():
                    out, _ = step(x)
                ev[i][1].record()
            ev[i][2].record()
            clear(x)
        t1.record()
        torch.cuda.synchronize()
        barrier()
    # ms: the whole region, or with a flush the sum of the steps' own event intervals
    elapsed = sum(e[0].elapsed_time(e[2]) for e in ev) if flush else t0.elapsed_time(t1)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev) if backward else 0.0
    if world > 1:
        tt = torch.tensor([elapsed], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        elapsed = float(tt.item())
    ms_step = elapsed / K
    tokens_job = b * L * world
    value = tokens_job / (ms_step / 1e3)

    # ---- end to end: pinned host inputs in, every result out, through the public operator.
    # Steps are independent, so the loop is pipelined over three streams: step i+1's inputs are
    # copied in while step i computes, and step i's results are copied out while step i+1
    # computes (the host link is full duplex); a sharded step's gradient exchange runs on a fourth.  Every step still moves all of its bytes both
    # ways; inputs alternate between two device buffer sets.
    names = tuple(k for k in ("u", "delta", "z", "B", "C", "dout", "A", "D", "delta_bias") if k in host)
    pin = {k: v.pin_memory() for k, v in host.items()}
    bufs = [{k: torch.empty_like(v, device=dev) for k, v in host.items()} for _ in range(2)]
    s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s_x = torch.cuda.Stream(dev) if exchange else None
    E = max(1, a.e2e_steps)
    h2d = sum(pin[k].numel() * pin[k].element_size() for k in names)
    outs_host = []

    def e2e_run(nsteps, t_start=None, t_end=None):
        in_done, cmp_done = [None] * nsteps, [None] * nsteps

        def copy_in(i):
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(cmp_done[i - 2])  # step i-2 has finished reading this buffer set
                for k in names:
                    bufs[i % 2][k].copy_(pin[k], non_blocking=True)
                in_done[i] = torch.cuda.Event()
                in_done[i].record(s_in)

        if t_start is not None:
            t_start.record(s_in)
        copy_in(0)
        nbytes = 0
        for i in range(nsteps):
            if i + 1 < nsteps:
                copy_in(i + 1)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(in_done[i])
                t = {k: bufs[i % 2][k].detach().requires_grad_(backward and k in leaves) for k in names}
                out, ls = scan_step(t)
                res = [out.detach()] + ([ls] if ls is not None else [])
                names_out = ["out"] + (["last_state"] if ls is not None else [])
                if backward:
                    res += [t[k].grad for k in leaves]
                    names_out += ["d" + k for k in leaves]
                cmp_done[i] = torch.cuda.Event()
                cmp_done[i].record(s_cmp)
            if not outs_host:
                outs_host.extend(torch.empty(r.shape, dtype=r.dtype, pin_memory=True) for r in res)
            # a sharded step's exchange runs on a stream of its own and only the copy-out of the
            # gradients it sums (a few hundred KB) waits for it there: the big results leave as soon
            # as the step is computed, so the ranks' copy / compute pipelines are not put in lockstep
            summed = [j for j, nm in enumerate(names_out) if exchange and nm in ("dA", "dD", "ddelta_bias")]
            if summed:
                with torch.cuda.stream(s_x):
                    s_x.wait_event(cmp_done[i])
                    for j in summed:
                        res[j].record_stream(s_x)
                    reduce_grads(t)
                    for j in summed:
                        outs_host[j].copy_(res[j], non_blocking=True)
            with torch.cuda.stream(s_out):
                s_out.wait_event(cmp_done[i])
                for j, (hbuf, r) in enumerate(zip(outs_host, res)):
                    if j not in summed:
                        hbuf.copy_(r, non_blocking=True)
                        r.record_stream(s_out)  # allocated on the compute stream, read here
            nbytes = sum(r.numel() * r.element_size() for r in res)
        if t_end is not None:
            if s_x is not None:
                s_out.wait_stream(s_x)  # the last exchange and its copy-out are inside the region
            t_end.record(s_out)  # s_out's last copy waited on the last compute, which waited on its inputs
        return nbytes

    e2e_run(2)  # warm-up: pinned output buffers, stream pools
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    # three timed runs of E steps each; the median run per rank (the host side of a shared
    # machine adds stalls now and then), then the max over ranks
    runs = []
    for _ in range(3):
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        with quiet_host():
            d2h = e2e_run(E, s0, s1)
            torch.cuda.synchronize()
        runs.append(s0.elapsed_time(s1) / E)
    e2e_ms = statistics.median(runs)
    if world > 1:
        tt = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    e2e_value = tokens_job / (e2e_ms / 1e3)

    # ---- shard verification (N > 1, outside every timed region): the shards are NCCL
    # all-gathered and each one's sampled rows are checked against the CPU oracle on its owner
    verification = None
    if world > 1:
        verification = verify_shards(x, host, shape, rank, world, dev, step, backward)
        dist.destroy_process_group()
    if rank != 0:
        return 0
    link = host_link(dev, pin, bufs[0], names, outs_host, s_in, s_out, e2e_ms, ms_step)
    per_step, why = count_own_launches(lambda: (scan_step(x), clear(x)))  # the group is gone by now
    launches_src = "torch profiler, one untimed step"
    if not per_step:
        per_step, launches_src = launches_per_step(d, n, backward), f"model (profiler: {why or 'no kernels seen'})"

    fwd_bytes, bwd_bytes = algorithmic_bytes(b, d, L, n, ES[shape["dtype"]], with_z, last)
    if not backward:
        bwd_bytes = 0
    peak, peak_kind = load_peaks()
    dom_ms, dom_bytes, dom = (bwd_ms, bwd_bytes, "ss_bwd_kernel") if bwd_ms >= fwd_ms else (fwd_ms, fwd_bytes, "ss_fwd_kernel")
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    step_gbs = (fwd_bytes + bwd_bytes) / (ms_step / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": a.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": shape["scaling"], "vs_baseline": None,
        "dtype": shape["dtype"], "data": "synthetic", "config": config_dict(world, shape),
        "hbm_gbs_step": step_gbs, "hbm_frac_step": step_gbs / peak, "hbm_frac_step_nominal_8tbs": step_gbs / 8000.0,
        "kernels_ms": {"fwd": fwd_ms, "bwd": bwd_ms},
        "roofline": {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_kind,
                     "algorithmic_bytes_per_launch": dom_bytes,
                     "traffic": profile_traffic(a.workload, dom)},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "pipeline": ("copy-in, compute and copy-out of consecutive steps on three streams"
                             + (", the gradient exchange on a fourth" if exchange else "")),
                "ms_per_step": e2e_ms, "runs_ms_per_step": runs, "steps_per_run": E, "host_link": link},
        "exchange": (None if not exchange else
                     {"collective": "NCCL all_reduce (sum) of dA / dD / ddelta_bias, once per step",
                      "bytes_per_step": 4 * d * (n + 2), "in_place_over_one_span": one_span}),
        "gpu_launches": per_step * K, "gpu_launches_per_step": per_step, "gpu_launches_source": launches_src,
        "clocks": clk.summary(),
    }
    line["compute"] = compute_floor(b, d, L, n, ms_step, line["clocks"].get("sm_mhz"), with_z, backward,
                                    ES[shape["dtype"]])
    if verification is not None:
        line["verification"] = verification
    if world == 1 and not a.no_reference_ext:
        try:
            line["reference_ext"] = reference_ext_compare(shape, dev, backward)
        except Exception as e:  # a reported comparison, never required
            line["reference_ext"] = {"unavailable": repr(e)}
    if world == 1 and not a.no_cpu_baseline:
        try:
            v, thr, sample, _ = cpu_sample_rate(b * d * L, b * L, a.cpu_seconds, shape=shape)
            line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": thr, "kind": "port", "sample": sample}
        except Exception as e:  # the baseline is reported, never required
            line["cpu_baseline"] = {"value": None, "unit": "tokens/s", "cores": None, "kind": "port",
                                    "sample": f"failed: {e!r}"}
    print(json.dumps(line), flush=True)
    return 0

if __name__ == "__main__":
    sys.exit(main())
