"""Benchmark of the B200 DeepSeek-V3 FP8 block-scale MoE layer.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (expert parallelism, one rank per GPU)

Workload (every N): the expert-parallel full layer of the benchmark configs -- T=4096
tokens, all 256 DeepSeek-V3 experts sharded 256/N per GPU through local_expert_offset,
hidden states / logits replicated on every rank, the bf16 partial outputs combined by an
NCCL reduce-scatter (rows T/N per rank).  At N=1 one GPU holds all 256 experts.  The
total work is fixed as N grows ("scaling": "strong").  A step is one layer call plus the
reduce-scatter; `value` is whole-job tokens/s = T / step time (max over ranks).

At N=1 the line also carries the single-GPU sweeps with 32 local experts: decode
T in {1,7,16,32,64,80} (HBM-bound), mid-batch T=901 with skewed routing, and prefill
T in {8192,16384} (tensor-bound), each timed per call after an L2 flush.

The timed steps are plain layer calls (moe_swarm_b200.run, or the peer-memory EP layer); the
per-stage split and the dominant kernel's launch time come from a separate loop of the same calls
with CUDA events between the stages.  The line also carries the skewed-load variant of the
workload (per-expert logit bias N(0, 0.5)).

Inputs are synthetic (seeded, distributions of the benchmark configs); weights are
random-init on the device.  The CPU baseline (`cpu_baseline`, and each sweep record's) and
`--impl reference` time the oracle port of the reference's PyTorch kernel
(reference/kernel_pytorch_v1.py) on the host cores with all threads, on the whole workload: the
256-expert layer as 8 reference calls of 32 local experts (offsets 0..224), measured, not
extrapolated.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = ("MoE-layer latency (µs) & tokens/s vs T; HBM/FP8-tensor roofline fraction; "
          "EP 1/2/4/8")
H, I, E_GLOBAL = 7168, 2048, 256
W13_BYTES = 2 * I * H          # fp8 bytes of one expert's gate/up weights
W2_BYTES = H * I
S13_BYTES = 32 * 56 * 4
S2_BYTES = 56 * 16 * 4
FLOP_PER_ASSIGN = 2 * (H * 2 * I) + 2 * (I * H)   # 88,080,384 (GEMM1 + GEMM2)
EP_T = 4096
STREAM_MAX_T = 512             # T at or below which the layer runs the swap-AB streaming kernels


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


# ----------------------------------------------------------------------------- clocks
class _SmiSampler:
    """nvidia-smi clock/throttle samples (read-only queries): the fallback when NVML is absent."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self, gpus):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                idx = int(f[0])
                if gpus is not None and idx not in gpus:
                    continue
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() in ("active", "1"):
                    reasons.add(n)
        if not sm:
            return None
        sm.sort()
        loaded = [s for s in sm if s > 0.5 * mx] or sm
        return {"sm_mhz": loaded[len(loaded) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi"}


class ClockSampler:
    """SM clock and clock-event reasons of this process's GPU during the timed region.

    A thread reads them through NVML every 10 ms (read-only queries) from start() to stop();
    the report keeps the samples taken between the host timestamps mark_begin() / mark_end()
    placed around the timed steps (the GPU runs them in that interval), so even a timed region
    of a few tens of milliseconds carries several samples.  Falls back to nvidia-smi when NVML
    is not available."""
    REASONS = ((0x4, "sw_power_cap"), (0x8, "hw_slowdown"), (0x20, "sw_thermal_slowdown"),
               (0x40, "hw_thermal_slowdown"), (0x80, "hw_power_brake_slowdown"))

    def __init__(self, device):
        self.samples = []
        self.t0 = self.t1 = None
        self.halt = threading.Event()
        self.thread = None
        self.smi = None
        try:
            import pynvml
            pynvml.nvmlInit()
            p = torch.cuda.get_device_properties(device)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            self.nv = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
            self.reasons_of = (getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None)
                               or pynvml.nvmlDeviceGetCurrentClocksThrottleReasons)
        except Exception:
            self.handle = None
            self.smi = _SmiSampler()

    def _run(self):
        while not self.halt.is_set():
            try:
                mhz = float(self.nv.nvmlDeviceGetClockInfo(self.handle, self.nv.NVML_CLOCK_SM))
                bits = int(self.reasons_of(self.handle))
                self.samples.append((time.perf_counter(), mhz, bits))
            except Exception:
                pass
            self.halt.wait(0.01)

    def start(self):
        if self.smi is not None:
            self.smi.start()
            return
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def mark_begin(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()

    def stop(self, gpus=None):
        if self.smi is not None:
            return self.smi.stop(gpus)
        self.halt.set()
        if self.thread is not None:
            self.thread.join(timeout=2)
        inside = [s for s in self.samples
                  if self.t0 is not None and self.t1 is not None and self.t0 <= s[0] <= self.t1]
        if not inside:
            return None
        sm = sorted(s[1] for s in inside)
        reasons = sorted({name for s in inside for bit, name in self.REASONS if s[2] & bit})
        bits = 0
        for s in inside:
            bits |= s[2]
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "sm_mhz_range": [sm[0], sm[-1]], "reason_bits": hex(bits),
                "samples": len(inside), "source": "nvml, 10 ms"}


# ----------------------------------------------------------------------------- workload
def ep_inputs(rank, world, device, seed=0):
    import moe_swarm_b200.workload as W
    E_local = E_GLOBAL // world
    act = W.make_activations(EP_T, seed)
    x = {k: v.to(device) for k, v in act.items()}
    x.update(W.make_weights_fast(E_local, seed * 1000 + rank, device=device))
    x["local_expert_offset"] = rank * E_local
    x["routed_scaling_factor"] = 2.5
    return x, act


def routing_facts(x):
    """Exact active experts / rows of this rank from the device routing (outside timing)."""
    import moe_swarm_b200 as M
    r = M.route(**x)
    counts = r["e_count"].cpu()
    T = x["routing_logits"].shape[0]
    return {"active": int((counts > 0).sum()), "rows": int(counts.sum()), "T": T,
            "e_count": counts}


def gemm_bytes(f):
    """Algorithmic HBM bytes per launch of each GEMM (each weight byte and each activation
    byte once; outputs once)."""
    a, R, T = f["active"], f["rows"], f["T"]
    g1 = a * (W13_BYTES + S13_BYTES) + R * (H + 56 * 4) + R * (2 * I + 16 * 4)
    g2 = a * (W2_BYTES + S2_BYTES) + R * (2 * I + 16 * 4) + T * H * 2
    return g1, g2


# ----------------------------------------------------------------------------- timers
class StageTimer:
    def __init__(self):
        from moe_swarm_b200 import _native as N
        self.N = N
        self.lib = N.lib()
        self.h = self.lib.moe_b200_timer_create()

    def run(self, x, out=None):
        """moe_swarm_b200.run with per-stage events (same launches, same stream)."""
        import moe_swarm_b200 as M
        T, E, dev = M._validate(x["routing_logits"], x["routing_bias"], x["hidden_states"],
                                x["hidden_states_scale"], x["gemm1_weights"], x["gemm1_weights_scale"],
                                x["gemm2_weights"], x["gemm2_weights_scale"])
        if out is None:
            out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        buf = M._workspace(dev, stream).get(T, E, stream)
        a = M._args(T, E, x["routing_logits"], x["routing_bias"], x["hidden_states"],
                    x["hidden_states_scale"], x["gemm1_weights"], x["gemm1_weights_scale"],
                    x["gemm2_weights"], x["gemm2_weights_scale"], x["local_expert_offset"],
                    x["routed_scaling_factor"], out)
        rc = self.lib.moe_b200_forward_timed(ctypes.byref(a), buf.data_ptr(), buf.numel(), stream, self.h)
        if rc != 0:
            raise RuntimeError(f"moe_b200_forward_timed failed: {self.N.last_error()}")
        return out

    def read(self, reset=True):
        ms = (ctypes.c_float * 3)()
        calls = ctypes.c_int32()
        rc = self.lib.moe_b200_timer_read(self.h, ms, ctypes.byref(calls), 1 if reset else 0)
        if rc != 0:
            raise RuntimeError(self.N.last_error())
        return [float(v) for v in ms], int(calls.value)


# ----------------------------------------------------------------------------- CPU baseline
SLICE_E = 32   # the reference's layer holds 32 local experts (spec/reference_official.py:44)


def slice_weights_cpu(dev_weights, E=SLICE_E):
    """Host copies of the first E experts of a device weight set: the operands of the CPU
    reference calls.  The reference's work depends on the routed rows, not on the weight values,
    so one 32-expert slice serves every offset."""
    return {k: dev_weights[k][:E].cpu() for k in ("gemm1_weights", "gemm1_weights_scale", "gemm2_weights",
                                                  "gemm2_weights_scale")}


def cpu_ep_layer(act_cpu, w_cpu):
    """One full EP workload on the host cores, measured (not extrapolated): the 256-expert layer as
    the reference computes it, 8 calls of the oracle port of reference/kernel_pytorch_v1.kernel with
    32 local experts each, at local_expert_offset 0, 32, ..., 224 (the reference's own EP convention,
    reference/kernel_pytorch_v1.py:126-130); returns the summed seconds."""
    from oracle import moe_ref as O
    x = dict(act_cpu)
    x.update(w_cpu)
    x["routed_scaling_factor"] = 2.5
    t0 = time.perf_counter()
    for off in range(0, E_GLOBAL, SLICE_E):
        x["local_expert_offset"] = off
        O.run_v1(**x)
    return time.perf_counter() - t0


def cpu_baseline_ep(act_cpu, w_cpu, steps=1):
    """The EP workload timed on the host cores with all threads: one warm-up slice call, then
    `steps` whole layers (8 slice calls each); the median layer time."""
    from oracle import moe_ref as O
    torch.set_num_threads(os.cpu_count() or 1)
    T = act_cpu["routing_logits"].shape[0]
    x = dict(act_cpu)
    x.update(w_cpu)
    x["local_expert_offset"] = 0
    x["routed_scaling_factor"] = 2.5
    O.run_v1(**x)   # warm-up (one 32-expert slice)
    secs = sorted(cpu_ep_layer(act_cpu, w_cpu) for _ in range(steps))
    med = secs[len(secs) // 2]
    return {"value": T / med, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": (f"the whole workload, measured: oracle port of reference/kernel_pytorch_v1.kernel, "
                       f"8 calls of 32 local experts at offsets 0..224 (T={T}), median of {steps} layer(s): "
                       f"{med:.2f} s per layer; one 32-expert weight slice serves every offset"),
            "seconds_per_layer": med, "layers": steps}


def cpu_sweep_point(x_cpu, T):
    """One call each of the oracle ports of reference/kernel_pytorch_v1.kernel and, for T <= 901,
    spec/reference_official.run on the host cores, for a sweep configuration (seconds)."""
    from oracle import moe_ref as O
    torch.set_num_threads(os.cpu_count() or 1)
    t0 = time.perf_counter()
    O.run_v1(**x_cpu)
    v1 = time.perf_counter() - t0
    rec = {"v1_s": round(v1, 3), "v1_tokens_per_s": round(T / v1, 1), "cores": torch.get_num_threads(),
           "kind": "port"}
    if T <= 901:
        t0 = time.perf_counter()
        O.run(**x_cpu)
        rec["official_s"] = round(time.perf_counter() - t0, 3)
    return rec


# ----------------------------------------------------------------------------- sweeps (N=1)
def time_calls(M, x, n, flush):
    """Median device time (µs) of n layer calls, each after an L2 flush."""
    times = []
    for _ in range(n):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        M.run(**x)
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e) * 1e3)
    times.sort()
    return times[len(times) // 2]


def roofline_record(f, T, us, peaks_, fp8_peak):
    """Algorithmic bytes and FLOPs of one call from its routing, achieved rates, and the
    roofline verdict: the slower of moving the bytes at the measured copy bandwidth and doing the
    FLOPs at the fp8 peak is the speed-of-light time."""
    g1, g2 = gemm_bytes(f)
    byts = g1 + g2 + T * (256 * 4 + 56 * 4)
    flops = f["rows"] * FLOP_PER_ASSIGN
    t_hbm = byts / (peaks_["hbm_gbs"] * 1e9)
    t_fp8 = flops / (fp8_peak * 1e12)
    floor = max(t_hbm, t_fp8)
    return {"active_experts": f["active"], "rows": f["rows"], "us": round(us, 1),
            "tokens_per_s": round(T / (us * 1e-6), 1),
            "hbm_gbs": round(byts / (us * 1e-6) / 1e9, 1),
            "hbm_frac": round(byts / (us * 1e-6) / 1e9 / peaks_["hbm_gbs"], 3),
            "tflops": round(flops / (us * 1e-6) / 1e12, 1),
            "fp8_frac": round(flops / (us * 1e-6) / 1e12 / fp8_peak, 3),
            "bound": "hbm" if t_hbm >= t_fp8 else "tensor",
            "floor_us": round(floor * 1e6, 1),
            "sol_frac": round(floor / (us * 1e-6), 3)}


FP8_PEAK_SOURCE = "2x the measured cuBLAS bf16 burst peak (no measured fp8 peak)"


def sweep(device, steps, peaks_, cpu=True):
    import moe_swarm_b200 as M
    import moe_swarm_b200.workload as W
    out = []
    weights = W.make_weights_fast(32, 7, device=device)
    w_cpu = slice_weights_cpu(weights) if cpu else None
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    timer = StageTimer()
    fp8_peak = 2.0 * peaks_["bf16_tflops"]
    for name, T, skew in [("decode", 1, 0.0), ("decode", 7, 0.0), ("decode", 16, 0.0), ("decode", 32, 0.0),
                          ("decode", 64, 0.0), ("decode", 80, 0.0), ("mid_skewed", 901, 0.5),
                          ("prefill", 8192, 0.0), ("prefill", 16384, 0.0)]:
        act = W.make_activations(T, 1000 + T if T != 1 else 1000, skew=skew)   # T=1: seed 1000 routes one local expert
        x = {k: v.to(device) for k, v in act.items()}
        x.update(weights)
        x["local_expert_offset"] = 0
        x["routed_scaling_factor"] = 2.5
        f = routing_facts(x)
        for _ in range(3):
            M.run(**x)
        n = max(5, min(steps, 30)) if T <= 1024 else max(3, min(steps, 10))
        us = time_calls(M, x, n, flush)
        # the per-stage split comes from separate calls: events between the kernels break their
        # programmatic-launch overlap, so those calls are slower than the timed ones
        timer.read(reset=True)
        for _ in range(min(n, 5)):
            flush.zero_()
            timer.run(x)
        torch.cuda.synchronize()
        stage_ms, calls = timer.read(reset=True)
        rec = {"workload": name, "T": T}
        rec.update(roofline_record(f, T, us, peaks_, fp8_peak))
        if T <= 1024:
            # the same call replayed from a CUDA graph (fixed shape: the serving decode mode)
            g = M.GraphRunner(**x)
            for _ in range(3):
                g.replay()
            gt = []
            for _ in range(n):
                flush.zero_()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                g.replay()
                e.record()
                e.synchronize()
                gt.append(s.elapsed_time(e) * 1e3)
            gt.sort()
            rec["graph_us"] = round(gt[len(gt) // 2], 1)
            del g
        rec["stage_us"] = {k: round(v * 1e3 / calls, 1) for k, v in zip(("route", "gemm1", "gemm2"), stage_ms)}
        if w_cpu is not None:
            xc = dict(act)
            xc.update(w_cpu)
            xc["local_expert_offset"] = 0
            xc["routed_scaling_factor"] = 2.5
            rec["cpu_baseline"] = cpu_sweep_point(xc, T)
        out.append(rec)
        del x
    return out, {"fp8_peak_tflops": fp8_peak, "fp8_peak_source": FP8_PEAK_SOURCE}


def replay(args):
    """--workloads: one JSON line per workload of a flashinfer-bench workload file, timed like
    the sweeps (median of L2-flushed calls) with the roofline verdict.  Random inputs come from
    the package's seeded generators; one random-init weight set is shared by all workloads."""
    import moe_swarm_b200 as M
    from moe_swarm_b200 import replay as R
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    pk = peaks()
    fp8_peak = 2.0 * pk["bf16_tflops"]
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    weights = None
    for wl in R.load(args.workloads):
        x = R.materialize(wl, args.blob_root, seed=0, device=device, weights=weights)
        weights = {k: x[k] for k in R.WEIGHTS}
        f = routing_facts(x)
        for _ in range(3):
            M.run(**x)
        us = time_calls(M, x, max(5, min(args.steps, 30)), flush)
        rec = {"metric": METRIC, "workload_uuid": wl.uuid, "T": wl.T, "local_expert_offset": wl.offset,
               "unit": "µs", "higher_is_better": False, "fp8_peak_source": FP8_PEAK_SOURCE}
        rec.update(roofline_record(f, wl.T, us, pk, fp8_peak))
        rec["status"] = M.device_status(device)
        print(json.dumps(rec), flush=True)


# ----------------------------------------------------------------------------- main
def profile_case(args):
    """A small fixed workload for ncu captures: the same layer calls as the bench, no timing."""
    import moe_swarm_b200 as M
    import moe_swarm_b200.workload as W
    T, E = (int(v) for v in args.case.split(":"))
    dev = torch.device("cuda", 0)
    x = {k: v.to(dev) for k, v in W.make_activations(T, 5).items()}
    x.update(W.make_weights_fast(E, 1, device=dev))
    x["local_expert_offset"] = 0
    x["routed_scaling_factor"] = 2.5
    for _ in range(args.warmup + args.steps):
        M.run(**x)
    torch.cuda.synchronize()
    status = M.device_status(dev)
    print(f"case T={T} E={E}: {args.warmup + args.steps} calls, device status {status}", flush=True)
    if status != 0:
        raise SystemExit(1)


def reference_arm(args, config):
    """--impl reference: the reference's own CPU implementation of the layer (the oracle port of
    reference/kernel_pytorch_v1.kernel; the reference is Python and cannot travel to the GPU box)
    timed on this box's host cores with all threads, on the same workload, metric and unit as the
    GPU arm.  A step is the whole T=4096, 256-expert layer: 8 reference calls of 32 local experts
    (the reference's layer size) at offsets 0..224.  If K such steps would take longer than about
    four minutes, a step is one of those calls instead, the offsets taken in turn, and the layer
    time is 8 x the median call; the line says which."""
    import moe_swarm_b200.workload as W
    from oracle import moe_ref as O
    torch.set_num_threads(os.cpu_count() or 1)
    act = W.make_activations(EP_T, 0)
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    w_cpu = slice_weights_cpu(W.make_weights_fast(SLICE_E, 0, device=dev))
    x = dict(act)
    x.update(w_cpu)
    x["routed_scaling_factor"] = 2.5
    x["local_expert_offset"] = 0
    t0 = time.perf_counter()
    O.run_v1(**x)                      # warm-up: one 32-expert call
    est_layer = 8 * (time.perf_counter() - t0)
    steps = max(1, args.steps)
    whole = steps * est_layer <= 240.0
    per_step = []
    for i in range(steps):
        if whole:
            per_step.append(cpu_ep_layer(act, w_cpu))
        else:
            x["local_expert_offset"] = SLICE_E * (i % 8)
            t0 = time.perf_counter()
            O.run_v1(**x)
            per_step.append(time.perf_counter() - t0)
    srt = sorted(per_step)
    med = srt[len(srt) // 2]
    layer_s = med if whole else 8 * med
    value = EP_T / layer_s
    sample = (f"oracle port of reference/kernel_pytorch_v1.kernel on {torch.get_num_threads()} threads; "
              + (f"each step the whole layer: 8 calls of 32 local experts at offsets 0..224, median "
                 f"{layer_s:.2f} s" if whole else
                 f"each step one call of 32 local experts, offsets 0..224 in turn; layer = 8 x median call "
                 f"= {layer_s:.2f} s"))
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": steps, "warmup": 1,
            "ms_per_step": round(med * 1e3, 1), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16 GEMMs, fp32 accumulate (CPU)",
            "data": "synthetic", "config": dict(config, step=("whole layer" if whole else "one 32-expert call")),
            "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": torch.get_num_threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-sweeps", action="store_true")
    ap.add_argument("--ep-combine", choices=["peer", "nccl"], default="peer",
                    help="N > 1: combine over peer memory inside the layer call (moe_b200_forward_ep), "
                         "or the layer followed by an NCCL reduce-scatter")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU reference baselines of the GPU arm")
    ap.add_argument("--workloads", default=None, metavar="FILE",
                    help="replay a flashinfer-bench workload file (jsonl): one JSON line per workload")
    ap.add_argument("--blob-root", default=None, help="directory the workload file's blob paths are relative to")
    ap.add_argument("--case", default=None, metavar="T:E",
                    help="profiling case: W + K untimed layer calls at T tokens with E local experts "
                         "(seeded inputs, weights generated on the device); prints a status line only")
    args = ap.parse_args()
    if args.case:
        return profile_case(args)
    if args.workloads:
        return replay(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    steps, warmup = args.steps, max(3, args.warmup)

    config = {"workload": "ep_full_layer_T4096 (benchmark config 4: 256 experts sharded 256/N per GPU)",
              "T": EP_T, "experts_total": E_GLOBAL, "experts_per_gpu": E_GLOBAL // world,
              "parallelism": f"ep{world}",
              "combine": ("none" if world == 1 else
                          "peer memory: epilogue stores into the owner's buffer over NVLink, rank-order fp32 sum "
                          "(moe_b200_forward_ep)" if args.ep_combine == "peer" else "nccl reduce_scatter bf16"),
              "l2": "inputs larger than L2 (>=1.4 GB of routed weights per GPU per step)"}

    if args.impl == "reference":
        if rank != 0:
            return
        return reference_arm(args, config)

    import moe_swarm_b200 as M
    from moe_swarm_b200 import _native as N
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    pk = peaks()

    x, act_cpu = ep_inputs(rank, world, device)
    f = routing_facts(x)
    T = EP_T
    shard = torch.empty((T // world, H), dtype=torch.bfloat16, device=device)
    timer = StageTimer()
    peer = world > 1 and args.ep_combine == "peer"
    layer = None
    if peer:
        from moe_swarm_b200 import ep as EP
        layer = EP.ExpertParallelMoE()

    def layer_args(inp):
        return (inp["routing_logits"], inp["routing_bias"], inp["hidden_states"], inp["hidden_states_scale"],
                inp["gemm1_weights"], inp["gemm1_weights_scale"], inp["gemm2_weights"],
                inp["gemm2_weights_scale"], inp["routed_scaling_factor"])

    def step(inp, use_timer=False):
        """One timed step: the product call (moe_swarm_b200.run, or the peer-memory EP layer), then
        the reduce-scatter when the combine is NCCL's."""
        if peer:
            return layer.forward(*layer_args(inp), combine="peer", out=shard)
        out = timer.run(inp) if use_timer else M.run(**inp)
        if world > 1:
            dist.reduce_scatter_tensor(shard, out)
            return shard
        return out

    if peer:
        # the peer buffers are created on the first call (collective); if this process cannot map
        # peer memory, every rank falls back to the NCCL reduce-scatter and the line says so
        try:
            step(x, False)
            ok = torch.ones(1, device=device)
        except Exception as exc:   # noqa: BLE001 -- reported in the line
            print(f"rank {rank}: peer-memory combine unavailable ({exc}); using the NCCL reduce-scatter",
                  file=sys.stderr, flush=True)
            ok = torch.zeros(1, device=device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if float(ok) < 1:
            peer = False
            config["combine"] = "nccl reduce_scatter bf16 (peer-memory combine unavailable on this box)"
    clocks = ClockSampler(device)
    if rank == 0:
        clocks.start()
    for _ in range(warmup):
        step(x, False)
    torch.cuda.synchronize()
    launches_per_step = N.lib().moe_b200_last_launch_count()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    timer.read(reset=True)
    clocks.mark_begin()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step(x)
    end.record()
    torch.cuda.synchronize()
    clocks.mark_end()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    status = M.device_status(device, T, E_GLOBAL // world)
    if status:
        raise RuntimeError(f"rank {rank}: device status {status:#x} after the timed steps (a bounded wait gave up)")
    # stage split and the dominant kernel's launch time: the same layer calls with CUDA events
    # between the stages on the launching stream, in their own loop (events between kernels break
    # the programmatic-launch overlap, so these calls are not the timed ones)
    timer.read(reset=True)
    for _ in range(steps):
        timer.run(x)
    torch.cuda.synchronize()
    stage_ms, calls = timer.read(reset=True)

    # the skewed-load variant of the workload (config 2's per-expert logit bias N(0, 0.5)): same
    # weights, activations from the skewed generator, timed like the main steps
    import moe_swarm_b200.workload as W
    xs = dict(x)
    xs.update({k: v.to(device) for k, v in W.make_activations(EP_T, 0, skew=0.5).items()})
    fs = routing_facts(xs)
    for _ in range(warmup):
        step(xs)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s3.record()
    for _ in range(steps):
        step(xs)
    e3.record()
    torch.cuda.synchronize()
    ts = torch.tensor([s3.elapsed_time(e3)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ts, op=dist.ReduceOp.MAX)
    skew_ms = float(ts[0]) / steps
    del xs
    visible = None
    ck = clocks.stop(visible) if rank == 0 else None
    t = torch.tensor([ms] + stage_ms, device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, stage_ms = float(t[0]), [float(v) for v in t[1:]]
    ms_per_step = ms / steps

    # e2e: host (pinned) activations -> device, layer, combine, result -> host.
    # Serial: each step's copies and layer back to back on one stream.  Pipelined (the
    # reported value): two buffer sets; step i+1's inputs upload on a copy stream while step i's
    # layer runs, and step i's result downloads on another while step i+1 runs -- every step's
    # bytes still cross PCIe inside the timed region, which runs from the first upload to the
    # last download.  With N > 1 ranks each rank uploads only its T/N tokens' activations and an
    # NCCL all-gather over NVLink assembles the replicated inputs on every rank (the broadcast
    # form of expert parallelism needs every token on every rank; 1/N of it crosses each host
    # link), in stream order before the layer.
    names = ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale")
    n_tok = T // world
    lo_t = rank * n_tok
    out_shape = tuple(shard.shape) if world > 1 else (T, H)
    d2h = out_shape[0] * out_shape[1] * 2
    NB = 2
    dev_in = [{k: torch.empty_like(x[k]) for k in names} for _ in range(NB)]
    xe = [dict(x, **dev_in[b]) for b in range(NB)]
    dev_out = [torch.empty(out_shape, dtype=torch.bfloat16, device=device) for _ in range(NB)]
    res_host = [torch.empty(out_shape, dtype=torch.bfloat16).pin_memory() for _ in range(NB)]
    cs = torch.cuda.current_stream(device)
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev = {n: [torch.cuda.Event() for _ in range(NB)] for n in ("in_ready", "in_free", "out_ready", "out_free")}
    used = [False] * NB
    gat_scale = [torch.empty((world, 56, n_tok), dtype=torch.float32, device=device) for _ in range(NB)]

    def input_plan(sharded):
        """Host tensors each rank uploads per step and the device buffers they land in: every
        rank's whole inputs ("full"), or (N > 1, "sharded") its own T/N tokens, replicated by an
        NCCL all-gather over NVLink in stream order before the layer."""
        if sharded:
            host = {"routing_logits": act_cpu["routing_logits"][lo_t:lo_t + n_tok],
                    "routing_bias": act_cpu["routing_bias"],
                    "hidden_states": act_cpu["hidden_states"][lo_t:lo_t + n_tok].view(torch.uint8),
                    "hidden_states_scale": act_cpu["hidden_states_scale"][:, lo_t:lo_t + n_tok]}
        else:
            host = {k: act_cpu[k] for k in names}
        host = {k: v.contiguous().pin_memory() for k, v in host.items()}
        up = [{k: torch.empty_like(v, device=device) for k, v in host.items()} for _ in range(NB)] if sharded else dev_in
        return host, up

    def assemble(b, up, sharded):
        if not sharded:
            return
        d, u = dev_in[b], up[b]
        dist.all_gather_into_tensor(d["routing_logits"], u["routing_logits"])
        dist.all_gather_into_tensor(d["hidden_states"].view(torch.uint8), u["hidden_states"])
        dist.all_gather_into_tensor(gat_scale[b], u["hidden_states_scale"])
        d["hidden_states_scale"].view(56, world, n_tok).copy_(gat_scale[b].permute(1, 0, 2))
        d["routing_bias"].copy_(u["routing_bias"])

    def layer_into(inp, dst):
        if peer:
            layer.forward(*layer_args(inp), combine="peer", out=dst)
        elif world > 1:
            dist.reduce_scatter_tensor(dst, M.run(**inp))
        else:
            M.run(**inp, out=dst)

    def e2e_serial_step(host, up, sharded):
        for k in host:
            up[0][k].copy_(host[k], non_blocking=True)
        assemble(0, up, sharded)
        layer_into(xe[0], dev_out[0])
        res_host[0].copy_(dev_out[0], non_blocking=True)

    def e2e_pipelined_step(i, host, up, sharded):
        b = i % NB
        with torch.cuda.stream(s_in):
            if used[b]:
                s_in.wait_event(ev["in_free"][b])     # step i-2's layer has read these inputs
            for k in host:
                up[b][k].copy_(host[k], non_blocking=True)
            ev["in_ready"][b].record(s_in)
        cs.wait_event(ev["in_ready"][b])
        if used[b]:
            cs.wait_event(ev["out_free"][b])          # step i-2's result has left for the host
        assemble(b, up, sharded)
        layer_into(xe[b], dev_out[b])
        ev["in_free"][b].record(cs)
        ev["out_ready"][b].record(cs)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev["out_ready"][b])
            res_host[b].copy_(dev_out[b], non_blocking=True)
            ev["out_free"][b].record(s_out)
        used[b] = True

    def timed(run_steps, first_stream):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(first_stream)
        cs.wait_stream(first_stream)
        run_steps()
        cs.wait_stream(s_out)
        e2.record(cs)
        torch.cuda.synchronize()
        te = torch.tensor([s2.elapsed_time(e2)], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        return float(te[0]) / steps

    host_full, up_full = input_plan(False)
    for _ in range(2):
        e2e_serial_step(host_full, up_full, False)
    e2e_serial_ms = timed(lambda: [e2e_serial_step(host_full, up_full, False) for _ in range(steps)], cs)
    e2e_modes = {}
    for sharded in ((False, True) if world > 1 else (False,)):
        host, up = input_plan(sharded)
        used[:] = [False] * NB
        for i in range(2):
            e2e_pipelined_step(i, host, up, sharded)
        e2e_modes["sharded" if sharded else "full"] = (
            timed(lambda: [e2e_pipelined_step(i, host, up, sharded) for i in range(steps)], s_in),
            sum(v.numel() * v.element_size() for v in host.values()))
        assert torch.equal(res_host[(steps - 1) % NB].view(torch.int16),
                           dev_out[(steps - 1) % NB].cpu().view(torch.int16))
    e2e_mode = min(e2e_modes, key=lambda m: e2e_modes[m][0])
    e2e_ms, h2d = e2e_modes[e2e_mode]

    sweeps = None
    cpu = None
    if world == 1 and rank == 0:
        if not args.no_sweeps:
            sweeps, sweep_meta = sweep(device, steps, pk, cpu=not args.no_cpu)
        if not args.no_cpu:
            cpu = cpu_baseline_ep(act_cpu, slice_weights_cpu(x), steps=1)

    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    g1, g2 = gemm_bytes(f)
    per_launch_ms = [v / steps for v in stage_ms]
    dom = 1 if per_launch_ms[1] >= per_launch_ms[2] else 2
    dom_bytes = g1 if dom == 1 else g2
    dom_ms = per_launch_ms[dom]
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        try:
            traffic = json.loads(tf.read_text()).get(f"ep{world}_gemm{dom}")
        except ValueError:
            traffic = None
    line = {
        "metric": METRIC,
        "value": round(T / (ms_per_step * 1e-3), 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp8 e4m3 x e4m3 -> fp32 (bf16 out)",
        "data": "synthetic (seeded activations; random-init weights on the device)",
        "config": config,
        "latency_us": round(ms_per_step * 1e3, 1),
        "stage_us": {k: round(v * 1e3, 1) for k, v in zip(("route", "gemm1", "gemm2"), per_launch_ms)},
        "routing": {"active_experts_rank0": f["active"], "rows_rank0": f["rows"]},
        "roofline": {"kernel": f"{'stream' if T <= STREAM_MAX_T else 'wide'}_kernel<{dom}>", "bound": "hbm",
                     "achieved": round(achieved, 1),
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 3),
                     "traffic": traffic, "algorithmic_bytes_per_launch": dom_bytes,
                     "peak_source": pk["source"] + " (MEASURED_PEAKS.json hbm_gbs, burst copy)"},
        "e2e": {"value": round(T / (e2e_ms * 1e-3), 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
                "mode": ("pipelined: 2 buffer sets, uploads and downloads on their own streams overlap "
                         "the neighbouring steps' layers; inputs: "
                         + ("each rank uploads its T/N tokens, an NCCL all-gather over NVLink replicates them"
                            if e2e_mode == "sharded" else "every rank uploads the whole step's inputs")),
                "by_input_mode": {m: {"value": round(T / (v[0] * 1e-3), 1), "h2d_bytes_per_step": v[1]}
                                  for m, v in e2e_modes.items()},
                "serial_value": round(T / (e2e_serial_ms * 1e-3), 1),
                "serial_ms_per_step": round(e2e_serial_ms, 4)},
        "skewed_variant": {"value": round(T / (skew_ms * 1e-3), 1), "unit": "tokens/s",
                           "ms_per_step": round(skew_ms, 4), "logit_skew": 0.5,
                           "routing": {"active_experts_rank0": fs["active"], "rows_rank0": fs["rows"],
                                       "max_rows_per_expert_rank0": int(fs["e_count"].max())}},
        "gpu_launches": launches_per_step * steps,
        "clocks": ck,
    }
    if cpu is not None:
        line["cpu_baseline"] = {k: (round(v, 3) if isinstance(v, float) else v) for k, v in cpu.items()
                                if k in ("value", "unit", "cores", "kind", "sample")}
    if sweeps is not None:
        line["sweeps"] = sweeps
        line["sweep_meta"] = sweep_meta
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
