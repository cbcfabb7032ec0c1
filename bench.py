#!/usr/bin/env python
"""Benchmark: embeddings/sec of the rembed encoder forward pass on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload bge-base-b256xL128] [--mode bf16|f16|int8_w|int8_full|fp32]
                    [--modes auto|none|m1,m2,...]

N > 1 runs under torchrun, one process per GPU.  Each rank embeds its own
batch of the workload (data parallel, no collective on the data path:
"scaling": "weak"); timing is the max over ranks of CUDA-event time.

One JSON line on rank 0:
  value     embeddings/s over all ranks, inputs resident in HBM
            (rg_forward_device), K steps bracketed by barrier + sync;
  e2e       the same through the public host API (rg_submit / rg_collect:
            host ids in, host embeddings out, copies inside the timed region);
  roofline  the dominant kernel (the tcgen05 GEMMs, 4 per layer), timed
            live with CUDA events around each launch in a second pass,
            against the burst bf16 peak when the timed region ran at the
            maximum SM clock (else the sustained one, burst beside it);
  parity    the timed batch's embeddings (last timed step) against the CPU
            oracle on its first sequences, with the mode's bar;
  cpu_baseline  the CPU restatement of the reference forward (oracle/) timed
            on those same sequences, all host cores;
  modes     the other numeric modes of the headline metric (f16, weight-only
            int8, full int8, strict fp32), each with its own value, e2e,
            roofline, parity and CPU baseline;
  clocks    NVML samples taken during the timed region.
``--impl reference`` times only the CPU path, on rank 0, as the reference
arm.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {
    # the headline: bge-base (BERT-base), 256 sequences x 128 tokens, CLS + L2
    "bge-base-b256xL128": dict(preset="bge-base", nseq=256, lo=128, hi=128),
    "bge-base-b256xU16-512": dict(preset="bge-base", nseq=256, lo=16, hi=512),
    "minilm-l6-b32xU8-128": dict(preset="minilm-l6", nseq=32, lo=8, hi=128),
    # the other architectures' configurations (per GPU; EmbeddingGemma's
    # 512-sequence batch is sharded over 8 GPUs: 64 per GPU)
    "qwen3-0.6b-b128xU32-1024": dict(preset="qwen3-0.6b", nseq=128, lo=32, hi=1024),
    "modernbert-base-b64xU512-8192": dict(preset="modernbert-base", nseq=64, lo=512, hi=8192),
    "embeddinggemma-300m-b64xU16-2048": dict(preset="embeddinggemma-300m", nseq=64, lo=16, hi=2048),
    # the configuration's whole 512-sequence batch (for --scaling strong over 8 GPUs)
    "embeddinggemma-300m-b512xU16-2048": dict(preset="embeddinggemma-300m", nseq=512, lo=16, hi=2048),
    "modernbert-base-b64xU512-8192-strong": dict(preset="modernbert-base", nseq=64, lo=512, hi=8192),
}
METRIC = "embeddings/sec at bge-base b256×L128 (fp & int8), 1–8 GPU; tensor-pipe util %"
# mode -> (Embedder keyword arguments, oracle quantisation name, dtype the path computes in)
MODES = {
    "f16": ({"fp16": True}, "QUANT_NONE", "f16"),
    "bf16": ({"fp16": False}, "QUANT_NONE", "bf16"),
    "int8_w": ({"int8": True}, "QUANT_WEIGHTS", "s8 weights x f16"),
    "int8_full": ({"int8_activations": True}, "QUANT_FULL", "s8"),
    "fp32": ({"strict_fp32": True}, "QUANT_NONE", "f32 (3xTF32 projections)"),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="bge-base-b256xL128")
    ap.add_argument("--mode", choices=list(MODES), default="bf16")
    ap.add_argument("--modes", default="auto",
                    help="further modes measured after --mode, each in a sub-object of the line: a comma list, "
                         "'none', or 'auto' (every other mode on the headline workload, none elsewhere)")
    ap.add_argument("--mode-steps", type=int, default=20, help="timed steps of each further mode (at most --steps)")
    ap.add_argument("--ramp-seconds", type=float, default=0.0,
                    help="untimed forwards before the warm-up steps (clock ramp; 0 = none: the timed region then "
                         "runs at the clocks the warm-up leaves, before the power cap settles)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="target length of the CPU baseline sample")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="weak: one process per GPU under torchrun, each with its own batch; strong: one process, "
                         "one context over --gpus devices, one batch split across them by rg_forward")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def make_inputs(wl, seed, n=None):
    from rembed_b200 import synth

    cfg = synth.preset(wl["preset"])
    ids, cu = synth.make_batch(cfg, n or wl["nseq"], wl["lo"], wl["hi"], seed=seed)
    return cfg, ids, cu


ORACLE_PATH = {"f16": "fp32", "bf16": "fp32", "int8_w": "weight-int8", "int8_full": "full int8", "fp32": "fp32"}


def head(ids, cu, n):
    """The first n sequences of a packed batch."""
    return ids[: cu[n]], cu[: n + 1]


def cosines(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


PARITY_BARS = {"bf16": "cos >= 0.9999, max-abs <= 2e-3", "f16": "cos >= 0.9999, max-abs <= 2e-3",
               "fp32": "max-abs <= 1e-4", "int8_w": "cos >= 0.999 (vs the oracle's weight-int8 path)",
               "int8_full": "cos >= 0.998 (vs the oracle's full-int8 path)"}


def parity_ok(mode, cos_min, max_abs):
    if mode == "fp32":
        return max_abs <= 1e-4
    if mode == "int8_w":
        return cos_min >= 0.999
    if mode == "int8_full":
        return cos_min >= 0.998
    return cos_min >= 0.9999 and max_abs <= 2e-3


# ---------------------------------------------------------------------------
def oracle_on(wl, mode, ids, cu, nthreads):
    """The oracle (CPU restatement of the reference forward, in the mode's
    path) on a packed batch, one serial forward per sequence across nthreads
    threads as the reference's Embed fans out (rembed.go:309-331): (outputs,
    seconds)."""
    import oracle
    from rembed_b200 import synth

    cfg = synth.preset(wl["preset"])
    w = synth.make_weights(cfg, seed=0)
    m = oracle.OracleModel(cfg, w, getattr(oracle, MODES[mode][1]))
    t0 = time.perf_counter()
    out = m.embed(ids, cu, nthreads=nthreads)
    dt = time.perf_counter() - t0
    m.close()
    return out, dt


def cpu_and_parity(wl, mode, ids, cu, got, target_s, nthreads, timed=True):
    """Time the oracle on the first n sequences of the timed batch (n sized for
    about target_s seconds of CPU work, at least 2 per thread) and compare the
    GPU's embeddings of the same sequences with its outputs."""
    nseq = len(cu) - 1
    n0 = min(nseq, nthreads)
    _, t1 = oracle_on(wl, mode, *head(ids, cu, n0), nthreads)  # calibration
    per_seq = t1 / n0 * nthreads  # seconds of one thread per sequence
    n = int(max(min(nseq, 2 * nthreads), min(nseq, target_s / max(per_seq / nthreads, 1e-6))))
    want, dt = oracle_on(wl, mode, *head(ids, cu, n), nthreads)
    g = got[:n]
    cos = cosines(g, want)
    err = float(np.abs(g.astype(np.float64) - want).max())
    par = {"n": n, "mode": mode, "min_cos": round(float(cos.min()), 7), "max_abs": float(f"{err:.3g}"),
           "bar": PARITY_BARS[mode], "ok": bool(parity_ok(mode, float(cos.min()), err)),
           "against": f"oracle ({ORACLE_PATH[mode]} path) on the first {n} sequences of the timed batch"}
    cpu = {
        "value": round(n / dt, 3), "unit": "embeddings/s", "cores": nthreads, "kind": "port",
        "sample": f"the first {n} sequences of the timed {wl['preset']} batch (L in [{wl['lo']},{wl['hi']}]), one "
                  f"serial forward each across {nthreads} threads, {dt:.1f} s; C restatement of the reference "
                  f"({ORACLE_PATH[mode]} path), not the Go binary; CPU: {cpu_model()}",
    }
    return cpu, par


def reference_arm(args, rank, world):
    if rank != 0:
        return
    wl = WORKLOADS[args.workload]
    import oracle
    from rembed_b200 import synth

    nth = host_threads()
    cfg = synth.preset(wl["preset"])
    w = synth.make_weights(cfg, seed=0)
    quant = getattr(oracle, MODES[args.mode][1])
    m = oracle.OracleModel(cfg, w, quant)
    # every step embeds 4 sequences per thread (so that one slow thread does
    # not set the pace); fewer only if that would take more than ~4 minutes
    _, ids1, cu1 = make_inputs(wl, seed=1, n=nth)
    t0 = time.perf_counter()
    m.embed(ids1, cu1, nthreads=nth)
    t_one = time.perf_counter() - t0
    per_thread = 4
    while per_thread > 1 and t_one * per_thread * (args.steps + args.warmup) > 240.0:
        per_thread //= 2
    _, ids, cu = make_inputs(wl, seed=1, n=nth * per_thread)
    for _ in range(args.warmup):
        m.embed(ids, cu, nthreads=nth)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        m.embed(ids, cu, nthreads=nth)
    dt = time.perf_counter() - t0
    value = nth * per_thread * args.steps / dt
    path = {"QUANT_NONE": "fp32", "QUANT_WEIGHTS": "weight-int8", "QUANT_FULL": "full-int8"}[MODES[args.mode][1]]
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "embeddings/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * dt / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": {"QUANT_NONE": "f32", "QUANT_WEIGHTS": "s8 weights x f32",
                                       "QUANT_FULL": "u8 x s8"}[MODES[args.mode][1]], "data": "synthetic",
        "config": {"workload": args.workload, "global_batch": wl["nseq"], "seq_len": f"{wl['lo']}-{wl['hi']}",
                   "parallelism": "cpu threads", "mode": path,
                   "compared_with": f"our --mode {args.mode} arm (the reference computes this path in fp32)"},
        "cpu_baseline": {"value": round(value, 3), "unit": "embeddings/s", "cores": nth, "kind": "port",
                         "sample": f"each step embeds {nth * per_thread} sequences of the workload ({per_thread} "
                                   f"per thread), one serial forward per sequence; C restatement of the reference "
                                   f"forward ({path} path; Go is not installed on this image); CPU: {cpu_model()}"},
        "e2e": {"value": round(value, 3), "unit": "embeddings/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    m.close()
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
class NvmlClockSampler:
    """SM clock, power and clock-event reasons read through NVML every 2 ms
    by a background thread while the timed region runs (reads only)."""

    def __init__(self, uuid: str | None):
        import pynvml  # nvidia_ml_py
        self.nv = pynvml
        pynvml.nvmlInit()
        if uuid:
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        else:
            self.h = pynvml.nvmlDeviceGetHandleByIndex(0)
        self.rows = []
        self.stop = threading.Event()

    def _run(self):
        nv, h = self.nv, self.h
        while not self.stop.is_set():
            try:
                self.rows.append({"sm": float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                  "power": nv.nvmlDeviceGetPowerUsage(h) / 1000.0,
                                  "reasons": int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))})
            except nv.NVMLError:
                pass
            self.stop.wait(0.002)

    def __enter__(self):
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *exc):
        self.stop.set()
        self.thread.join(timeout=5)

    def summary(self):
        nv = self.nv
        try:
            mx = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
        except nv.NVMLError:
            mx = None
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": ["no samples"]}
        bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
        # the other event reasons, reported apart (a clock lock shows as
        # user_defined_clocks or applications_clocks_setting)
        other = {"gpu_idle": nv.nvmlClocksEventReasonGpuIdle,
                 "applications_clocks_setting": nv.nvmlClocksEventReasonApplicationsClocksSetting,
                 "sync_boost": nv.nvmlClocksEventReasonSyncBoost,
                 "hw_power_brake_slowdown": nv.nvmlClocksEventReasonHwPowerBrakeSlowdown,
                 "display_clock_setting": nv.nvmlClocksEventReasonDisplayClockSetting,
                 "user_defined_clocks": getattr(nv, "nvmlClocksEventReasonUserDefinedClocks", 0)}
        reasons = sorted({k for r in self.rows for k, b in bits.items() if r["reasons"] & b})
        others = sorted({k for r in self.rows for k, b in other.items() if b and r["reasons"] & b})
        sm = [r["sm"] for r in self.rows]
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": reasons, "other_reasons": others,
                "sm_mhz_range": [min(sm), max(sm)], "samples": len(self.rows),
                "source": "NVML every 2 ms during the timed region",
                "samples_with_a_reason": sum(1 for r in self.rows if r["reasons"] & sum(bits.values())),
                "power_w_max": round(max(r["power"] for r in self.rows), 1)}


def clock_sampler(uuid: str | None):
    """NVML sampler, or nvidia-smi when NVML cannot be loaded."""
    try:
        return NvmlClockSampler(uuid)
    except Exception:  # no pynvml / no NVML library: fall back to nvidia-smi
        return ClockSampler(uuid)


class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms during the timed region."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"rembed_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
            if self.uuid:
                cmd += ["-i", self.uuid]
            self.proc = subprocess.Popen(cmd, stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if not self.proc or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in self.path.read_text().splitlines():
            p = [x.strip() for x in line.split(",")]
            if len(p) < 10:
                continue
            try:
                rows.append({"sm": float(p[2]), "max": float(p[3]), "power": float(p[4]), "active": p[5],
                             "hw_slowdown": p[6], "hw_thermal_slowdown": p[7], "sw_thermal_slowdown": p[8],
                             "sw_power_cap": p[9]})
            except ValueError:
                continue
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        load = [r for r in rows if r["power"] > 200] or rows
        reasons = sorted({k for r in load for k in ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                                      "sw_power_cap") if r[k].lower() == "active"})
        return {"sm_mhz": float(np.median([r["sm"] for r in load])), "sm_max_mhz": max(r["max"] for r in rows),
                "reasons": reasons, "samples": len(rows), "samples_under_load": len(load),
                "power_w_max": max(r["power"] for r in rows)}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def committed_traffic(workload: str, mode: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary (profiles/traffic.json), or None."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(f"{workload}/{mode}")
    except (ValueError, OSError):
        return None


def peak_for(mode, peaks, clocks):
    """(peak TFLOP/s, which, the other fraction's peak or None) for a mode's
    GEMMs.  The burst cuBLAS figure applies when the timed region ran at the
    maximum SM clock (a short region, like a kernel timed alone); otherwise
    the sustained one, with the burst fraction reported beside it."""
    sm, mx = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
    at_max = bool(sm and mx and sm >= 0.97 * mx)
    burst, sust = peaks["bf16_tflops"], peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    # dense int8 runs at 2x the bf16 rate; 3xTF32 makes three passes at the
    # tf32 rate (half of bf16) for each fp32 product
    scale = {"int8_full": 2.0, "fp32": 1.0 / 6.0}.get(mode, 1.0)
    if at_max:
        return burst * scale, "burst", None
    return sust * scale, "sustained", burst * scale


class Measured:
    pass


def measure_mode(args, mode, wl, cfg, weights, ids, cu, world, local_rank, dist, primary):
    """value, e2e and the GEMM roofline of one numeric mode on this rank."""
    import torch

    from rembed_b200 import ranks
    from rembed_b200.embedder import Embedder

    emb = Embedder(cfg, weights, devices=[local_rank], **MODES[mode][0])
    nseq, T = len(cu) - 1, int(cu[-1])
    d_ids = torch.from_numpy(ids).cuda()
    d_cu = torch.from_numpy(cu).cuda()
    d_out = torch.empty((nseq, emb.dim), device="cuda", dtype=torch.float32)
    # A dedicated stream: the library launches every kernel of the forward on
    # it, so CUDA events recorded on it bracket exactly that work.
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    assert stream.cuda_stream != 0
    steps = args.steps if primary else max(3, min(args.steps, args.mode_steps))

    def step():
        emb.forward_device(d_ids.data_ptr(), d_cu.data_ptr(), cu, d_out.data_ptr(), stream=stream.cuda_stream)

    def barrier():
        ranks.barrier(dist)
        torch.cuda.synchronize()

    # optional clock ramp: the forward repeated for --ramp-seconds before the
    # warm-up steps, so that the (short) timed region runs at the clock the
    # workload settles to under the 1 kW power cap instead of the boost clock
    # the first steps see (measured on the headline: 0 s 37.5-38.0 K,
    # 0.25 s 36.2-36.6 K, 0.5 s 35.5-35.6 K embeddings/s)
    t_ramp = time.perf_counter()
    while time.perf_counter() - t_ramp < args.ramp_seconds:
        for _ in range(4):
            step()
        torch.cuda.synchronize()
    for _ in range(max(args.warmup, 1)):
        step()
    emb.sync()
    r = Measured()
    r.launches_per_step = emb.last_launches()

    # ---- value: device-resident inputs ----
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(local_rank).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        uuid = None
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with clock_sampler(uuid) as clk:
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    emb.sync()
    barrier()
    r.ms = ranks.max_over_ranks(dist, e0.elapsed_time(e1), device="cuda")
    r.clocks = clk.summary()
    r.steps = steps
    r.value = world * nseq * steps / (r.ms / 1000.0)
    r.out = d_out.cpu().numpy()  # the last timed step's embeddings (parity sample)

    # ---- e2e: host buffers through the public API ----
    # Every step stages its ids from host memory into pinned memory, copies
    # them to the device, runs the forward and copies the embeddings back to
    # a host array; steps are pipelined as a serving loop would run them
    # (rg_submit of step k+1 before rg_collect of step k).
    host_outs = [np.empty((nseq, emb.dim), dtype=np.float32) for _ in range(2)]

    def e2e_steps(n):
        pending = None
        for k in range(n):
            nxt = emb.submit(ids, cu, out=host_outs[k % 2])
            if pending is not None:
                pending.result()
            pending = nxt
        pending.result()

    e2e_steps(3)
    barrier()
    t0 = time.perf_counter()
    e2e_steps(steps)
    wall = time.perf_counter() - t0
    barrier()
    e2e_ms = ranks.max_over_ranks(dist, 1000.0 * wall, device="cuda")
    r.e2e = {"value": round(world * nseq * steps / (e2e_ms / 1000.0), 2), "unit": "embeddings/s",
             "h2d_bytes_per_step": int(ids.nbytes + cu.nbytes), "d2h_bytes_per_step": int(host_outs[0].nbytes + 4),
             "how": "rg_submit/rg_collect from host arrays, wall clock, two batches in flight"}

    # ---- roofline: per-kernel-class device time, second pass ----
    emb.profile(True)
    for _ in range(steps):
        step()
    stats = emb.profile_stats()
    emb.profile(False)
    peaks, peak_src = measured_peaks()
    g = stats["gemm"]
    total_ms = sum(v["ms"] for v in stats.values())
    peak, which, other = peak_for(mode, peaks, r.clocks)
    gemm_avg_ms = g["ms"] / max(g["launches"], 1)
    achieved = (g["flops"] / max(g["launches"], 1)) / (gemm_avg_ms / 1000.0) / 1e12
    unit_note = {"int8_full": "TOPS against 2x the bf16 peak (dense int8 rate)",
                 "fp32": "fp32-equivalent TFLOP/s against the bf16 peak / 6 (3xTF32: three tf32 passes, tf32 at "
                         "half the bf16 rate)"}.get(mode, "TFLOP/s against the bf16 peak (kind::f16 rate)")
    r.roofline = {
        "kernel": "tcgen05 GEMM (gemm_kernel), all dense projections",
        "bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
        "frac": round(achieved / peak, 4), "traffic": committed_traffic(args.workload, mode),
        "peak_source": f"{peak_src} {which} bf16 ({'median SM clock at max' if which == 'burst' else 'SM clock below max'}"
                       f"); {unit_note}",
        "algorithmic_per_launch": {"flops": g["flops"] / max(g["launches"], 1),
                                   "bytes": g["bytes"] / max(g["launches"], 1)},
        "avg_launch_ms": round(gemm_avg_ms, 4),
        "timing": "CUDA events around every launch on the library's stream in a second pass (per-launch events "
                  "break the programmatic-launch overlap, so this pass is slower than the timed one)",
        "share_of_forward": round(g["ms"] / total_ms, 4) if total_ms else None,
        "kernel_classes": {k: {"ms_per_step": round(v["ms"] / steps, 4),
                               "launches_per_step": v["launches"] // max(steps, 1),
                               "achieved_tflops": round(v["flops"] / (v["ms"] / 1000) / 1e12, 1) if v["ms"] else 0,
                               "achieved_gbs": round(v["bytes"] / (v["ms"] / 1000) / 1e9, 1) if v["ms"] else 0}
                           for k, v in stats.items() if v["launches"]},
    }
    if other:
        r.roofline["frac_of_burst"] = round(achieved / other, 4)
    pipe = committed_tensor_pipe(args.workload, mode)
    if pipe:
        r.roofline["tensor_pipe_pct_ncu"] = pipe
    r.gemm_tflops_effective = round(g["flops"] / max(steps, 1) / (r.ms / steps / 1000) / 1e12, 1)
    emb.close()
    torch.cuda.set_stream(torch.cuda.default_stream())
    return r


def committed_tensor_pipe(workload: str, mode: str):
    """ncu tensor-pipe utilisation per GEMM of one layer from the committed
    capture summary (profiles/traffic.json), or None."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(f"{workload}/{mode}/tensor_pipe_pct")
    except (ValueError, OSError):
        return None


def ours(args, rank, world, local_rank):
    import torch

    from rembed_b200 import ranks, synth

    torch.cuda.set_device(local_rank)
    dist = ranks.init(ranks.RankInfo(rank, world, local_rank), "nccl", device=torch.device("cuda", local_rank))
    wl = WORKLOADS[args.workload]
    cfg = synth.preset(wl["preset"])
    weights = synth.make_weights(cfg, seed=0)
    _, ids, cu = make_inputs(wl, seed=ranks.batch_seed(rank))
    nseq, T = len(cu) - 1, int(cu[-1])
    modes = args.modes
    if modes == "auto":
        modes = ",".join(MODES) if args.workload == "bge-base-b256xL128" else "none"
    extra = [m for m in (modes.split(",") if modes not in ("", "none") else []) if m != args.mode]
    for m in extra:
        if m not in MODES:
            raise SystemExit(f"unknown mode {m}")
    main_r = measure_mode(args, args.mode, wl, cfg, weights, ids, cu, world, local_rank, dist, primary=True)
    others = {m: measure_mode(args, m, wl, cfg, weights, ids, cu, world, local_rank, dist, primary=False)
              for m in extra}
    del weights
    line = {
        "metric": METRIC, "value": round(main_r.value, 2), "unit": "embeddings/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(main_r.ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": MODES[args.mode][2],
        "data": "synthetic (seeded random-init weights N(0,0.02) of the named architecture; seeded token ids)",
        "config": {"workload": args.workload, "global_batch": world * nseq, "per_gpu_batch": nseq,
                   "seq_len": f"{wl['lo']}-{wl['hi']}", "tokens_per_gpu_step": T, "parallelism": f"dp{world}",
                   "mode": args.mode,
                   "l2": "no flush: per-step working set (activations ~0.8 GB + weights) exceeds the 126 MB L2",
                   "clock_ramp_s": args.ramp_seconds},
        "roofline": main_r.roofline,
        "e2e": main_r.e2e,
        "clocks": main_r.clocks,
        "gpu_launches": int(main_r.launches_per_step * args.steps),
        "gemm_tflops_effective": main_r.gemm_tflops_effective,
    }
    if rank == 0 and not args.no_cpu_baseline:
        nth = host_threads()
        cpu, par = cpu_and_parity(wl, args.mode, ids, cu, main_r.out, args.cpu_seconds, nth)
        line["parity"] = par
        if world == 1:
            line["cpu_baseline"] = cpu
    if others:
        line["modes"] = {}
        for m, r in others.items():
            sub = {"value": round(r.value, 2), "unit": "embeddings/s", "ms_per_step": round(r.ms / r.steps, 4),
                   "steps": r.steps, "dtype": MODES[m][2], "e2e": r.e2e, "roofline": {
                       k: r.roofline[k] for k in ("achieved", "peak", "unit", "frac", "frac_of_burst", "peak_source",
                                                  "avg_launch_ms", "share_of_forward", "kernel_classes",
                                                  "traffic", "tensor_pipe_pct_ncu") if k in r.roofline},
                   "clocks": {k: r.clocks.get(k) for k in ("sm_mhz", "sm_max_mhz", "reasons")},
                   "gpu_launches": int(r.launches_per_step * r.steps)}
            if rank == 0 and not args.no_cpu_baseline:
                cpu, par = cpu_and_parity(wl, m, ids, cu, r.out, args.cpu_seconds / 4, host_threads())
                sub["parity"] = par
                if world == 1:
                    sub["cpu_baseline"] = cpu
            line["modes"][m] = sub
    ranks.finish(dist)
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    args = parse()
    from rembed_b200.ranks import rank_info

    info = rank_info()
    rank, world, local_rank = info.rank, info.world, info.local_rank
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return
    if args.scaling == "strong":
        if world != 1:
            raise SystemExit("--scaling strong runs as one process (no torchrun)")
        strong(args)
        return
    ours(args, rank, world, local_rank)


def strong(args):
    """One process, one context over --gpus devices: each step embeds the
    workload's whole batch through the public host API (rg_submit /
    rg_collect), which splits the sequences over the devices by estimated
    cost (longest first to the least loaded device) and writes every result
    into its row of the host output.  Host arrays in and out, so value and
    e2e are the same measurement here."""
    import torch

    from rembed_b200 import ranks, synth
    from rembed_b200.embedder import Embedder

    wl = WORKLOADS[args.workload]
    cfg = synth.preset(wl["preset"])
    weights = synth.make_weights(cfg, seed=0)
    _, ids, cu = make_inputs(wl, seed=ranks.batch_seed(0))
    nseq = len(cu) - 1
    devs = list(range(args.gpus))
    emb = Embedder(cfg, weights, devices=devs, **MODES[args.mode][0])
    del weights
    outs = [np.empty((nseq, emb.dim), dtype=np.float32) for _ in range(2)]

    def steps(n):
        pending = None
        for k in range(n):
            nxt = emb.submit(ids, cu, out=outs[k % 2])
            if pending is not None:
                pending.result()
            pending = nxt
        pending.result()

    t_ramp = time.perf_counter()
    while time.perf_counter() - t_ramp < args.ramp_seconds:
        steps(2)
    steps(max(args.warmup, 1))
    uuid = None
    with clock_sampler(uuid) as clk:
        t0 = time.perf_counter()
        steps(args.steps)
        wall = time.perf_counter() - t0
    for d in devs:
        torch.cuda.synchronize(d)
    value = nseq * args.steps / wall
    one = outs[(args.steps - 1) % 2].copy()
    emb.close()
    # the same batch on one device: the split must not change any embedding
    with Embedder(cfg, synth.make_weights(cfg, seed=0), devices=[0], **MODES[args.mode][0]) as e1:
        ref = e1.embed_packed(ids, cu)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "embeddings/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * wall / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": MODES[args.mode][2],
        "data": "synthetic (seeded random-init weights N(0,0.02) of the named architecture; seeded token ids)",
        "config": {"workload": args.workload, "global_batch": nseq, "seq_len": f"{wl['lo']}-{wl['hi']}",
                   "tokens_per_step": int(cu[-1]), "parallelism": f"one context over {args.gpus} GPUs, sequences "
                   f"split by estimated cost (longest first)", "mode": args.mode, "clock_ramp_s": args.ramp_seconds},
        "e2e": {"value": round(value, 2), "unit": "embeddings/s", "h2d_bytes_per_step": int(ids.nbytes + cu.nbytes),
                "d2h_bytes_per_step": int(outs[0].nbytes),
                "how": "rg_submit/rg_collect from host arrays, wall clock, two batches in flight"},
        "identical_to_one_gpu": bool(np.array_equal(one, ref)),
        "clocks_gpu0": clk.summary(),
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
