#!/usr/bin/env python
"""Benchmark of the selective-scan hot path (fused forward + VJP) on B200.

Workload (one "step"): the fused, gated selective scan forward and its VJP on
the largest point of the reference benchmark's op sweep: batch 64, L 4096,
d_inner 1536, d_state 16, fp32, seeded synthetic inputs with the sweep's
distributions.  Inputs (6.4 GB) are far larger than L2, so no flush is needed.

value : algorithmic GB/s of fwd+VJP (fwd_bytes / bwd_bytes below) over all
        ranks, inputs resident in HBM, kernels called through the C ABI,
        device-timed with CUDA events, max over ranks.
e2e   : the same metric through the public Python API (selective_scan_cuda +
        backward) with host-resident inputs: every step copies the inputs
        from pinned host memory and reads every output back.
N > 1 : one process per GPU; each rank scans its own batch shard (weak
        scaling, no collective on the data path).

`--impl reference` times the CPU oracle (the reference's sequential scan,
restated; MLX cannot run here) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "scan fwd+VJP HBM GB/s vs peak"
N_STATE = 16
WORKLOAD = dict(batch=64, seqlen=4096, d_inner=1536)
CPU_SAMPLE = dict(batch=1, seqlen=512, d_inner=1536)


def fwd_bytes(b, l, d, n=N_STATE, es=4):
    """read u, delta, z, B, C, A, D; write y (sequence tensors of es bytes an
    element, A and D fp32)."""
    return es * (4 * b * l * d + 2 * b * l * n) + 4 * (d * n + d)


def bwd_bytes(b, l, d, n=N_STATE, es=4):
    """read u, delta, z, dy, B, C, A, D; write du, ddelta, dz, dB, dC, dA, dD."""
    return es * (7 * b * l * d + 4 * b * l * n) + 4 * (2 * d * n + 2 * d)


# MUFU (exp2 / reciprocal) operations per (token, channel) of the gated scan:
# forward 16 decays exp(delta A) + 2 for the gate's sigmoid; VJP 16 decays in
# the recompute + 16 in the reverse pass + 2 for the gate.  The B200 SM
# retires 16 MUFU results per clock.
MUFU_PER_TD = {"fwd": 18, "bwd": 34}
MUFU_PER_SM_CLK = 16


def mufu_roofline(b, l, d, fwd_ms, bwd_ms, clk, sms=148):
    """Compute roofline of the scan kernels on the exp unit: MUFU operations
    per launch / time, against 16 results per SM per clock at the median SM
    clock sampled during the timed region (the scans are bound by it rather
    than by HBM)."""
    mhz = (clk or {}).get("sm_mhz") or 1965.0
    peak = MUFU_PER_SM_CLK * sms * mhz * 1e6 / 1e12  # T ops/s
    out = {"unit": "Tops/s", "peak": peak, "peak_source": f"16 per SM per clock x {sms} SMs x {mhz:.0f} MHz"}
    for name, ms in (("fwd", fwd_ms), ("bwd", bwd_ms)):
        ops = MUFU_PER_TD[name] * b * l * d
        out[name] = {"ops_per_launch": ops, "achieved": ops / (ms / 1e3) / 1e12,
                     "frac": ops / (ms / 1e3) / 1e12 / peak}
    return out


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of the
# dominant kernels on the bench workload, from the ncu capture summarised in
# profiles/scan_dram_traffic_b64_l4096_d1536.md (captured at L 512 on the same
# grid; every tensor grows in proportion to L, so scaled by 8).  A constant
# of this file, not read from the summary at run time.
NCU_TRAFFIC = {
    "vmscan_bwd": 13043200000,
    "scan_fwd_kernel": 7807500000,
}


def profiled_traffic(kernel):
    """Per-launch DRAM bytes of `kernel` on the default bench workload, or None
    for another workload (not captured)."""
    if (WORKLOAD["batch"], WORKLOAD["seqlen"], WORKLOAD["d_inner"]) != (64, 4096, 1536):
        return None
    return NCU_TRAFFIC.get(kernel)


def check_status(where):
    """Fail the run if a scan kernel gave up a bounded device wait (its outputs
    would be wrong): vmscan_device_status synchronises and clears the sticky
    status word."""
    import torch

    from mlx_vision_mamba_b200 import device_status

    st = device_status(torch.device("cuda", torch.cuda.current_device()), clear=True)
    if st != 0:
        raise RuntimeError(f"{where}: a device-side wait timed out (vmscan status {st}); result discarded")


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            cells = [c.strip() for c in line.split(",")]
            if len(cells) >= 9:
                rows.append(cells)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def make_inputs(b, l, d, device, seed):
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    f = dict(device=device, dtype=torch.float32)
    t = {
        "u": torch.randn(b, l, d, generator=g, **f),
        "z": torch.randn(b, l, d, generator=g, **f),
        "delta": torch.nn.functional.softplus(0.5 * torch.randn(b, l, d, generator=g, **f) - 3.0),
        "A": -torch.arange(1, N_STATE + 1, **f).repeat(d, 1),
        "B": torch.randn(b, l, N_STATE, generator=g, **f),
        "C": torch.randn(b, l, N_STATE, generator=g, **f),
        "D": torch.ones(d, **f),
        "dy": torch.randn(b, l, d, generator=g, **f),
    }
    return t


class AbiScan:
    """Preallocated fwd + VJP through the C ABI (no allocation in the timed loop).

    bf16=True casts the sequence tensors (u, delta, z, B, C, dy) to bf16 and
    calls vmscan_fwd_bf16 / vmscan_bwd_bf16 (A, D, dA, dD, checkpoints fp32)."""

    def __init__(self, t, bf16=False):
        import torch

        from mlx_vision_mamba_b200 import _native

        self.lib = lib = _native.load()
        if bf16:
            t = {k: (v.to(torch.bfloat16) if k not in ("A", "D") else v) for k, v in t.items()}
        # the fp32 entry points take one more pointer (y_lo / dz_lo: NULL = plain fp32 outputs)
        self.fwd_fn = lib.vmscan_fwd_bf16 if bf16 else (lambda *a: lib.vmscan_fwd(*a[:18], None, *a[18:]))
        self.bwd_fn = lib.vmscan_bwd_bf16 if bf16 else (lambda *a: lib.vmscan_bwd(*a[:31], None, *a[31:]))
        self.t = t
        b, l, d = t["u"].shape
        self.shape = (b, l, d)
        dev = t["u"].device
        sd = t["u"].dtype
        self.y = torch.empty_like(t["u"])
        self.ck = torch.empty(lib.vmscan_ckpt_elems(b, l, d, N_STATE, None), device=dev)
        self.g = {k: torch.empty_like(t["u"]) for k in ("du", "ddelta", "dz")}
        self.g["dA"] = torch.empty(d, N_STATE, device=dev)
        self.g["dB"] = torch.empty(b, l, N_STATE, device=dev, dtype=sd)
        self.g["dC"] = torch.empty(b, l, N_STATE, device=dev, dtype=sd)
        self.g["dD"] = torch.empty(d, device=dev)
        self.fws_n = lib.vmscan_fwd_workspace_bytes(b, l, d, N_STATE, None)
        self.fws = torch.empty(max(self.fws_n, 16), dtype=torch.uint8, device=dev)
        self.fws_ptr = self.fws.data_ptr() if self.fws_n > 0 else None
        self.ws_n = lib.vmscan_bwd_workspace_bytes(b, l, d, N_STATE, None, 0)
        self.ws = torch.empty(self.ws_n, dtype=torch.uint8, device=dev)

    def _S(self, x):
        from mlx_vision_mamba_b200 import _native

        return _native.Strides(x.stride(0), x.stride(1))

    def fwd(self, stream):
        t, S = self.t, self._S
        b, l, d = self.shape
        st = self.fwd_fn(b, l, d, N_STATE, t["u"].data_ptr(), S(t["u"]), t["delta"].data_ptr(),
                                 S(t["delta"]), t["A"].data_ptr(), t["B"].data_ptr(), S(t["B"]), t["C"].data_ptr(),
                                 S(t["C"]), t["D"].data_ptr(), t["z"].data_ptr(), S(t["z"]), self.y.data_ptr(),
                                 S(self.y), self.ck.data_ptr(), None, self.fws_ptr, self.fws_n, stream)
        if st:
            raise RuntimeError(f"vmscan_fwd: {self.lib.vmscan_strerror(st).decode()}")

    def bwd(self, stream):
        t, g, S = self.t, self.g, self._S
        b, l, d = self.shape
        st = self.bwd_fn(
            b, l, d, N_STATE, t["u"].data_ptr(), S(t["u"]), t["delta"].data_ptr(), S(t["delta"]),
            t["A"].data_ptr(), t["B"].data_ptr(), S(t["B"]), t["C"].data_ptr(), S(t["C"]), t["D"].data_ptr(),
            t["z"].data_ptr(), S(t["z"]), self.ck.data_ptr(), t["dy"].data_ptr(), S(t["dy"]),
            g["du"].data_ptr(), S(g["du"]), g["ddelta"].data_ptr(), S(g["ddelta"]), g["dA"].data_ptr(),
            g["dB"].data_ptr(), S(g["dB"]), g["dC"].data_ptr(), S(g["dC"]), g["dD"].data_ptr(),
            g["dz"].data_ptr(), S(g["dz"]), None, self.ws.data_ptr(), self.ws_n, stream)
        if st:
            raise RuntimeError(f"vmscan_bwd: {self.lib.vmscan_strerror(st).decode()}")


def cpu_oracle_step(sample, threads, seed=0, chunked=False):
    """One fwd+VJP of the oracle (the reference's sequential scan, or its
    chunked variant mamba_fast.py:17-75; torch CPU fp32)."""
    import torch

    from oracle import scan_ref

    torch.set_num_threads(threads)
    inp = scan_ref.sweep_inputs(sample["batch"], sample["seqlen"], sample["d_inner"], seed=seed)
    fn = scan_ref.selective_scan_chunked if chunked else scan_ref.selective_scan
    t0 = time.perf_counter()
    scan_ref.scan_vjp(inp, gated=True, dtype=torch.float32, scan_fn=fn)
    return time.perf_counter() - t0


def cpu_model() -> str:
    """The host CPU's model name (first "model name" line of /proc/cpuinfo)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline(steps=1, warmup=0, budget_s=20.0):
    """Both CPU restatements of the reference (sequential and chunked scan),
    each timed for about half the budget; the faster one is the baseline."""
    threads = os.cpu_count() or 1
    s = CPU_SAMPLE
    byt = fwd_bytes(s["batch"], s["seqlen"], s["d_inner"]) + bwd_bytes(s["batch"], s["seqlen"], s["d_inner"])
    res = {}
    for chunked in (False, True):
        for _ in range(max(warmup, 1)):  # the first call pays torch's thread-pool start-up
            cpu_oracle_step(s, threads, chunked=chunked)
        times = []
        t_start = time.perf_counter()
        while len(times) < max(steps, 1) or (time.perf_counter() - t_start < budget_s / 2 and len(times) < 50):
            times.append(cpu_oracle_step(s, threads, chunked=chunked))
            if time.perf_counter() - t_start > budget_s / 2 and len(times) >= steps:
                break
        res["chunked" if chunked else "sequential"] = (statistics.median(times), len(times))
    best = min(res, key=lambda k: res[k][0])
    per, n = res[best]
    return {
        "value": byt / per / 1e9,
        "unit": "GB/s",
        "cores": threads,
        "cpu_model": cpu_model(),
        "kind": "port",
        "sample": f"oracle {best} scan fwd+VJP (torch CPU fp32, {threads} threads) on batch "
                  f"{s['batch']} of the same workload (L {s['seqlen']}, d_inner {s['d_inner']}), "
                  f"median of {n} runs, {per:.2f} s each",
        "variants": {k: {"s_per_step": v[0], "gbs": byt / v[0] / 1e9, "runs": v[1]} for k, v in res.items()},
    }, per


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    base, per = cpu_baseline(steps=args.steps, warmup=args.warmup, budget_s=30.0)
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name(), **WORKLOAD, "d_state": N_STATE, "sample": CPU_SAMPLE},
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_name():
    w = WORKLOAD
    return (f"gated selective scan fwd+VJP, op-sweep point batch {w['batch']} L {w['seqlen']} "
            f"d_inner {w['d_inner']} d_state {N_STATE} (per GPU)")


def launch_only(reps, bf16):
    """REPS forward + VJP pairs through the C ABI on the sweep's seeded inputs,
    untimed: the launches a small `ncu` capture selects from.  Returns the
    process exit code (1 if a bounded device wait gave up)."""
    import torch

    dev = torch.device("cuda", 0)
    b, l, d = WORKLOAD["batch"], WORKLOAD["seqlen"], WORKLOAD["d_inner"]
    runner = AbiScan(make_inputs(b, l, d, dev, seed=3), bf16=bf16)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    for _ in range(reps):
        runner.fwd(stream)
        runner.bwd(stream)
    torch.cuda.synchronize()
    st = runner.lib.vmscan_device_status(stream, 1)
    print(json.dumps({"launch_only": {"batch": b, "seqlen": l, "d_inner": d, "io": "bf16" if bf16 else "f32",
                                      "reps": reps, "device_status": st}}), flush=True)
    return 1 if st else 0


def launch_only_gemm(reps, which):
    """REPS launches of one projection GEMM of the VisionMamba-2D block (64 x
    196 tokens, E 384, K=4) on split operands made once beforehand, untimed."""
    import torch

    from mlx_vision_mamba_b200 import device_status
    from mlx_vision_mamba_b200.linear import gemm_tf32x3, tf32_split

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(4)
    t = 64 * 196
    name, kind = which.rsplit("_", 1)
    fin, fout = (384, 6144) if name == "in_proj" else (3072, 384)
    x = tf32_split(torch.randn(t, fin, device=dev, generator=g))
    w = tf32_split(torch.randn(fout, fin, device=dev, generator=g) / fin ** 0.5)
    dy = tf32_split(torch.randn(t, fout, device=dev, generator=g))
    for _ in range(reps):
        if kind == "fwd":
            gemm_tf32x3(x, False, w, False, t, fout, fin)
        elif kind == "dx":
            gemm_tf32x3(dy, False, w, True, t, fin, fout)
        else:
            gemm_tf32x3(dy, True, x, True, fout, fin, t)
    st = device_status(dev, clear=True)
    print(json.dumps({"launch_only": {"gemm": which, "reps": reps, "device_status": st}}), flush=True)
    return 1 if st else 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-model", action="store_true", help="skip the VisionMamba-2D training measurement")
    ap.add_argument("--batch", type=int, default=WORKLOAD["batch"], help="per-GPU batch (profiling runs)")
    ap.add_argument("--seqlen", type=int, default=WORKLOAD["seqlen"])
    ap.add_argument("--dinner", type=int, default=WORKLOAD["d_inner"])
    ap.add_argument("--model-eager", action="store_true", help="run the model steps eagerly (no CUDA graph)")
    ap.add_argument("--encoder", choices=["3d", "4d"],
                    help="only time VisionMamba-3D (K=6, global batch 16) or -4D (K=8, global "
                         "batch 8) training and print one JSON line")
    ap.add_argument("--parallel", choices=["dp", "dirshard"], default="dp",
                    help="with --encoder: data parallel, or the scan directions split over the ranks")
    ap.add_argument("--sweep", action="store_true",
                    help="time forward and VJP separately on the 12 op-sweep points and print a table")
    ap.add_argument("--io", choices=["f32", "bf16"], default="f32",
                    help="with --sweep: sequence tensors in fp32 (the reference's dtype) or bf16")
    ap.add_argument("--conv", action="store_true",
                    help="only time the conv1d + SiLU kernels (forward, VJP) at the model's block shape")
    ap.add_argument("--dt", action="store_true",
                    help="only time the dt_proj + softplus kernels (forward, VJP) at the model's block shape")
    ap.add_argument("--model-profile", action="store_true",
                    help="print the per-kernel device-time table of one VisionMamba-2D training step and exit")
    ap.add_argument("--model-batch", type=int,
                    help="with --model-profile, or alone: images per VisionMamba-2D step on one GPU (e.g. 8 = one "
                         "GPU's share of the 8-GPU run); alone it prints only the model line")
    ap.add_argument("--gemm", action="store_true",
                    help="only time the tensor-core projection GEMMs at the VisionMamba-2D shapes against "
                         "PyTorch's fp32 GEMM")
    ap.add_argument("--launch-only", type=int, metavar="REPS",
                    help="run REPS forward + VJP pairs through the C ABI at --batch/--seqlen/--dinner (--io "
                         "picks fp32 or bf16 I/O), or with --launch-gemm REPS projection GEMMs, untimed, and exit "
                         "nonzero if the device status is set (small ncu captures)")
    ap.add_argument("--launch-gemm", choices=["in_proj_fwd", "in_proj_dx", "in_proj_dw", "out_proj_fwd",
                                              "out_proj_dx", "out_proj_dw"],
                    help="with --launch-only: the VisionMamba-2D projection GEMM to launch")
    args = ap.parse_args()
    WORKLOAD.update(batch=args.batch, seqlen=args.seqlen, d_inner=args.dinner)
    if args.impl == "reference":
        run_reference(args)
        return
    if args.launch_only:
        if args.launch_gemm:
            sys.exit(launch_only_gemm(args.launch_only, args.launch_gemm))
        sys.exit(launch_only(args.launch_only, args.io == "bf16"))
    if args.model_profile:
        profile_model(args.warmup, args.model_batch)
        return
    if args.model_batch:
        import torch

        line = run_model(torch.device("cuda", 0), 0, 1, steps=20, warmup=max(args.warmup, 3),
                         barrier=lambda: None, graphed=not args.model_eager, batch=args.model_batch)
        print(json.dumps({"vision_mamba_2d_train_batch": line}), flush=True)
        return
    if args.sweep:
        run_sweep(max(args.steps, 20), max(args.warmup, 3), bf16=args.io == "bf16")
        return
    if args.conv:
        import torch

        print(json.dumps({"conv1d_silu": time_conv(torch.device("cuda", 0))}), flush=True)
        return
    if args.dt:
        import torch

        print(json.dumps({"dt_softplus": time_dt(torch.device("cuda", 0))}), flush=True)
        return
    if args.gemm:
        import torch

        print(json.dumps({"projection_gemm": time_gemm(torch.device("cuda", 0))}), flush=True)
        return

    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        # collectives captured in a CUDA graph (the model step) cannot be polled
        # by NCCL's asynchronous error watchdog
        os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "0")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    args.warmup = max(args.warmup, 3)

    if args.encoder:
        barrier = (lambda: dist.barrier(device_ids=[local])) if world > 1 else (lambda: None)
        line = run_encoder(dev, rank, world, args.encoder, args.parallel, max(3, min(args.steps, 10)), args.warmup,
                           barrier)
        if rank == 0:
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    b, l, d = WORKLOAD["batch"], WORKLOAD["seqlen"], WORKLOAD["d_inner"]
    t = make_inputs(b, l, d, dev, seed=1234 + rank)
    runner = AbiScan(t)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        runner.fwd(stream)
        runner.bwd(stream)
    torch.cuda.synchronize()

    K = args.steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    e0.record()
    for i in range(K):
        ev[i][0].record()
        runner.fwd(stream)
        ev[i][1].record()
        runner.bwd(stream)
        ev[i][2].record()
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    check_status("timed fwd+VJP")
    barrier()
    total_ms = e0.elapsed_time(e1)
    fwd_ms = statistics.mean(ev[i][0].elapsed_time(ev[i][1]) for i in range(K))
    bwd_ms = statistics.mean(ev[i][1].elapsed_time(ev[i][2]) for i in range(K))
    tmax = torch.tensor([total_ms], device=dev)
    if world > 1:
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
    total_ms = float(tmax.item())

    fb, bb = fwd_bytes(b, l, d), bwd_bytes(b, l, d)
    value = world * K * (fb + bb) / (total_ms / 1e3) / 1e9
    peak, peak_kind = measured_peaks()
    bwd_gbs = bb / (bwd_ms / 1e3) / 1e9
    fwd_gbs = fb / (fwd_ms / 1e3) / 1e9

    # ---- the MambaBlock shape of the reference's only published scan numbers ----
    cfg1 = time_config1(dev, stream) if rank == 0 else None

    # ---- the direction-aware conv1d + SiLU kernels at the model's block shape ----
    conv = time_conv(dev) if rank == 0 else None
    dtk = time_dt(dev) if rank == 0 else None

    # ---- the same workload through the bf16 I/O entry points (not the metric) ----
    bf16_io = time_bf16_io(t, dev, stream, K, args.warmup) if rank == 0 else None

    # ---- end to end through the public API with host buffers ----
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(t, dev, K=max(2, min(K, 8)), warmup=2, world=world, barrier=barrier)
    del runner, t
    torch.cuda.empty_cache()

    # ---- VisionMamba-2D training throughput (second half of the metric) ----
    model_line = None
    model_scaling = None
    if not args.no_model:
        msteps = max(3, min(K, 10))
        model_line = run_model(dev, rank, world, steps=msteps, warmup=3, barrier=barrier,
                               graphed=not args.model_eager)
        one = model_line
        if world > 1:
            # the 1-GPU point of the same curve, in the same job: rank 0 trains
            # on the whole global batch alone while the other ranks wait
            one = run_model(dev, 0, 1, steps=msteps, warmup=3, barrier=None, graphed=not args.model_eager,
                            single=True) if rank == 0 else None
            barrier()
        if rank == 0:
            model_scaling = {
                "model": "VisionMamba-2D K=4 training (fwd, MSE, bwd, AdamW), global batch 64, strong scaling",
                "n_gpus": world, "img_per_s": model_line["img_per_s"], "ms_per_step": model_line["ms_per_step"],
                "per_gpu_batch": model_line["per_gpu_batch"],
                "one_gpu_img_per_s": one["img_per_s"], "one_gpu_ms_per_step": one["ms_per_step"],
                "speedup_vs_one_gpu": model_line["img_per_s"] / one["img_per_s"],
                "efficiency_vs_one_gpu": model_line["img_per_s"] / one["img_per_s"] / world,
                "one_gpu_source": "this run" if world == 1 else "this job, rank 0 alone on the whole batch",
            }

    base = None
    if rank == 0 and world == 1 and not args.no_cpu:
        base, _ = cpu_baseline(steps=1, warmup=0, budget_s=15.0)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "GB/s",
            "n_gpus": world,
            "steps": K,
            "warmup": args.warmup,
            "ms_per_step": total_ms / K,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic",
            "config": {
                "workload": workload_name(),
                "batch_per_gpu": b, "global_batch": b * world, "seq_len": l, "d_inner": d, "d_state": N_STATE,
                "gated": True, "parallelism": f"weak x{world} (independent batch shards, no collective)",
                "l2": f"inputs {4 * 4 * b * l * d / 1e9:.2f} GB per GPU vs 126 MB L2; no flush",
            },
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
            "fwd_gbs": fwd_gbs, "bwd_gbs": bwd_gbs,
            "roofline": {
                "kernel": "scan_bwd_kernel + reduce_dbc_kernel + reduce_dad_kernel (vmscan_bwd)",
                "bound": "hbm", "achieved": bwd_gbs, "peak": peak, "unit": "GB/s", "frac": bwd_gbs / peak,
                "peak_source": peak_kind, "traffic": profiled_traffic("vmscan_bwd"),
                "algorithmic_bytes_per_launch": bb,
                "fwd": {"kernel": "scan_fwd_kernel", "achieved": fwd_gbs, "frac": fwd_gbs / peak,
                        "algorithmic_bytes_per_launch": fb, "traffic": profiled_traffic("scan_fwd_kernel")},
                "fwd_plus_bwd_frac": value / world / peak,
                "mufu": mufu_roofline(b, l, d, fwd_ms, bwd_ms, clk,
                                      sms=torch.cuda.get_device_properties(dev).multi_processor_count),
            },
            "gpu_launches": 4 * K,
            "clocks": clk,
            "e2e": e2e,
            "config1_scan": cfg1,
            "bf16_io": bf16_io,
            "conv1d_silu": conv,
            "dt_softplus": dtk,
            "cpu_baseline": base,
            "vision_mamba_2d_train": model_line,
            "model_scaling": model_scaling,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_model(dev, rank, world, steps, warmup, barrier, graphed=True, single=False, batch=None):
    """VisionMamba-2D (K=4, 224x224x1, patch 16, E 384, depth 6) training steps:
    forward, MSE, backward (DDP all-reduce over NCCL when world > 1), AdamW.
    Global batch 64 split over the ranks (strong scaling), fp32 (TF32 off).
    `graphed`: the whole step is one CUDA graph replay (train.GraphedTrainStep).
    `single`: this rank alone trains on the whole global batch (the 1-GPU
    point of the strong-scaling curve, measured inside a multi-GPU job; no
    DDP, no collective, no barrier).  `batch` (single GPU only): images per
    step instead of the global batch, e.g. 8 to time one GPU's share of the
    8-GPU step without the all-reduce; img/s then counts those images."""
    import torch
    import torch.distributed as dist

    from mlx_vision_mamba_b200 import train

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    cfg = train.VISION_MAMBA_2D
    if single:
        rank, world, barrier = 0, 1, (lambda: None)
    a, b = train.shard(cfg.global_batch, rank, world)
    if batch is not None:
        assert world == 1 or single, "batch overrides apply to single-GPU runs"
        a, b = 0, int(batch)
    wrap = (lambda m: m) if single else (lambda m: train.wrap_data_parallel(m, dev))
    side = torch.cuda.Stream(dev)
    if graphed:
        with torch.cuda.stream(side):  # DDP is constructed on the capture's side stream
            model = wrap(train.build_encoder(cfg, dev, seed=0))
        torch.cuda.current_stream(dev).wait_stream(side)
    else:
        model = wrap(train.build_encoder(cfg, dev, seed=0))
    opt = train.make_optimizer(model, capturable=graphed)
    x, tgt = train.synthetic_batch(cfg, b - a, dev, seed=100 + rank)
    if graphed:
        gstep = train.GraphedTrainStep(model, opt, x, tgt, side_stream=side)
        step = lambda: gstep()  # noqa: E731
    else:
        gstep = None
        step = lambda: train.train_step(model, opt, x, tgt)  # noqa: E731
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        loss = step()
    e1.record()
    torch.cuda.synchronize()
    loss = float(loss.item())
    if gstep is not None:
        gstep.close()  # checks the scan kernels' device status
    else:
        check_status("VisionMamba-2D eager steps")
    ms = e0.elapsed_time(e1)
    tm = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    ms = float(tm.item())
    n_params = sum(p.numel() for p in model.parameters())
    del model, opt
    torch.cuda.empty_cache()
    imgs = cfg.global_batch if batch is None else b - a
    return {"img_per_s": imgs * steps / (ms / 1e3), "ms_per_step": ms / steps, "steps": steps,
            "warmup": warmup, "global_batch": imgs, "per_gpu_batch": b - a, "scaling": "strong",
            "dtype": "f32 (TF32 off)", "params": n_params, "loss": loss,
            "execution": "one CUDA graph per step (forward, backward, all-reduce, AdamW)" if graphed else "eager",
            "parallelism": f"DDP NCCL all-reduce x{world}" if world > 1 else "single GPU",
            "config": "img 224x224x1, patch 16, embed 384, depth 6, d_state 16, K=4 directions, MSE vs N(0,1)"}


def time_config1(dev, stream, iters=50):
    """Gated scan forward + VJP at the reference's published MambaBlock shape (batch 2, L 196,
    d_inner 1536: one MambaBlock of d_model 768), median of `iters` launches
    with a 256 MB L2 flush before each.  The reference publishes 1.2 ms for its
    fused Metal scan at this shape on an Apple M5 Pro (README.md:25); that is
    other hardware, so this is reported beside it, not as vs_baseline."""
    import statistics

    import torch

    t = make_inputs(2, 196, 1536, dev, seed=3)
    runner = AbiScan(t)
    st = torch.cuda.current_stream(dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev)
    for _ in range(5):
        runner.fwd(stream)
        runner.bwd(stream)
    res = {"fwd": [], "bwd": []}
    for _ in range(iters):
        flush.fill_(1.0)
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        e[0].record(st)
        runner.fwd(stream)
        e[1].record(st)
        runner.bwd(stream)
        e[2].record(st)
        e[2].synchronize()
        res["fwd"].append(e[0].elapsed_time(e[1]))
        res["bwd"].append(e[1].elapsed_time(e[2]))
    f, b = statistics.median(res["fwd"]), statistics.median(res["bwd"])
    del runner, t, flush
    return {"shape": "batch 2, L 196, d_inner 1536, d_state 16, gated", "fwd_ms": f, "bwd_ms": b,
            "fwd_plus_bwd_ms": f + b, "reference_published_ms": 1.2,
            "reference_published_on": "Apple M5 Pro, MLX 0.31, metal_fused scan (README.md:25)"}


def time_bf16_io(t, dev, stream, K, warmup):
    """The headline workload with the sequence tensors in bf16
    (vmscan_fwd_bf16 / vmscan_bwd_bf16; fp32 arithmetic and state).  Reported
    beside the metric, which stays fp32 like the reference."""
    import torch

    b, l, d = t["u"].shape
    runner = AbiScan(t, bf16=True)
    st = torch.cuda.current_stream(dev)
    for _ in range(warmup):
        runner.fwd(stream)
        runner.bwd(stream)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    torch.cuda.synchronize()
    for i in range(K):
        ev[i][0].record(st)
        runner.fwd(stream)
        ev[i][1].record(st)
        runner.bwd(stream)
        ev[i][2].record(st)
    torch.cuda.synchronize()
    f = statistics.mean(ev[i][0].elapsed_time(ev[i][1]) for i in range(K))
    bw = statistics.mean(ev[i][1].elapsed_time(ev[i][2]) for i in range(K))
    fb, bb = fwd_bytes(b, l, d, es=2), bwd_bytes(b, l, d, es=2)
    peak, _ = measured_peaks()
    del runner
    torch.cuda.empty_cache()
    return {"api": "vmscan_fwd_bf16 + vmscan_bwd_bf16", "fwd_ms": f, "bwd_ms": bw, "ms_per_step": f + bw,
            "fwd_gbs": fb / f / 1e6, "bwd_gbs": bb / bw / 1e6, "fwd_frac": fb / f / 1e6 / peak,
            "bwd_frac": bb / bw / 1e6 / peak, "algorithmic_bytes_per_step": fb + bb}


def time_conv(dev, iters=20):
    """Direction-aware causal conv1d + SiLU through the C ABI with
    preallocated buffers (forward, and VJP incl. the dw/dbias reductions) at
    the VisionMamba-2D block shape (64, 196, 768, K=4), row-major and
    column-major scan order on the 14 x 14 grid; median of `iters` launches
    after 3 warm-up ones, a 256 MB buffer overwritten before each.
    Algorithmic bytes per (token, channel): forward 8 (read x, write out),
    VJP 12 (read x and dout, write dx)."""
    import torch

    from mlx_vision_mamba_b200 import _native, directions_for

    lib = _native.load()
    b, l, c, k = 64, 196, 768, 4
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(b, l, c, device=dev, generator=g)
    w = torch.randn(c, k, 1, device=dev, generator=g) * 0.5
    bias = torch.randn(c, device=dev, generator=g) * 0.1
    dy = torch.randn(b, l, c, device=dev, generator=g)
    out, dx = torch.empty_like(x), torch.empty_like(x)
    dw, db = torch.empty_like(w), torch.empty_like(bias)
    ws_n = lib.vmscan_conv1d_bwd_workspace_bytes(b, l, c, k)
    ws = torch.empty(ws_n, dtype=torch.uint8, device=dev)
    S = _native.Strides(l * c, c)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev)
    st = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(st.cuda_stream)
    peak, _ = measured_peaks()
    res = {"shape": f"batch {b}, L {l}, channels {c}, K {k}", "api": "vmscan_conv1d_silu_fwd / _bwd"}
    for name, d in (("row_major", None), ("col_major", directions_for(4, (14, 14))[2])):
        dref = ctypes.byref(d.to_native()) if d is not None else None

        def fwd():
            rc = lib.vmscan_conv1d_silu_fwd(b, l, c, k, x.data_ptr(), S, w.data_ptr(), bias.data_ptr(),
                                            out.data_ptr(), S, None, None, dref, sp)
            assert rc == 0, rc

        def bwd():
            rc = lib.vmscan_conv1d_silu_bwd(b, l, c, k, x.data_ptr(), S, w.data_ptr(), bias.data_ptr(),
                                            dy.data_ptr(), S, dx.data_ptr(), S, None, dw.data_ptr(), db.data_ptr(), dref,
                                            ws.data_ptr(), ws_n, sp)
            assert rc == 0, rc

        tms = {}
        for fname, fn in (("fwd", fwd), ("bwd", bwd)):
            ts = []
            for it in range(iters + 3):
                flush.fill_(1.0)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                fn()
                e1.record(st)
                e1.synchronize()
                if it >= 3:
                    ts.append(e0.elapsed_time(e1))
            tms[fname] = statistics.median(ts)
        fb, bb = 8 * b * l * c, 12 * b * l * c
        res[name] = {"fwd_ms": tms["fwd"], "bwd_ms": tms["bwd"], "fwd_gbs": fb / tms["fwd"] / 1e6,
                     "bwd_gbs": bb / tms["bwd"] / 1e6, "fwd_frac": fb / tms["fwd"] / 1e6 / peak,
                     "bwd_frac": bb / tms["bwd"] / 1e6 / peak}
    del x, w, bias, dy, out, dx, ws, flush
    torch.cuda.empty_cache()
    return res


def time_dt(dev, iters=20):
    """dt_proj + bias + softplus (forward) and its softplus VJP through the C
    ABI at the VisionMamba-2D block shape: 64 x 196 tokens, dt_rank 24 read
    from the x_dbc rows (width 56), d_inner 768; median of `iters` launches
    after 3 warm-up ones, a 256 MB buffer overwritten before each.
    Algorithmic bytes per (token, channel): forward 4 (write delta), VJP 8
    (read ddelta, write dpre); the x rows and W add under 1 %."""
    import torch

    from mlx_vision_mamba_b200 import _native

    lib = _native.load()
    ntok, r, wide, dn = 64 * 196, 24, 56, 768
    g = torch.Generator(device=dev).manual_seed(12)
    xw = torch.randn(ntok, wide, device=dev, generator=g)
    w = torch.randn(dn, r, device=dev, generator=g) / r**0.5
    bias = torch.randn(dn, device=dev, generator=g)
    gin = torch.randn(ntok, dn, device=dev, generator=g)
    out = torch.empty(ntok, dn, device=dev)
    part = torch.empty(lib.vmscan_dt_softplus_bias_rows(ntok), dn, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev)
    st = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(st.cuda_stream)
    peak, _ = measured_peaks()

    def fwd():
        assert lib.vmscan_dt_softplus_fwd(ntok, r, dn, xw.data_ptr(), wide, w.data_ptr(), bias.data_ptr(),
                                          out.data_ptr(), dn, sp) == 0

    def bwd():
        assert lib.vmscan_dt_softplus_bwd(ntok, r, dn, xw.data_ptr(), wide, w.data_ptr(), bias.data_ptr(),
                                          gin.data_ptr(), dn, out.data_ptr(), dn, None, part.data_ptr(), sp) == 0

    res = {"shape": f"{ntok} tokens, dt_rank {r}, d_inner {dn}", "api": "vmscan_dt_softplus_fwd / _bwd"}
    for name, fn, byt in (("fwd", fwd, 4 * ntok * dn), ("bwd", bwd, 8 * ntok * dn)):
        ts = []
        for it in range(iters + 3):
            flush.fill_(1.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn()
            e1.record(st)
            e1.synchronize()
            if it >= 3:
                ts.append(e0.elapsed_time(e1))
        ms = statistics.median(ts)
        res[name + "_ms"] = ms
        res[name + "_gbs"] = byt / ms / 1e6
        res[name + "_frac"] = byt / ms / 1e6 / peak
    del xw, w, bias, gin, out, flush
    torch.cuda.empty_cache()
    return res


def time_gemm(dev, iters=20):
    """The block's projection GEMMs at the VisionMamba-2D shapes (64 x 196
    tokens, E 384, K=4 directions: in_proj 384 -> 6144, out_proj 3072 -> 384;
    forward, input gradient, weight gradient) on the tensor cores
    (vmscan_gemm_tf32x3 from split operands; the split passes timed
    separately) against PyTorch's fp32 GEMM with TF32 off.  Median of `iters`
    after 3 warm-ups.  TFLOP/s counts the fp32 GEMM's 2 M N K."""
    import torch

    from mlx_vision_mamba_b200.linear import gemm_tf32x3, tf32_split

    old_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device=dev).manual_seed(21)
    st = torch.cuda.current_stream(dev)
    with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
        bf16_peak = json.load(f).get("bf16_tflops")

    def med(fn):
        ts = []
        for it in range(iters + 3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn()
            e1.record(st)
            e1.synchronize()
            if it >= 3:
                ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    t = 64 * 196
    rows = []
    for name, fin, fout in (("in_proj", 384, 6144), ("out_proj", 3072, 384)):
        x = torch.randn(t, fin, device=dev, generator=g)
        w = torch.randn(fout, fin, device=dev, generator=g) / fin ** 0.5
        dy = torch.randn(t, fout, device=dev, generator=g)
        xs, ws, ds = tf32_split(x), tf32_split(w), tf32_split(dy)
        cases = (
            ("fwd", t, fout, fin, lambda: gemm_tf32x3(xs, False, ws, False, t, fout, fin), lambda: x @ w.t(),
             lambda: tf32_split(x)),
            ("dx", t, fin, fout, lambda: gemm_tf32x3(ds, False, ws, True, t, fin, fout), lambda: dy @ w,
             lambda: tf32_split(dy)),
            ("dw", fout, fin, t, lambda: gemm_tf32x3(ds, True, xs, True, fout, fin, t), lambda: dy.t() @ x, None),
        )
        for kind, m, n, k, ours, theirs, split in cases:
            ms_ours, ms_torch = med(ours), med(theirs)
            flops = 2.0 * m * n * k
            row = {"gemm": f"{name} {kind}", "m": m, "n": n, "k": k, "ms": ms_ours, "tflops": flops / ms_ours / 1e9,
                   "torch_fp32_ms": ms_torch, "torch_fp32_tflops": flops / ms_torch / 1e9,
                   "speedup": ms_torch / ms_ours}
            if split is not None:
                row["split_ms"] = med(split)
            rows.append(row)
        del x, w, dy, xs, ws, ds
    torch.cuda.empty_cache()
    torch.backends.cuda.matmul.allow_tf32 = old_tf32
    return {"api": "vmscan_gemm_tf32x3 (+ vmscan_tf32_split)", "tensor_peak_note":
            f"3 tf32 MMAs per output; measured bf16 peak {bf16_peak} TFLOP/s (tf32 is half)", "shapes": rows}


SWEEP = [(b, l, d) for b in (8, 64) for l in (196, 1024, 4096) for d in (768, 1536)]


def run_sweep(iters, warmup, bf16=False):
    """The op sweep (batch x L x d_inner = {8, 64} x {196, 1024, 4096} x {768,
    1536}, gated, seeded inputs with the sweep's distributions): forward and
    VJP through the C ABI timed separately with CUDA events, median of `iters`
    launches after `warmup`; a 256 MB buffer is overwritten before every timed
    launch whose inputs fit in L2, so no point is timed from a warm cache.
    Prints one JSON line per point and a table."""
    import statistics

    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream_t = torch.cuda.current_stream(dev)
    stream = ctypes.c_void_p(stream_t.cuda_stream)
    peak, peak_kind = measured_peaks()
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev)
    rows = []
    for b, l, d in SWEEP:
        t = make_inputs(b, l, d, dev, seed=7)
        runner = AbiScan(t, bf16=bf16)
        es = 2 if bf16 else 4
        in_bytes = es * 4 * b * l * d
        need_flush = in_bytes < 2 * 126 * 1024 * 1024
        res = {}
        for name, fn in (("fwd", runner.fwd), ("bwd", runner.bwd)):
            for _ in range(warmup):
                fn(stream)
            times = []
            for _ in range(iters):
                if need_flush:
                    flush.fill_(1.0)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream_t)
                fn(stream)
                e1.record(stream_t)
                e1.synchronize()
                times.append(e0.elapsed_time(e1))
            res[name] = statistics.median(times)
        fb, bb = fwd_bytes(b, l, d, es=es), bwd_bytes(b, l, d, es=es)
        row = {"io": "bf16" if bf16 else "f32", "batch": b, "seqlen": l, "d_inner": d, "fwd_ms": res["fwd"], "bwd_ms": res["bwd"],
               "fwd_gbs": fb / res["fwd"] / 1e6, "bwd_gbs": bb / res["bwd"] / 1e6,
               "fwd_frac": fb / res["fwd"] / 1e6 / peak, "bwd_frac": bb / res["bwd"] / 1e6 / peak,
               "l2_flush": need_flush, "peak": peak, "peak_source": peak_kind}
        rows.append(row)
        print(json.dumps(row), flush=True)
        del runner, t
        torch.cuda.empty_cache()
    print("| batch | L | d_inner | fwd ms | fwd GB/s | fwd % peak | VJP ms | VJP GB/s | VJP % peak |")
    print("|---:|---:|---:|---:|---:|---:|---:|---:|---:|")
    for r in rows:
        print(f"| {r['batch']} | {r['seqlen']} | {r['d_inner']} | {r['fwd_ms']:.4f} | {r['fwd_gbs']:.0f} | "
              f"{100 * r['fwd_frac']:.1f} | {r['bwd_ms']:.4f} | {r['bwd_gbs']:.0f} | {100 * r['bwd_frac']:.1f} |")


def profile_model(warmup, batch=None):
    """Device time per kernel of one VisionMamba-2D training step (1 GPU,
    torch.profiler over 2 steps after `warmup` steps), grouped as in the
    committed model-step summary; prints a table, not a bench line.  `batch`
    (default: the global batch of 64) sets the images per step, e.g. 8 for
    one GPU's share of the 8-GPU run."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    from mlx_vision_mamba_b200 import train

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    dev = torch.device("cuda", 0)
    cfg = train.VISION_MAMBA_2D
    model = train.build_encoder(cfg, dev, seed=0)
    opt = train.make_optimizer(model)
    x, tgt = train.synthetic_batch(cfg, batch or cfg.global_batch, dev, seed=100)
    for _ in range(max(warmup, 1)):
        train.train_step(model, opt, x, tgt)
    torch.cuda.synchronize()
    steps = 2
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            train.train_step(model, opt, x, tgt)
        torch.cuda.synchronize()
    rows = sorted(((e.device_time_total, e.count, e.key) for e in prof.key_averages() if e.device_time_total > 0),
                  reverse=True)
    total = sum(r[0] for r in rows)
    groups = {"gemm": 0.0, "scan_bwd": 0.0, "scan_fwd": 0.0, "conv": 0.0, "dt_proj": 0.0, "vmscan_reduce": 0.0,
              "other": 0.0}
    for t_us, _, key in rows:
        k = ("gemm" if "gemm" in key else "scan_bwd" if "scan_bwd_kernel" in key else
             "scan_fwd" if "scan_fwd_kernel" in key else "conv" if "vmscan::conv" in key else
             "dt_proj" if "vmscan::dt_softplus" in key else
             "vmscan_reduce" if "vmscan::reduce" in key else "other")
        groups[k] += t_us
    print(f"total device time per step: {total / steps / 1e3:.2f} ms")
    for k, v in groups.items():
        print(f"  {k:14s} {v / steps / 1e3:8.3f} ms  {100 * v / total:5.1f} %")
    print("top kernels:")
    for t_us, n, key in rows[:25]:
        print(f"  {t_us / steps / 1e3:8.3f} ms {100 * t_us / total:5.1f} % x{n // steps:4d} {key[:100]}")


ENCODERS = {
    "3d": ("VisionMamba-3D", "VisionMamba-3D K=6, input (16, 128, 128, 128, 1), patch 16 (512 tokens), E 384, "
           "depth 6, MSE vs N(0,1)"),
    "4d": ("VisionMamba-4D", "VisionMamba-4D K=8, input (8, 8, 64, 64, 64, 1), patch 16, temporal patch 1 "
           "(512 tokens), E 384, depth 6, MSE vs N(0,1)"),
}


def run_encoder(dev, rank, world, which, mode, steps, warmup, barrier):
    """VisionMamba-3D (K=6, 128^3 volumes, global batch 16)
    or -4D (K=8, 8 frames of 64^3, global batch 8) training steps,
    one CUDA graph per step.  "dp": the global batch split over the ranks,
    gradients averaged by DDP.  "dirshard": every rank takes the whole batch
    and runs its share of each layer's scan directions; the direction sums and
    the block-input gradients are all-reduced inside the step."""
    import torch
    import torch.distributed as dist

    from mlx_vision_mamba_b200 import train

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    cfg = train.VISION_MAMBA_3D if which == "3d" else train.VISION_MAMBA_4D
    name, workload = ENCODERS[which]
    side = torch.cuda.Stream(dev)
    if mode == "dp":
        a, b = train.shard(cfg.global_batch, rank, world)
        with torch.cuda.stream(side):
            model = train.wrap_data_parallel(train.build_encoder(cfg, dev, seed=0), dev)
        batch, seed = b - a, 100 + rank
    else:
        model = train.build_encoder(cfg, dev, seed=0)
        if world > 1:
            model.shard_directions(dist.group.WORLD)
        batch, seed = cfg.global_batch, 100
    torch.cuda.current_stream(dev).wait_stream(side)
    opt = train.make_optimizer(model, capturable=True)
    x, tgt = train.synthetic_batch(cfg, batch, dev, seed=seed)
    step = train.GraphedTrainStep(model, opt, x, tgt, side_stream=side)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        loss = step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    loss = float(loss.item())
    step.close()
    tm = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    ms = float(tm.item())
    return {"metric": f"{name} train img/s", "value": cfg.global_batch * steps / (ms / 1e3), "unit": "img/s",
            "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms / steps,
            "higher_is_better": True, "scaling": "strong", "dtype": "f32 (TF32 off)", "data": "synthetic",
            "loss": loss, "config": {"workload": workload,
                                     "global_batch": cfg.global_batch,
                                     "parallelism": (f"data parallel x{world} (DDP)" if mode == "dp" else
                                                     f"scan directions split x{world}, whole batch per rank"),
                                     "execution": "one CUDA graph per step"}}


def measure_host_link(dev, gib=1, reps=3):
    """Pinned host <-> device copy bandwidth of this GPU's link (GB/s):
    upload alone, download alone, and both at once on two streams (the
    pattern run_e2e uses), each the mean of `reps` copies of `gib` GiB."""
    import torch

    n = gib * 256 * 1024 * 1024
    hs = [torch.empty(n, dtype=torch.float32).pin_memory() for _ in range(2)]
    ds = [torch.empty(n, dtype=torch.float32, device=dev) for _ in range(2)]
    s_up, s_down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    comp = torch.cuda.current_stream(dev)

    def up():
        with torch.cuda.stream(s_up):
            ds[0].copy_(hs[0], non_blocking=True)

    def down():
        with torch.cuda.stream(s_down):
            hs[1].copy_(ds[1], non_blocking=True)

    def timed(fns):
        for f in fns:
            f()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        s_up.wait_stream(comp)
        s_down.wait_stream(comp)
        for _ in range(reps):
            for f in fns:
                f()
        comp.wait_stream(s_up)
        comp.wait_stream(s_down)
        e1.record(comp)
        torch.cuda.synchronize()
        return n * 4 * reps / (e0.elapsed_time(e1) / 1e3) / 1e9

    res = {"h2d_gbs": timed([up]), "d2h_gbs": timed([down]), "duplex_gbs_each_way": timed([up, down]),
           "method": f"{gib} GiB pinned copies, mean of {reps}, CUDA events"}
    del hs, ds
    torch.cuda.empty_cache()
    return res


def run_e2e(t, dev, K, warmup, world, barrier):
    """Public API (selective_scan_cuda + backward) with pinned host inputs and
    outputs.  Every step copies its own inputs host->device and its output and
    all gradients device->host inside the timed region; the copies run on
    their own streams, double-buffered, so step i+1's upload and step i-1's
    download overlap step i (PCIe is full duplex)."""
    import torch

    from mlx_vision_mamba_b200 import selective_scan_cuda

    host = {k: v.detach().cpu().pin_memory() for k, v in t.items()}
    b, l, d = t["u"].shape
    shapes = (("y", (b, l, d)), ("du", (b, l, d)), ("ddelta", (b, l, d)), ("dz", (b, l, d)), ("dA", (d, N_STATE)),
              ("dB", (b, l, N_STATE)), ("dC", (b, l, N_STATE)), ("dD", (d,)))
    outs = [{k: torch.empty(sh, dtype=torch.float32).pin_memory() for k, sh in shapes} for _ in range(2)]
    din = [{k: torch.empty_like(v, device=dev) for k, v in host.items()} for _ in range(2)]
    h2d = sum(v.numel() * 4 for v in host.values())
    d2h = sum(v.numel() * 4 for v in outs[0].values())
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    done = [torch.cuda.Event(), torch.cuda.Event()]
    for ev in done:
        ev.record(comp)

    def step(i):
        sl = i & 1
        with torch.cuda.stream(s_in):
            s_in.wait_event(done[sl])  # step i-2 finished reading this input slot
            for k, v in host.items():
                din[sl][k].copy_(v, non_blocking=True)
        comp.wait_stream(s_in)
        leaves = {}
        for k in ("u", "delta", "A", "B", "C", "D", "z"):
            leaves[k] = din[sl][k].detach().requires_grad_(True)
        y = selective_scan_cuda(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"],
                                leaves["D"], z=leaves["z"])
        y.backward(din[sl]["dy"])
        res = {"y": y.detach()}
        for k in ("u", "delta", "z", "A", "B", "C", "D"):
            res["d" + k] = leaves[k].grad
        done[sl].record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(done[sl])
            for k, v in res.items():
                v.record_stream(s_out)
                outs[sl][k].copy_(v, non_blocking=True)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    s_in.wait_stream(comp)
    for i in range(K):
        step(i)
    comp.wait_stream(s_out)
    e1.record(comp)
    torch.cuda.synchronize()
    check_status("e2e fwd+VJP")
    ms = e0.elapsed_time(e1)
    tm = torch.tensor([ms], device=dev)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    ms = float(tm.item())
    byt = fwd_bytes(b, l, d) + bwd_bytes(b, l, d)
    link = measure_host_link(dev)
    return {"value": world * K * byt / (ms / 1e3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms / K, "steps": K,
            "host_link": link,
            "copy_gbs_each_way": max(h2d, d2h) / (ms / K / 1e3) / 1e9,
            "api": "mlx_vision_mamba_b200.selective_scan_cuda(...).backward(dy), pinned host buffers, "
                   "uploads / downloads on their own streams (double-buffered, overlapping the previous / next step)"}


if __name__ == "__main__":
    main()
