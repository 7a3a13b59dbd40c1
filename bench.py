"""bench.py -- headline benchmark of the TeamRedBench B200 backend.

Workload: the hbm STREAM triad a = b + s*c on float32
arrays of 2^30 elements (uniform[-1,1) inputs, s = 3.0), one independent
replica per GPU.  One step = one triad launch over the full arrays
(12.88 GB of algorithmic HBM traffic).  Inputs (12 GiB) are far larger than
the 126 MB L2, so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Under torchrun each rank drives LOCAL_RANK's GPU; timed windows are bracketed
by barrier + synchronize; `value` = all ranks' bytes / max-over-ranks time.
Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path


ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_ELEMS = 1 << 30
SCALE = 3.0
DTYPE = "float32"
BYTES_PER_STEP = 3 * N_ELEMS * 4
METRIC = "triad HBM GB/s (float32, 2^30 elements per GPU)"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
CLOCK_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
               "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
               "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


def parse_args() -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--variant", default="auto", help="hbm kernel variant: auto | vec | bulk")
    p.add_argument("--e2e-steps", type=int, default=3)
    p.add_argument("--no-extras", action="store_true", help="skip the secondary measurements")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def load_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text()), "measured"
        except (OSError, ValueError):
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(kernel_key: str) -> dict | None:
    """DRAM traffic of one full-size launch of a kernel, from the committed ncu
    capture (profiles/ncu_traffic.json)."""
    path = ROOT / "profiles" / "ncu_traffic.json"
    if not path.exists():
        return None
    try:
        data = json.loads(path.read_text())[kernel_key]
        return {k: data[k] for k in ("traffic_bytes_per_launch", "dram_read_bytes_per_launch",
                                     "dram_write_bytes_at_kernel_end", "written_back_after_kernel_end_bytes",
                                     "elements", "traffic_rule")}
    except (OSError, ValueError, KeyError, TypeError):
        return None


class ClockSampler:
    """nvidia-smi sampling of SM clocks / throttle reasons during a timed region."""

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={CLOCK_QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.file.name) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9 and parts[1].isdigit():
                    rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(float(r[1]) for r in rows), "sm_max_mhz": float(rows[0][2]),
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def dist_setup(gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_baseline_leg(torch_module) -> dict:
    """The oracle port timed on this host's cores, on a bounded sample (2^28 elements)."""
    import numpy as np

    import oracle

    n = 1 << 28
    rng = np.random.default_rng(0)
    b = (rng.random(n, dtype=np.float32) * 2 - 1).astype(np.float32)
    c = (rng.random(n, dtype=np.float32) * 2 - 1).astype(np.float32)
    out = np.empty_like(b)
    threads = oracle.default_threads()
    oracle.hbm("float32", "triad", b, c, SCALE, threads, out=out)  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.hbm("float32", "triad", b, c, SCALE, threads, out=out)
        reps += 1
        if time.perf_counter() - t0 > 5.0 or reps >= 40:
            break
    elapsed = (time.perf_counter() - t0) / reps
    del b, c, out
    return {"value": round(3 * n * 4 / elapsed / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"float32 triad over 2^28 elements (3.2 GB per pass), {reps} passes, oracle/trb_oracle.c",
            "gemm": cpu_gemm_baseline(torch_module)}


def cpu_gemm_baseline(torch_module) -> dict:
    """The reference's torch-CPU GEMM case (bf16 torch.mm, mfu.py:230-252) on this
    host's cores, beside the kernels' bf16 figures: a bounded sample of one
    warm-up and two or three timed calls per size (about 3 s in all)."""
    from oracle import reference_cpu

    prev = torch_module.get_num_threads()
    torch_module.set_num_threads(host_threads())
    out = {"kind": "reference torch.mm restated (oracle/reference_cpu.py)", "unit": "TFLOP/s",
           "cpu_capability": torch_module.backends.cpu.get_cpu_capability()}
    try:
        for size, iters in ((4096, 3), (8192, 2)):
            r = reference_cpu.time_gemm(torch_module, "bfloat16", size, size, size, 1, iters)
            out[f"bfloat16_{size}"] = {"value": round(r["tflops"], 3), "elapsed_s": round(r["elapsed_s"], 4),
                                       "cores": r["threads"], "sample": f"1 warm-up + {iters} timed calls"}
    finally:
        torch_module.set_num_threads(prev)
    return out


def host_threads() -> int:
    """Every core this process may run on (torchrun's OMP_NUM_THREADS=1 does not apply here)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover - non-Linux
        return os.cpu_count() or 1


def run_reference(args) -> None:
    """The reference's torch-CPU triad on this host's cores (rank 0 only; the
    other ranks exit without work).  It runs with every host thread at every
    N: the host's CPU path is one machine-wide resource, so N CPU replicas
    would only split the same cores and DRAM bandwidth between them."""
    world, rank, _ = dist_setup(args.gpus)
    if rank != 0:
        return
    import torch

    from oracle import reference_cpu

    threads = host_threads()
    torch.set_num_threads(threads)
    r = reference_cpu.time_hbm(torch, "triad", N_ELEMS, DTYPE, SCALE, args.warmup, args.steps)
    value = round(r["gbps"], 3)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": max(world, args.gpus),
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["elapsed_s"] * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "hbm_triad_float32_2^30", "elements": N_ELEMS, "scale": SCALE,
                   "path": "torch.add(b, c, alpha=s, out=a) on CPU (reference hbm.py:29-39)",
                   "host_aggregate": "one process on every host thread; N CPU replicas would share these cores"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": r["threads"], "kind": "port",
                         "sample": "full workload: float32 triad over 2^30 elements per step, torch CPU",
                         "cpu_capability": torch.backends.cpu.get_cpu_capability()},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200(args) -> None:
    import torch

    from teamredbench_b200 import _native
    from teamredbench_b200.kernels import gemm, stream_op

    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        # NCCL may print its version banner on stdout when its communicator
        # comes up (depending on the environment's NCCL settings); the
        # contract is one JSON line there, so fd 1 points at stderr until the
        # first collective has created the communicator.
        sys.stdout.flush()
        saved_stdout = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
            warm = torch.zeros(1, device=torch.device("cuda", local))
            dist.all_reduce(warm)
            torch.cuda.synchronize(local)
        finally:
            sys.stdout.flush()
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)
    dev = torch.device("cuda", local)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    g = torch.Generator(device=dev).manual_seed(0)
    b = torch.rand(N_ELEMS, generator=g, device=dev) * 2 - 1
    c = torch.rand(N_ELEMS, generator=g, device=dev) * 2 - 1
    a = torch.empty_like(b)
    stream = torch.cuda.current_stream(dev)

    def step():
        stream_op("triad", a, b, c, SCALE, variant=args.variant)

    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize(dev)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as sampler:
        start.record(stream)
        for _ in range(args.steps):
            step()
        stop.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    local_s = start.elapsed_time(stop) / 1e3
    max_s = max_over_ranks(local_s)
    clocks = sampler.summary()
    err = _native.device_error(local, clear=True)
    if err:
        raise RuntimeError(f"device error word {err} after the timed loop")

    peaks, peak_source = load_peaks()
    per_launch_s = local_s / max(args.steps, 1)
    achieved = BYTES_PER_STEP / per_launch_s / 1e9
    cap = load_traffic("hbm_triad_float32")
    same_size = cap is not None and cap["elements"] == N_ELEMS
    roofline = {"bound": "hbm", "achieved": round(achieved, 2), "peak": peaks.get("hbm_gbs"), "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": f"{peak_source} (STREAM copy, burst)",
                "traffic": cap["traffic_bytes_per_launch"] if same_size else None,
                "algorithmic_bytes_per_launch": BYTES_PER_STEP,
                "traffic_detail": ({k: cap[k] for k in ("dram_read_bytes_per_launch", "dram_write_bytes_at_kernel_end",
                                                        "written_back_after_kernel_end_bytes", "traffic_rule")}
                                   if same_size else None)}
    value = world * BYTES_PER_STEP * args.steps / max_s / 1e9

    # ---- e2e: the same triad through the C-ABI host entry point (pinned host
    # buffers; H2D of b and c and D2H of a inside every step).
    del a
    hb = b.cpu().pin_memory()
    hc = c.cpu().pin_memory()
    del b, c
    torch.cuda.empty_cache()
    ha = torch.empty_like(hb).pin_memory()
    _native.hbm_host(DTYPE, "triad", ha.data_ptr(), hb.data_ptr(), hc.data_ptr(), N_ELEMS, SCALE, local)  # warm-up
    barrier()
    e2e_local = 0.0
    for _ in range(max(args.e2e_steps, 1)):
        res = _native.hbm_host(DTYPE, "triad", ha.data_ptr(), hb.data_ptr(), hc.data_ptr(), N_ELEMS, SCALE, local)
        e2e_local += res.elapsed_s
    barrier()
    e2e_max = max_over_ranks(e2e_local)
    e2e_steps = max(args.e2e_steps, 1)
    e2e = {"value": round(world * BYTES_PER_STEP * e2e_steps / e2e_max / 1e9, 3), "unit": "GB/s",
           "h2d_bytes_per_step": 2 * N_ELEMS * 4, "d2h_bytes_per_step": N_ELEMS * 4, "steps": e2e_steps,
           "path": "trb_hbm_host (pinned host buffers, 64 MiB chunks on 3 streams)"}
    del ha, hb, hc
    torch.cuda.empty_cache()
    e2e["roofline"] = e2e_roofline(torch, dev, barrier, max_over_ranks, world, e2e["value"],
                                   e2e["h2d_bytes_per_step"], e2e["d2h_bytes_per_step"])

    # ---- GEMM replicas (BASELINE metric: bf16 / fp8 MFU per GPU at 1/2/4/8 GPUs)
    gemm_box = gemm_replicas(torch, dev, stream, barrier, max_over_ranks, world, local, dist)

    extras = {}
    if not args.no_extras:
        extras = secondary_measurements(torch, dev, stream, peaks)
        extras["scope"] = f"single-GPU measurements on rank {rank}"

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_leg(torch)

    if dist is not None:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(max_s / max(args.steps, 1) * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "hbm_triad_float32_2^30", "elements_per_gpu": N_ELEMS, "scale": SCALE,
                   "variant": args.variant, "parallelism": f"replicas{world}",
                   "l2": "inputs 12 GiB per GPU >> 126 MB L2; no flush needed"},
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": args.steps, "clocks": clocks,
        "gemm_replicas": gemm_box, "extras": extras,
    }
    print(json.dumps(line), flush=True)


def e2e_roofline(torch, dev, barrier, max_over_ranks, world, e2e_value, h2d_step, d2h_step) -> dict:
    """What bounds `e2e`: pinned host<->device copies, measured on every rank at
    once (512 MiB with cudaMemcpyAsync: H2D alone, D2H alone, and both directions
    together on two streams).  A step moves h2d_step bytes in and d2h_step out;
    it cannot be faster than its H2D bytes at the H2D-alone rate, so the limit
    is the triad's algorithmic bytes over that time, for all ranks together.
    All ranks share the host's DRAM and PCIe root, which also caps these
    copies as N grows."""
    nbytes = 1 << 29  # 512 MiB per direction: every rank already holds 12 GiB pinned for e2e
    h_in = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    h_out = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d_in = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    d_out = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def timed(h2d: bool, d2h: bool, reps: int = 3) -> float:
        e0, e1, mid = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
                       torch.cuda.Event())
        torch.cuda.synchronize(dev)
        barrier()
        e0.record(s1)
        s2.wait_event(e0)
        for _ in range(reps):
            if h2d:
                with torch.cuda.stream(s1):
                    d_in.copy_(h_in, non_blocking=True)
            if d2h:
                with torch.cuda.stream(s2):
                    h_out.copy_(d_out, non_blocking=True)
        mid.record(s2)
        s1.wait_event(mid)
        e1.record(s1)
        torch.cuda.synchronize(dev)
        return max_over_ranks(e0.elapsed_time(e1) / 1e3 / reps)

    timed(True, True, 1)  # warm-up
    t_h2d, t_d2h, t_both = timed(True, False), timed(False, True), timed(True, True)
    h2d_gbps = world * nbytes / t_h2d / 1e9
    d2h_gbps = world * nbytes / t_d2h / 1e9
    both_each_gbps = world * nbytes / t_both / 1e9  # each direction, both running
    # A step cannot be faster than bringing its inputs in at the rate the
    # host-to-device copies reach on their own.  Its D2H copies overlap them
    # but compete for host memory and PCIe, which is why e2e sits below this.
    step_s = world * h2d_step / (h2d_gbps * 1e9)
    limit = world * BYTES_PER_STEP / step_s / 1e9
    del h_in, h_out, d_in, d_out
    torch.cuda.empty_cache()
    return {"bound": "pcie (pinned host copies, all ranks at once)", "limit_gbps": round(limit, 2),
            "frac": round(e2e_value / limit, 4), "h2d_gbps": round(h2d_gbps, 2), "d2h_gbps": round(d2h_gbps, 2),
            "h2d_and_d2h_concurrent_gbps_each": round(both_each_gbps, 2),
            "how": "512 MiB cudaMemcpyAsync per direction, max over ranks; limit = triad bytes / (h2d bytes / "
                   "h2d-alone rate); the d2h and both-at-once rates are context"}


def gemm_replicas(torch, dev, stream, barrier, max_over_ranks, world, local, dist) -> dict:
    """bf16 and fp8 (e4m3) 8192^3 GEMM on every GPU at once, one independent
    replica per rank (BASELINE configs[2]/[3]; A, B ~ N(0,1)/sqrt(K), A drawn
    first; fp8 with per-tensor scales absmax/448, bf16 output).  Two windows,
    each bracketed by barrier + synchronize and timed with CUDA events, max over
    ranks: a burst of 20 launches, and ~1.5 s of back-to-back launches under
    the power cap with nvidia-smi clocks sampled on every rank."""
    from teamredbench_b200.kernels import gemm

    m = n = k = 8192
    flops = 2.0 * m * n * k
    nominal = {"bfloat16": 2250.0, "float8_e4m3fn": 4500.0}
    out = {}
    g = torch.Generator(device=dev).manual_seed(0)
    for name in ("bfloat16", "float8_e4m3fn"):
        a32 = torch.randn(m, k, generator=g, device=dev) / k ** 0.5
        b32 = torch.randn(k, n, generator=g, device=dev) / k ** 0.5
        if name == "bfloat16":
            a, b, sa, sb = a32.to(torch.bfloat16), b32.to(torch.bfloat16), 1.0, 1.0
        else:
            sa, sb = float(a32.abs().max()) / 448.0, float(b32.abs().max()) / 448.0
            a, b = (a32 / sa).to(torch.float8_e4m3fn), (b32 / sb).to(torch.float8_e4m3fn)
        del a32, b32
        c = torch.empty((m, n), device=dev, dtype=torch.bfloat16)

        def run(iters):
            for _ in range(iters):
                gemm(a, b, c, dtype=name, scale_a=sa, scale_b=sb)

        run(5)
        torch.cuda.synchronize(dev)

        def window(iters, sample=False):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier()
            torch.cuda.synchronize(dev)
            with (ClockSampler(local) if sample else contextlib.nullcontext()) as sampler:
                e0.record(stream)
                run(iters)
                e1.record(stream)
                torch.cuda.synchronize(dev)
            barrier()
            return max_over_ranks(e0.elapsed_time(e1) / 1e3), (sampler.summary() if sampler else None)

        burst_iters = 20
        t_burst, _ = window(burst_iters)
        sus_iters = max(50, int(1.5 / (t_burst / burst_iters)))
        sus_iters = int(max_over_ranks(float(sus_iters)))  # every rank runs the same count
        t_sus, clocks = window(sus_iters, sample=True)
        if dist is not None:
            gathered = [None] * world
            dist.all_gather_object(gathered, clocks)
        else:
            gathered = [clocks]
        box_burst = world * flops * burst_iters / t_burst / 1e12
        box_sus = world * flops * sus_iters / t_sus / 1e12
        out[name + "_8192"] = {
            "burst_box_tflops": round(box_burst, 1), "burst_per_gpu_tflops": round(box_burst / world, 1),
            "burst_mfu_pct_nominal": round(100 * box_burst / world / nominal[name], 2),
            "sustained_box_tflops": round(box_sus, 1), "sustained_per_gpu_tflops": round(box_sus / world, 1),
            "sustained_mfu_pct_nominal": round(100 * box_sus / world / nominal[name], 2),
            "sustained_launches": sus_iters, "sustained_window_s": round(t_sus, 3),
            "clocks_per_rank": [{kk: cl.get(kk) for kk in ("sm_mhz", "reasons", "power_w_max")} if cl else None
                                for cl in gathered],
        }
        del a, b, c
        torch.cuda.empty_cache()
    return out


def secondary_measurements(torch, dev, stream, peaks) -> dict:
    """bf16 triad, fp32 copy/scale, the 8192^3 bf16 / fp8 GEMMs, the skinny bf16
    GEMMs and float32 / float64 8192^3 (configs[1]-[3])."""
    from teamredbench_b200 import _native
    from teamredbench_b200.kernels import gemm, stream_op

    out = {}

    def timed(fn, iters=10, warm=3):
        for _ in range(warm):
            fn()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        s.record(stream)
        for _ in range(iters):
            fn()
        e.record(stream)
        torch.cuda.synchronize(dev)
        return s.elapsed_time(e) / 1e3 / iters

    g = torch.Generator(device=dev).manual_seed(0)
    for dt_name, torch_dt in (("float32", torch.float32), ("bfloat16", torch.bfloat16)):
        b = (torch.rand(N_ELEMS, generator=g, device=dev) * 2 - 1).to(torch_dt)
        c = (torch.rand(N_ELEMS, generator=g, device=dev) * 2 - 1).to(torch_dt)
        a = torch.empty_like(b)
        es = b.element_size()
        for mode in ("copy", "scale", "triad"):
            if dt_name == "float32" and mode == "triad":
                continue
            src = c if mode == "scale" else b
            t = timed(lambda: stream_op(mode, a, src, c if mode == "triad" else None, SCALE))
            moved = (3 if mode == "triad" else 2) * N_ELEMS * es
            out[f"hbm_{mode}_{dt_name}_gbps"] = round(moved / t / 1e9, 2)
        del a, b, c
    torch.cuda.empty_cache()

    # 8192^3 GEMMs (BASELINE configs[2]/[3]): A, B ~ N(0,1)/sqrt(K), A first.
    m = n = k = 8192
    nominal = {"bfloat16": 2250.0, "float8_e4m3fn": 4500.0}
    for name in ("bfloat16", "float8_e4m3fn"):
        a32 = torch.randn(m, k, generator=g, device=dev) / k ** 0.5
        b32 = torch.randn(k, n, generator=g, device=dev) / k ** 0.5
        if name == "bfloat16":
            a, b, sa, sb = a32.to(torch.bfloat16), b32.to(torch.bfloat16), 1.0, 1.0
        else:
            sa, sb = float(a32.abs().max()) / 448.0, float(b32.abs().max()) / 448.0
            a, b = (a32 / sa).to(torch.float8_e4m3fn), (b32 / sb).to(torch.float8_e4m3fn)
        del a32, b32
        c = torch.empty((m, n), device=dev, dtype=torch.bfloat16)
        t = timed(lambda: gemm(a, b, c, dtype=name, scale_a=sa, scale_b=sb), iters=20, warm=5)
        tflops = 2.0 * m * n * k / t / 1e12
        out[f"gemm_{name}_8192_tflops"] = round(tflops, 1)
        out[f"gemm_{name}_8192_mfu_pct_nominal"] = round(100 * tflops / nominal[name], 2)
        if name == "bfloat16":
            out["gemm_bfloat16_8192_frac_of_measured_cublas_burst"] = round(tflops / peaks["bf16_tflops"], 4)
        del a, b, c
        torch.cuda.empty_cache()
    # Skinny shapes (configs[3]: M = 16 / 128, N = K = 8192, bf16): HBM-bound, so
    # report the byte rate against the measured copy peak.  20 launches replayed
    # from a CUDA graph (the Python wrapper's host cost would otherwise show).
    def graph_timed(fn, reps=20, iters=5):
        fn()
        torch.cuda.synchronize(dev)
        cap = torch.cuda.Stream(dev)
        with torch.cuda.stream(cap):
            fn()
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=cap):
                for _ in range(reps):
                    fn()
        graph.replay()
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(iters):
            graph.replay()
        e.record(stream)
        torch.cuda.synchronize(dev)
        del graph
        return s.elapsed_time(e) / 1e3 / (reps * iters)

    for m in (16, 128):
        a = (torch.randn(m, k, generator=g, device=dev) / k ** 0.5).to(torch.bfloat16)
        b = (torch.randn(k, n, generator=g, device=dev) / k ** 0.5).to(torch.bfloat16)
        c = torch.empty((m, n), device=dev, dtype=torch.bfloat16)
        t = graph_timed(lambda: gemm(a, b, c))
        moved = (m * k + k * n + m * n) * 2
        out[f"gemm_bfloat16_skinny_m{m}_us"] = round(t * 1e6, 2)
        out[f"gemm_bfloat16_skinny_m{m}_frac_of_measured_hbm"] = round(moved / t / 1e9 / peaks["hbm_gbs"], 4)
        del a, b, c
    # float32 (three tf32 products) and float64 (CUDA cores) at 8192^3 -- the
    # reference's high-precision native path.
    for name, torch_dt in (("float32", torch.float32), ("float64", torch.float64)):
        a = torch.randn(8192, 8192, generator=g, device=dev, dtype=torch_dt) / 8192 ** 0.5
        b = torch.randn(8192, 8192, generator=g, device=dev, dtype=torch_dt) / 8192 ** 0.5
        c = torch.empty_like(a)
        t = timed(lambda: gemm(a, b, c), iters=5 if name == "float64" else 10, warm=2)
        out[f"gemm_{name}_8192_tflops"] = round(2.0 * 8192 ** 3 / t / 1e12, 1)
        del a, b, c
        torch.cuda.empty_cache()
    if _native.device_error(dev.index, clear=True):
        out["device_error"] = True
    return out


if __name__ == "__main__":
    arguments = parse_args()
    if arguments.impl == "reference":
        run_reference(arguments)
    else:
        run_b200(arguments)
