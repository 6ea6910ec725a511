"""Benchmark of the flight4s hot path on B200.

Headline workload (one "step"): the three full-array reductions over
n = 2^32 elements sharded contiguously over the N GPUs of one node
(strong scaling: the total is fixed at 2^32 per array):
    sum f32 (N(0,1), f64 accumulation), max/argmax f32 (same array),
    sum i32 (uniform [-1000, 1000]),
each one kernel launch per GPU followed, for N > 1, by one NCCL all_reduce
of the per-GPU partial.  Algorithmic bytes: 4 B per element per reduction,
48 GiB per step in total.  Inputs (16 GiB per array) are far larger than
L2 (126 MB), so no L2 flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Rank 0 prints one JSON line.  `value` is device-resident whole-job GB/s
(inputs already in HBM); `e2e` is the same step through the public
host-buffer call (f4s_reduce_host: pinned host -> device copies inside the
timed region).  At N = 1 the line also carries a per-kernel table for the
other hot-path kernels (vectorAdd, block sum, softmax, RMSNorm, FP8), the
CPU baseline (the same passes and warm-up as the reference arm) and how far
the f32 sum is from the reference's own Float fold on the same 2^32
elements (`results.f32_sum_vs_reference_float_fold`).  For N > 1,
`step_split` splits the step into kernel time and exposed collective time
(the same launches timed without their collectives), per rank.
`--impl reference` times the CPU restatement of the reference's path (the
oracle port, all host threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import datetime as _dt
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_TOTAL = 1 << 32
SEED = 0x5EED
HBM_PEAK_FALLBACK = 6650.0


def _peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return HBM_PEAK_FALLBACK, "fallback"


def _traffic_table() -> dict:
    """Per-launch DRAM bytes per element from the committed ncu summary."""
    p = ROOT / "profiles" / "dram_traffic.txt"
    out = {}
    if p.exists():
        for line in p.read_text().splitlines():
            parts = line.split()
            if len(parts) >= 2 and not line.startswith("#"):
                try:
                    out[parts[0]] = float(parts[1])
                except ValueError:
                    pass
    return out


class _stdout_to_stderr:
    """Points file descriptor 1 at stderr for the duration of the block."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)


# --------------------------------------------------------------- clocks
def _gpu_uuid(device: int) -> str:
    """NVML / nvidia-smi identifier of CUDA device `device` of this process."""
    import torch
    return "GPU-" + str(torch.cuda.get_device_properties(device).uuid)


class ClockSampler:
    def __init__(self, gpus: str):
        self.path = Path(f"/tmp/f4s_clocks_{os.getpid()}.csv")
        q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={gpus}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        self.windows: list[tuple[float, float]] = []
        # NVML read every ~2 ms as well (nvidia-smi's 100 ms period leaves a
        # sub-second timed region with one sample or none); read-only queries
        self.nvml: list[tuple[float, float, float, int]] = []
        self._handles = []
        try:
            import pynvml
            pynvml.nvmlInit()
            for tok in gpus.split(","):
                tok = tok.strip()
                self._handles.append(pynvml.nvmlDeviceGetHandleByIndex(int(tok)) if tok.isdigit()
                                     else pynvml.nvmlDeviceGetHandleByUUID(tok))
            self._nv = pynvml
            self._stop = threading.Event()
            self._thread = threading.Thread(target=self._poll, daemon=True)
            self._thread.start()
        except Exception:
            self._handles = []

    def _poll(self):
        nv = self._nv
        while not self._stop.is_set():
            t = time.time()
            for h in self._handles:
                try:
                    self.nvml.append((t, float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                      float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)),
                                      int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))))
                except Exception:
                    return
            time.sleep(0.002)

    def mark(self, t0: float, t1: float):
        self.windows.append((t0, t1))

    def summary(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait(timeout=10)
        rows = []
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = _dt.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(f[2]), float(f[3]), f[6:10]))
            except ValueError:
                continue
        self.path.unlink(missing_ok=True)
        if self._handles:
            self._stop.set()
            self._thread.join(timeout=5)
            nv = self._nv
            bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                    "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                    "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                    "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
            for t, sm, mx, r in self.nvml:
                rows.append((t, sm, mx, ["Active" if r & b else "Not Active" for b in bits.values()]))
        inside = [r for r in rows if any(a - 0.05 <= r[0] <= b + 0.05 for a, b in self.windows)]
        use = inside or rows
        if not use:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        mhz = sorted(r[1] for r in use)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in use for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": mhz[len(mhz) // 2], "sm_max_mhz": max(r[2] for r in use), "reasons": reasons,
                "samples": len(use), "samples_in_timed_region": len(inside)}


# ------------------------------------------------------------ CPU legs
def cpu_reference_run(n: int, steps: int, warmup: int, threads: int) -> dict:
    """The reference's CPU path restated (oracle): per-thread sequential
    Float folds (Array.sum), argmax and Int sum over `n` elements each."""
    import numpy as np

    from oracle import oracle as orc
    rng = np.random.default_rng(SEED)
    x = rng.standard_normal(n, dtype=np.float32)
    xi = rng.integers(-1000, 1001, n, dtype=np.int32)
    times = []
    for k in range(warmup + steps):
        t0 = time.perf_counter()
        orc.lib.orc_mt_sum_f32(x.ctypes.data, n, threads)
        orc.lib.orc_mt_argmax_f32(x.ctypes.data, n, threads)
        orc.lib.orc_mt_sum_i32(xi.ctypes.data, n, threads)
        t1 = time.perf_counter()
        if k >= warmup:
            times.append(t1 - t0)
    sec = sum(times) / len(times)
    gbs = 3 * 4 * n / sec / 1e9
    return {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"sum f32 + argmax f32 + sum i32 over 2^{n.bit_length() - 1} elements each, "
                      f"{steps} timed passes", "ms_per_step": sec * 1e3,
            "elements_per_s": 3 * n / sec}


# ------------------------------------------------------- GPU headline
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-kernels", action="store_true", help="skip the per-kernel table")
    ap.add_argument("--cpu-sample-log2", type=int, default=28)
    ap.add_argument("--e2e-max-log2", type=int, default=30,
                    help="cap on the per-rank host sample of each array in the e2e leg (pinned host memory)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--no-overlap", action="store_true",
                    help="launch each reduction only after the previous kernel finished (no launch overlap)")
    ap.add_argument("--profile", default=None,
                    help="profiling mode: run one kernel (or 'all') a few times on a small case and exit")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    threads = os.cpu_count() or 1

    if args.impl == "reference":
        if rank != 0:
            return
        r = cpu_reference_run(1 << args.cpu_sample_log2, args.steps, args.warmup, threads)
        line = {"metric": "achieved HBM GB/s", "value": r["value"], "unit": "GB/s", "impl": "reference",
                "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32/i32", "data": "synthetic (seeded numpy)",
                "elements_per_s": r["elements_per_s"],
                "config": {"workload": "full-array sum f32 + max/argmax f32 + sum i32 (reference CPU path, "
                                       "bounded sample)", "n": 1 << args.cpu_sample_log2},
                "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": r["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import numpy as np
    import torch
    import torch.distributed as dist

    import flight4s_b200 as f4s
    from flight4s_b200.sharded import ShardedReducer

    if args.profile:
        profile_run(args.profile)
        return

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        # NCCL may print a version banner on stdout while the communicator
        # comes up; keep stdout for the one JSON line.
        with _stdout_to_stderr():
            # NCCL on a high-priority stream: the step's small all_reduces are
            # scheduled ahead of the next step's reduction CTAs (measured
            # 2-3 us less exposed collective time per step at 2^29 per rank)
            opts = dist.ProcessGroupNCCL.Options()
            opts.is_high_priority_stream = True
            dist.init_process_group("nccl", device_id=dev, timeout=_dt.timedelta(seconds=300), pg_options=opts)
            dist.barrier(device_ids=[local])
            torch.cuda.synchronize()
    ctx = f4s.CudaContext.open(local)
    hp = ctx.hotpath()
    red = ShardedReducer(hp, dev, N_TOTAL)
    count, offset = red.count, red.offset
    stream = torch.cuda.current_stream()

    x = torch.empty(count, dtype=torch.float32, device=dev)
    xi = torch.empty(count, dtype=torch.int32, device=dev)
    hp.fill_synthetic(x, count, f4s.NORMAL_F32, seed=SEED, offset=offset, stream=stream)
    hp.fill_synthetic(xi, count, f4s.UNIFORM_I32, seed=SEED, offset=offset, ilo=-1000, ihi=1000, stream=stream)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    names = ["f4s_reduce_sum_f32", "f4s_reduce_argmax_f32", "f4s_reduce_sum_i32"]

    def step():
        # the three kernels back to back, their all_reduces (N > 1) after them
        with red.batch(stream):
            red.sum_f32_async(x, stream)
            red.argmax_f32_async(x, stream)
            red.sum_i32_async(xi, stream)

    # Inputs are resident and no kernel writes them inside the step, so each
    # reduction may start while the previous one finishes (launch overlap).
    hp.set_launch_overlap(not args.no_overlap)
    for _ in range(args.warmup):
        step()
    red.wait()
    # the GPUs the ranks use, by UUID (CUDA's device order need not be NVML's)
    sampler = ClockSampler(",".join(_gpu_uuid(i) for i in range(world))) if rank == 0 else None
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    time.sleep(0.3)  # let the sampler start
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_host0 = time.time()
    start.record(stream)
    for _ in range(args.steps):
        step()
    red.wait(stream)  # the last collectives belong to the timed region
    end.record(stream)
    torch.cuda.synchronize()
    t_host1 = time.time()
    barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.mark(t_host0, t_host1)
    ms_local = start.elapsed_time(end)
    ms_t = torch.tensor([ms_local], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_total = float(ms_t.item())
    ms_step = ms_total / args.steps

    # Each kernel alone: the same launches with events around each and no
    # overlap (an event between two kernels ends their overlap), after the
    # timed region; the per-kernel breakdown beside the step's figure.
    red.wait()
    hp.set_launch_overlap(False)
    kout = torch.zeros(2, dtype=torch.int64, device=dev)
    kops = [(f4s.REDUCE_SUM_F32, x), (f4s.REDUCE_ARGMAX_F32, x), (f4s.REDUCE_SUM_I32, xi)]
    kev = {name: [] for name in names}
    torch.cuda.synchronize()
    for rep in range(4 if world == 1 else 10):
        for name, (op, buf) in zip(names, kops):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            hp.reduce_into(op, buf, kout, n=count, stream=stream, index_base=offset, workspace=red.workspace)
            b.record(stream)
            if rep > 0:
                kev[name].append((a, b))
    torch.cuda.synchronize()
    kernel_ms_alone = {name: sum(a.elapsed_time(b) for a, b in evs) / len(evs) for name, evs in kev.items()}
    hp.set_launch_overlap(not args.no_overlap)

    # N > 1: the same kernels without their collectives, timed the same way,
    # so the step splits into kernel time and exposed collective time (each
    # the max over ranks), plus every rank's own figures
    step_split = None
    if world > 1:
        def kernels_only():
            for op, buf in kops:
                hp.reduce_into(op, buf, kout, n=count, stream=stream, index_base=offset, workspace=red.workspace)

        for _ in range(2):
            kernels_only()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        ka, kb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ka.record(stream)
        for _ in range(args.steps):
            kernels_only()
        kb.record(stream)
        torch.cuda.synchronize()
        mine = torch.tensor([ka.elapsed_time(kb) / args.steps, ms_local / args.steps]
                            + [kernel_ms_alone[name] for name in names], dtype=torch.float64, device=dev)
        every = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        rows = torch.stack(every).cpu().tolist()
        k_only = max(r[0] for r in rows)
        step_split = {"kernels_only_ms_per_step": k_only, "step_ms": ms_step,
                      "exposed_collective_ms_per_step": ms_step - k_only,
                      "per_rank": [{"rank": i, "kernels_only_ms": r[0], "step_ms": r[1],
                                    "kernel_ms_alone": dict(zip(names, r[2:]))}
                                   for i, r in enumerate(rows)],
                      "how": "CUDA events on each rank's compute stream; kernels-only = the same three launches "
                             "per step (same launch overlap) with no collectives"}

    # results of the last step (checked against torch on the full array at N = 1)
    red.wait()
    hp.set_launch_overlap(False)  # the rest (e2e, the kernel table) launches each kernel on its own
    s_val = float(red.f64.item())
    i_val = int(red.i32.item())
    v_max, i_max = ShardedReducer.argmax_result(red.arg)
    verified = None
    f32_parity = None
    if world == 1:
        ref_i = int(torch.sum(xi, dtype=torch.int64).item())
        ok_i = i_val == (ref_i + 2**31) % 2**32 - 2**31
        ok_a = i_max == int(torch.argmax(x).item())
        ref_s = torch.sum(x, dtype=torch.float64).item()
        abs_s = torch.sum(x.abs(), dtype=torch.float64).item()
        ok_s = abs(s_val - ref_s) <= 1e-5 * abs_s
        verified = bool(ok_i and ok_a and ok_s)
        f32_parity = reference_fold_gap(x, s_val, ref_s, abs_s) if not args.no_cpu else None

    peak, peak_kind = _peaks()
    bytes_step = 3 * 4 * N_TOTAL
    value = bytes_step / (ms_step / 1e3) / 1e9
    elements_s = 3 * N_TOTAL / (ms_step / 1e3)

    # ---- e2e through the host-buffer public call
    e2e = None
    if args.e2e_steps <= 0:
        e2e = {"value": None, "unit": "GB/s", "skipped": "--e2e-steps 0"}
    else:
      try:
        # pinned host sample per rank, capped so all ranks together pin at most 2^e2e_max_log2 x 8 bytes
        e2e_count = min(count, (1 << args.e2e_max_log2) // world)
        e2e = run_e2e(ctx, hp, red, x, xi, e2e_count, world, dev, args.e2e_steps, barrier)
      except Exception as exc:  # reported, not hidden
        e2e = {"value": None, "unit": "GB/s", "error": f"{type(exc).__name__}: {exc}"}
    del x, xi
    torch.cuda.empty_cache()

    kernels = None
    if world == 1 and not args.no_kernels:
        kernels = kernel_table(ctx, hp, dev, peak)

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    clocks = sampler.summary() if sampler else None
    # the three launches of a step are equal in size and run back to back,
    # overlapping start and finish: each one's average duration is a third
    # of the step (CUDA events on the launching stream over the timed region)
    per_launch_ms = ms_local / args.steps / 3
    dominant = max(kernel_ms_alone, key=kernel_ms_alone.get)
    per_launch_bytes = 4 * count
    achieved = per_launch_bytes / (per_launch_ms / 1e3) / 1e9
    traffic_per_elem = _traffic_table().get(dominant)
    # the same passes and warm-up as the reference arm (bench.py --impl reference)
    cpu = cpu_reference_run(1 << args.cpu_sample_log2, 20, 5, threads) if world == 1 and not args.no_cpu else None
    if cpu is not None:
        # the same port on one core, beside the all-core figure
        one = cpu_reference_run(1 << max(args.cpu_sample_log2 - 2, 10), 1, 1, 1)
        cpu["single_thread"] = {k: one[k] for k in ("value", "unit", "cores", "sample")}
    line = {
        "metric": "achieved HBM GB/s", "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32/i32", "data": "synthetic (device Philox: N(0,1) f32, U[-1000,1000] i32)",
        "elements_per_s": elements_s, "hbm_fraction": value / (peak * world),
        "config": {"workload": "full-array sum f32 + max/argmax f32 + sum i32, n=2^32 each, sharded over GPUs",
                   "n_total": N_TOTAL, "n_per_gpu": count, "parallelism": f"shard{world} + nccl all_reduce",
                   "launch_overlap": not args.no_overlap,
                   "l2": "inputs 16 GiB per array >> 126 MB L2 (no flush needed)"},
        "roofline": {"bound": "hbm", "kernel": " + ".join(names) + " (three equal launches per step, each "
                     "starting while the previous one finishes)", "achieved": achieved, "peak": peak,
                     "peak_kind": f"{peak_kind} hbm_gbs (copy) of MEASURED_PEAKS.json" if peak_kind == "measured"
                     else "fallback 6.65 TB/s", "unit": "GB/s", "frac": achieved / peak,
                     "traffic": (traffic_per_elem * count) if traffic_per_elem else None,
                     "traffic_kernel": dominant,
                     "algorithmic_bytes_per_launch": per_launch_bytes,
                     "launch_ms": per_launch_ms,
                     "kernel_ms_alone": kernel_ms_alone,
                     "frac_alone": {k: per_launch_bytes / (v / 1e3) / 1e9 / peak for k, v in kernel_ms_alone.items()}},
        "results": {"sum_f32": s_val, "sum_i32": i_val, "max_f32": v_max, "argmax": i_max, "verified_vs_torch": verified,
                    "f32_sum_vs_reference_float_fold": f32_parity},
        "step_split": step_split,
        "gpu_launches": 3 * args.steps * world,
        "clocks": clocks,
        "e2e": e2e,
        "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample", "single_thread")}
        if cpu else None,
        "kernels": kernels,
    }
    print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def reference_fold_gap(x, ours: float, exact: float, abs_sum: float) -> dict:
    """The f32 sum here against what the reference returns for the same
    array: its F32 ReduceSum accumulates in Float
    (core/src/main/scala/flight4s/core/types/CudaType.scala:216-218) and its
    own check is Scala's Array[Float].sum, a sequential Float fold
    (runtime/src/test/scala/flight4s/runtime/cuda/CudaResourcesJniSuite.scala:238).
    The fold runs on the host over 256 MiB chunks copied back from the
    device, carrying its Float accumulator; `exact` is torch's f64 sum of the
    same device data.  Gaps are relative to sum|x|."""
    import numpy as np

    from oracle import oracle as orc
    t0 = time.perf_counter()
    fold = 0.0
    chunk = 1 << 26
    for c in range(0, x.numel(), chunk):
        fold = orc.sum_f32_sequential(x[c:c + chunk].cpu().numpy(), fold)
    rounded = float(np.float32(ours))
    return {"n": int(x.numel()), "ours_f64": ours, "ours_rounded_to_f32": rounded, "reference_float_fold": fold,
            "exact": exact, "sum_abs": abs_sum,
            "rel_gap_ours": abs(ours - exact) / abs_sum, "rel_gap_ours_rounded_f32": abs(rounded - exact) / abs_sum,
            "rel_gap_reference_fold": abs(fold - exact) / abs_sum, "rel_gap_ours_f32_vs_fold": abs(rounded - fold) / abs_sum,
            "fold_seconds": time.perf_counter() - t0,
            "exact_is": "torch.sum(x, dtype=float64) on the device"}


def run_e2e(ctx, hp, red, x, xi, count, world, dev, steps, barrier) -> dict:
    """Same step through f4s_reduce_host: the rank's shard in pinned host
    memory, chunked H2D copies overlapped with the kernels, the result
    copied back to the host; for N > 1 the partials are combined across
    ranks exactly as in the device path."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import flight4s_b200 as f4s
    from flight4s_b200._native import check, lib

    hx = ctx.allocate_pinned("f32", count)
    hxi = ctx.allocate_pinned("i32", count)
    check(lib.f4s_copy_device_to_host(ctx.handle, x.data_ptr(), 0, hx.address, 4 * count), "shard to host")
    check(lib.f4s_copy_device_to_host(ctx.handle, xi.data_ptr(), 0, hxi.address, 4 * count), "shard to host")
    staging = ctx.allocate("u8", 256 + 2 * (256 << 20))
    s_copy, s_comp = ctx.create_stream(non_blocking=True), ctx.create_stream(non_blocking=True)
    base = red.offset

    def step():
        # sum and argmax of the f32 array share one transfer of each chunk
        rs, ra = hp.reduce_host_sum_argmax(hx.array, staging, s_copy, s_comp, index_base=base)
        ri = hp.reduce_host(f4s.REDUCE_SUM_I32, hxi.array, staging, s_copy, s_comp)
        if world > 1:
            t = torch.tensor([rs[:1].view(np.float64)[0]], dtype=torch.float64, device=dev)
            k = torch.tensor([int(ra.view(np.int64)[0])], dtype=torch.int64, device=dev)
            ti = torch.tensor([int(ri[:1].view(np.int32)[0])], dtype=torch.int32, device=dev)
            dist.all_reduce(t)
            dist.all_reduce(k, op=dist.ReduceOp.MAX)
            dist.all_reduce(ti)
            return t.item(), k.item(), ti.item()
        return rs, ra, ri

    step()  # warm-up
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    t1 = time.perf_counter()
    sec = torch.tensor([(t1 - t0) / steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(sec, op=dist.ReduceOp.MAX)
    sec_step = float(sec.item())
    for b in (hx, hxi):
        b.close()
    staging.close()
    s_copy.close()
    s_comp.close()
    return {"value": 3 * 4 * count * world / sec_step / 1e9, "unit": "GB/s",
            "h2d_bytes_per_step": 2 * 4 * count * world, "d2h_bytes_per_step": (8 + 16 + 4) * world,
            "ms_per_step": sec_step * 1e3, "steps": steps, "elements_per_rank": count,
            "sample": f"{count} elements of each array per rank ({3 * 4 * count * world / 2**30:g} GiB of reduction "
                      f"input per step over {world} GPU(s)) from pinned host memory, {steps} timed steps",
            "api": "f4s_reduce_host_sum_argmax_f32 + f4s_reduce_host (pinned host shard, chunked H2D "
                   "overlapped with the kernels; each host byte crosses PCIe once per step)",
            "bytes_counted": "3 reductions x 4 B x elements, as in value"}


def profile_run(which: str) -> None:
    """Small cases for ncu: each selected kernel 1 warm-up + 3 launches.
    Inputs exceed L2 (126 MB) except the block sum, whose benchmark size is
    4 MiB (2^20 f32); the row ops and FP8 run at their benchmark shapes
    (32768 x 8192, 16384 x 16384); at most ~2.2 GB is on the device at once."""
    import torch

    import flight4s_b200 as f4s
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    ctx = f4s.CudaContext.open(0)
    hp = ctx.hotpath()
    want = (lambda k: True) if which == "all" else (lambda k: k == which)

    def rep(fn):
        for _ in range(4):
            fn()
        torch.cuda.synchronize()

    n = 1 << 28
    if any(want(k) for k in ("reduce_sum_f32", "reduce_argmax_f32", "reduce_sum_i32")):
        x = torch.empty(n, dtype=torch.float32, device=dev)
        hp.fill_synthetic(x, n, f4s.NORMAL_F32, seed=SEED)
        out = torch.zeros(2, dtype=torch.int64, device=dev)
        if want("reduce_sum_f32"):
            rep(lambda: hp.reduce_into(f4s.REDUCE_SUM_F32, x, out))
        if want("reduce_argmax_f32"):
            rep(lambda: hp.reduce_into(f4s.REDUCE_ARGMAX_F32, x, out))
        if want("reduce_sum_i32"):
            hp.fill_synthetic(x, n, f4s.UNIFORM_I32, seed=SEED, ilo=-1000, ihi=1000)
            rep(lambda: hp.reduce_into(f4s.REDUCE_SUM_I32, x, out))
        del x
    typed = [k for k in ("bf16", "f16", "e4m3", "e5m2", "f64", "u32") if want(f"reduce_sum_{k}")]
    if typed:
        raw = torch.randint(0, 256, (1 << 30,), dtype=torch.uint8, device=dev)
        out = torch.zeros(2, dtype=torch.int64, device=dev)
        for k in typed:
            rep(lambda: hp.reduce_sum_into(k, raw, out, n=(1 << 30) // f4s.hotpath.SUM_TYPE_BYTES[k]))
        del raw
    typed_arg = [k for k in ("f16", "i32", "u32", "f64") if want(f"reduce_argmax_{k}")]
    if typed_arg:
        raw = torch.randint(0, 256, (1 << 30,), dtype=torch.uint8, device=dev)
        out = torch.zeros(2, dtype=torch.int64, device=dev)
        for k in typed_arg:
            rep(lambda: hp.reduce_argmax_into(k, raw, out, n=(1 << 30) // f4s.hotpath.ARGMAX_TYPE_BYTES[k]))
        del raw
    if want("reduce_ordered_f32"):
        raw = torch.randint(0, 256, (1 << 30,), dtype=torch.uint8, device=dev)
        out = torch.zeros(2, dtype=torch.int64, device=dev)
        rep(lambda: hp.reduce_sum_into("f32", raw, out, n=1 << 28, policy="deterministic"))
        del raw
    if want("convert"):
        m = 1 << 26
        xf = torch.empty(m, dtype=torch.float32, device=dev)
        hp.fill_synthetic(xf, m, f4s.NORMAL_F32, seed=SEED, p0=0.0, p1=100.0)
        h16 = torch.empty(m, dtype=torch.uint16, device=dev)
        q8 = torch.empty(m, dtype=torch.uint8, device=dev)
        rep(lambda: hp.convert_into("f32", "bf16", xf, h16))
        rep(lambda: hp.convert_into("f32", "e4m3", xf, q8))
        rep(lambda: hp.convert_into("e4m3", "f32", q8, xf))
        del xf, h16, q8
    if want("vector_add_f32") or want("vector_add_bf16"):
        m = 1 << 26
        for dtype, kind, fn, key in [(torch.float32, f4s.UNIFORM_F32, hp.vector_add_f32, "vector_add_f32"),
                                     (torch.bfloat16, f4s.UNIFORM_BF16, hp.vector_add_bf16, "vector_add_bf16")]:
            if not want(key):
                continue
            a = torch.empty(m, dtype=dtype, device=dev)
            b = torch.empty_like(a)
            c = torch.empty_like(a)
            hp.fill_synthetic(a, m, kind, seed=1)
            hp.fill_synthetic(b, m, kind, seed=2)
            rep(lambda: fn(a, b, c))
            del a, b, c
    if want("block_sum"):
        m = 1 << 20
        x = torch.empty(m, dtype=torch.float32, device=dev)
        hp.fill_synthetic(x, m, f4s.UNIFORM_F32, seed=SEED)
        parts = torch.empty(m // 256, dtype=torch.float32, device=dev)
        o = torch.empty(1, dtype=torch.float32, device=dev)
        ws = torch.zeros(hp.block_reduce_workspace_bytes(m), dtype=torch.uint8, device=dev)
        rep(lambda: hp.block_reduce_sum_f32_into(x, parts, o, ws))
    rows, cols = 32768, 8192  # the row-op benchmark shape: 512 MiB in, 512 MiB out
    if want("softmax") or want("rmsnorm"):
        xb = torch.empty(rows * cols, dtype=torch.bfloat16, device=dev)
        yb = torch.empty_like(xb)
        w = torch.empty(cols, dtype=torch.bfloat16, device=dev)
        hp.fill_synthetic(xb, rows * cols, f4s.NORMAL_BF16, seed=SEED)
        hp.fill_synthetic(w, cols, f4s.NORMAL_BF16, seed=SEED + 1, p0=1.0, p1=0.1)
        if want("softmax"):
            rep(lambda: hp.softmax_rows_bf16(xb, yb, rows, cols))
        if want("rmsnorm"):
            rep(lambda: hp.rmsnorm_rows_bf16(xb, w, yb, rows, cols, 1e-6))
        del xb, yb
    if want("fp8_quant") or want("fp8_dequant"):
        rows = cols = 16384  # the FP8 benchmark shape
        m = rows * cols
        xb = torch.empty(m, dtype=torch.bfloat16, device=dev)
        hp.fill_synthetic(xb, m, f4s.NORMAL_BF16_OUTLIERS, seed=SEED, p0=0.0, p1=2.0, p2=1e-3, p3=50.0)
        q = torch.empty(m, dtype=torch.uint8, device=dev)
        s = torch.empty(m // 128, dtype=torch.float32, device=dev)
        y = torch.empty_like(xb)
        hp.fp8_quantize_e4m3(xb, q, s, rows, cols)
        if want("fp8_quant"):
            rep(lambda: hp.fp8_quantize_e4m3(xb, q, s, rows, cols))
        if want("fp8_dequant"):
            rep(lambda: hp.fp8_dequantize_e4m3(q, s, y, rows, cols))
    torch.cuda.synchronize()
    print(f"profile run done: {which}")
    ctx.close()


def kernel_table(ctx, hp, dev, peak) -> dict:
    """The other hot-path kernels at their benchmark configurations, 1 GPU,
    CUDA events around `reps` back-to-back launches after warm-up.  Every
    section allocates its own buffers after releasing the previous ones to
    the driver: carved out of one reused allocator segment, an input and an
    output 1 GiB apart measured 3-8% slower for the write-heavy kernels."""
    import torch

    import flight4s_b200 as f4s
    out = {}
    stream = torch.cuda.current_stream()

    def timeit(fn, reps=20, warm=3, flush=None):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(reps):
            if flush is not None:
                flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            times.append((a, b))
        torch.cuda.synchronize()
        # median kernel time over the reps (the per-kernel figure the
        # measurement plan asks for; the mean is reported beside it)
        ms = sorted(a.elapsed_time(b) for a, b in times)
        timeit.mean = sum(ms) / len(ms)
        return ms[len(ms) // 2] if len(ms) % 2 else 0.5 * (ms[len(ms) // 2 - 1] + ms[len(ms) // 2])

    def row(name, nbytes, elems, ms, **extra):
        gbs = nbytes / (ms / 1e3) / 1e9
        out[name] = {"ms": ms, "gbs": gbs, "frac": gbs / peak, "elements_per_s": elems / (ms / 1e3),
                     "bytes": nbytes, **extra}
        if "timing" not in extra:  # event-timed: median of 20 reps, mean beside it
            out[name].update(ms_mean=timeit.mean, reps=20, stat="median")

    n = 1 << 28
    a = torch.empty(n, dtype=torch.float32, device=dev)
    b = torch.empty_like(a)
    c = torch.empty_like(a)
    hp.fill_synthetic(a, n, f4s.UNIFORM_F32, seed=1)
    hp.fill_synthetic(b, n, f4s.UNIFORM_F32, seed=2)
    row("vector_add_f32 n=2^28", 12 * n, n, timeit(lambda: hp.vector_add_f32(a, b, c, stream=stream)))
    del a, b, c
    torch.cuda.empty_cache()  # next section on freshly allocated buffers
    a = torch.empty(n, dtype=torch.bfloat16, device=dev)
    b = torch.empty_like(a)
    c = torch.empty_like(a)
    hp.fill_synthetic(a, n, f4s.UNIFORM_BF16, seed=1)
    hp.fill_synthetic(b, n, f4s.UNIFORM_BF16, seed=2)
    row("vector_add_bf16 n=2^28", 6 * n, n, timeit(lambda: hp.vector_add_bf16(a, b, c, stream=stream)))
    del a, b, c
    torch.cuda.empty_cache()  # next section on freshly allocated buffers

    # block sum, n = 2^20 (4 MiB: L2-resident when hot)
    n = 1 << 20
    x = torch.empty(n, dtype=torch.float32, device=dev)
    hp.fill_synthetic(x, n, f4s.UNIFORM_F32, seed=SEED)
    parts = torch.empty(n // 256, dtype=torch.float32, device=dev)
    o = torch.empty(1, dtype=torch.float32, device=dev)
    ws = torch.zeros(hp.block_reduce_workspace_bytes(n), dtype=torch.uint8, device=dev)
    # A 4 MiB block sum runs for a few microseconds, less than one host-side
    # launch through Python, so it is timed as CUDA-graph replays of
    # back-to-back calls (device time per call: the tiles kernel and its
    # one-CTA upper pass).
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def graph_ms(body, count):
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            body()  # warm-up outside capture
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=side):
                for _ in range(count):
                    body()
        g.replay()
        torch.cuda.synchronize()
        times = []
        for _ in range(7):  # median of 7 replays
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b) / count)
        return sorted(times)[3]

    bs = lambda: hp.block_reduce_sum_f32_into(x, parts, o, ws, stream=torch.cuda.current_stream())  # noqa: E731
    row("block_reduce_sum_f32 n=2^20 hot-L2", 4 * n + 4 * (n // 256), n, graph_ms(bs, 100), timing="cuda graph, median of 7 replays")
    flushed = graph_ms(lambda: (flush.zero_(), bs()), 50) - graph_ms(lambda: flush.zero_(), 50)
    row("block_reduce_sum_f32 n=2^20 L2-flushed", 4 * n + 4 * (n // 256), n, flushed, timing="cuda graph, median of 7 replays")
    del flush
    torch.cuda.empty_cache()  # next section on freshly allocated buffers

    # ReduceSum over the other accumulator input types, 8 GiB of input each
    # (random bits; larger than L2, so no flush is needed between launches)
    raw = torch.randint(0, 256, (8 << 30,), dtype=torch.uint8, device=dev)
    acc = torch.zeros(2, dtype=torch.int64, device=dev)
    for dtype, size in [("bf16", 2), ("f16", 2), ("e4m3", 1), ("e5m2", 1), ("f64", 8), ("u32", 4)]:
        count = (8 << 30) // size
        row(f"reduce_sum_{dtype} 8 GiB", 8 << 30, count,
            timeit(lambda: hp.reduce_sum_into(dtype, raw, acc, n=count, stream=stream)))
    # max / argmax over the other OrderedTypes (16-byte records), same bytes
    for dtype, size in [("f16", 2), ("i32", 4), ("u32", 4), ("f64", 8)]:
        count = (8 << 30) // size
        row(f"reduce_argmax_{dtype} 8 GiB", 8 << 30, count,
            timeit(lambda: hp.reduce_argmax_into(dtype, raw, acc, n=count, stream=stream)))
    # the order-fixed ("deterministic") policy of the same sums
    for dtype, size in [("f32", 4), ("bf16", 2), ("e4m3", 1)]:
        count = (8 << 30) // size
        ws_o = torch.zeros(hp.policy_workspace_bytes(dtype, count, "deterministic"), dtype=torch.uint8, device=dev)
        row(f"reduce_sum_{dtype} deterministic 8 GiB", 8 << 30, count,
            timeit(lambda: hp.reduce_sum_into(dtype, raw, acc, n=count, stream=stream, workspace=ws_o,
                                              policy="deterministic")))
    del raw
    torch.cuda.empty_cache()  # next section on freshly allocated buffers

    # ReduceSum of a pinned host array through the host-buffer call (PCIe
    # host-to-device copies inside the call), fast and order-fixed; the call
    # synchronizes its own two streams, so it is timed by the host clock
    n = 1 << 28
    hx = ctx.allocate_pinned("f32", n)
    hx.array[:] = 1.0
    staging = ctx.allocate("u8", 256 + 2 * (256 << 20))
    s_copy, s_comp = ctx.create_stream(non_blocking=True), ctx.create_stream(non_blocking=True)
    for policy in ("fast", "deterministic"):
        for _ in range(2):
            hp.reduce_host_sum("f32", hx.array, staging, s_copy, s_comp, policy=policy)
        ts = []
        for _ in range(5):
            t0 = time.perf_counter()
            hp.reduce_host_sum("f32", hx.array, staging, s_copy, s_comp, policy=policy)
            ts.append(time.perf_counter() - t0)
        row(f"host-buffer reduce_sum_f32 {policy} 1 GiB", 4 * n, n, sorted(ts)[2] * 1e3,
            timing="host wall clock, median of 5 synchronous calls", bound="PCIe host-to-device")
    for b in (s_copy, s_comp, staging, hx):
        b.close()

    # elementwise Convert, 2^28 elements (f32 side 1 GiB)
    n = 1 << 28
    xf = torch.empty(n, dtype=torch.float32, device=dev)
    hp.fill_synthetic(xf, n, f4s.NORMAL_F32, seed=SEED, p0=0.0, p1=100.0)
    h16 = torch.empty(n, dtype=torch.uint16, device=dev)
    q8 = torch.empty(n, dtype=torch.uint8, device=dev)
    yf = torch.empty_like(xf)
    row("convert f32->bf16 rn n=2^28", 6 * n, n, timeit(lambda: hp.convert_into("f32", "bf16", xf, h16, stream=stream)))
    row("convert f32->f16 rz n=2^28", 6 * n, n,
        timeit(lambda: hp.convert_into("f32", "f16", xf, h16, rounding="toward_zero", stream=stream)))
    row("convert f32->e4m3 satfinite n=2^28", 5 * n, n,
        timeit(lambda: hp.convert_into("f32", "e4m3", xf, q8, stream=stream)))
    row("convert e4m3->f32 n=2^28", 5 * n, n, timeit(lambda: hp.convert_into("e4m3", "f32", q8, yf, stream=stream)))
    row("convert f16->f32 n=2^28", 6 * n, n, timeit(lambda: hp.convert_into("f16", "f32", h16, yf, stream=stream)))
    del xf, h16, q8, yf
    torch.cuda.empty_cache()  # next section on freshly allocated buffers

    rows, cols = 32768, 8192
    xb = torch.empty(rows * cols, dtype=torch.bfloat16, device=dev)
    yb = torch.empty_like(xb)
    w = torch.empty(cols, dtype=torch.bfloat16, device=dev)
    hp.fill_synthetic(xb, rows * cols, f4s.NORMAL_BF16, seed=SEED)
    hp.fill_synthetic(w, cols, f4s.NORMAL_BF16, seed=SEED + 1, p0=1.0, p1=0.1)
    row("softmax_rows_bf16 32768x8192", 4 * rows * cols, rows * cols,
        timeit(lambda: hp.softmax_rows_bf16(xb, yb, rows, cols, stream=stream)))
    row("rmsnorm_rows_bf16 32768x8192", 4 * rows * cols + 2 * cols, rows * cols,
        timeit(lambda: hp.rmsnorm_rows_bf16(xb, w, yb, rows, cols, 1e-6, stream=stream)))
    del xb, yb, w
    torch.cuda.empty_cache()  # next section on freshly allocated buffers

    rows = cols = 16384
    n = rows * cols
    xb = torch.empty(n, dtype=torch.bfloat16, device=dev)
    hp.fill_synthetic(xb, n, f4s.NORMAL_BF16_OUTLIERS, seed=SEED, p0=0.0, p1=2.0, p2=1e-3, p3=50.0)
    q = torch.empty(n, dtype=torch.uint8, device=dev)
    s = torch.empty(n // 128, dtype=torch.float32, device=dev)
    y = torch.empty_like(xb)
    qb = 2 * n + n + 4 * (n // 128)
    row("fp8_quantize_e4m3 16384x16384", qb, n, timeit(lambda: hp.fp8_quantize_e4m3(xb, q, s, rows, cols, stream=stream)))
    row("fp8_dequantize_e4m3 16384x16384", qb, n,
        timeit(lambda: hp.fp8_dequantize_e4m3(q, s, y, rows, cols, stream=stream)))
    del xb, q, s, y
    torch.cuda.empty_cache()
    return out


if __name__ == "__main__":
    main()
