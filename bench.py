"""Benchmark of the MXFP8 quantizer hot path (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step = one quantization of this rank's 8192 x 8192 bf16 N(0,1) matrix
into E4M3 payload + packed UE8M0 scales.  Under torchrun
with N ranks every rank quantizes its own 8192-row shard of a (8192*N) x 8192
matrix (64 row chunks of 128 rows each): weak scaling, no collective on the
data path; the timed region is bracketed by barriers and reported as the max
over ranks, with every rank's own time beside it.  Metric: effective TB/s =
(2MK + MK + MK/32) bytes / device time, summed over ranks.

Inputs rotate over enough workspaces (X, Q, S sets) that one rotation is more
than three times the L2 size, so every step streams from HBM.

Device timing: CUDA events on the launching stream around exactly K launches.
Before the start event the stream is held by a short spin kernel (torch's
``cuda._sleep``, ``--hold-ms``) while the host queues the launches, so the
timed region holds K back-to-back kernels and not the host's submission of
the first one (the method of nvbench's blocking kernel).  ``--hold-ms 0``
times without it.

The same JSON line also carries BASELINE config 5 (131072 x 16384 N(0, 2),
split by 128-row chunks over the ranks: strong scaling) under "c5", the
end-to-end figure through the public API with host buffers under "e2e" next
to the bare copy ceiling of the same bytes, and the CPU baselines.

``--impl reference`` times the reference recipe's CPU implementation (the
integer-exact C restatement in oracle/, all host threads) on a bounded row
sample of the same workload; rank 0 alone runs it.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import pathlib
import re
import statistics
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
M_DEFAULT, K_DEFAULT = 8192, 8192
METRIC = "effective TB/s (2MK+MK+MK/32 B / device time) at 8192x8192 bf16; % of HBM peak"
SCALE_VEC = 32
B200_L2_BYTES = 126 * 1024 * 1024  # when no device can be queried (CPU-only runs of the reference arm)
C5_M, C5_K = 131072, 16384


def algo_bytes(m: int, k: int) -> int:
    return 2 * m * k + m * k + m * (k // SCALE_VEC)


def launches_per_call(m: int, k: int, ld_x: int, q_any_offset: bool = False) -> int:
    """Kernel launches one mxfp8_quantize call makes: the pipelined kernel
    splits problems of more than 148*128 tiles (148*64 on its unaligned-row
    path and its any-offset store path, which run two CTAs per SM) into
    launches of whole 128-row tiles, mirroring kMaxTilesPerLaunch and
    kMaxTilesPerLaunchRows in csrc/quantize_tma.cu.  X is assumed 16-byte
    aligned (torch allocations are)."""
    col_tiles = -(-(-(-k // SCALE_VEC)) // 4)
    row_tiles = -(-m // 128)
    max_tiles = 148 * 128 if ld_x % 8 == 0 and not q_any_offset else 148 * 64
    rows_per_launch = max(1, max_tiles // col_tiles) if row_tiles * col_tiles > max_tiles else row_tiles
    return -(-row_tiles // rows_per_launch)


def measured_hbm_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def committed_traffic(m: int, k: int) -> float | None:
    """DRAM bytes per launch from the committed ncu summaries, if any."""
    for p in sorted((ROOT / "profiles").glob("*.md")) + sorted((ROOT / "profiles").glob("*.txt")):
        mt = re.search(rf"traffic_bytes_per_launch\[{m}x{k}\]:\s*([0-9.eE+]+)", p.read_text())
        if mt:
            return float(mt.group(1))
    return None


def l2_bytes() -> int:
    try:
        import torch

        if torch.cuda.is_available():
            return int(torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size)
    except Exception:
        pass
    return B200_L2_BYTES


def workspace_plan(m: int, k: int, l2: int) -> dict:
    """Rotating (X, Q, S) workspaces: enough that one rotation is > 3x L2."""
    q_cols = -(-k // SCALE_VEC) * SCALE_VEC
    s_bytes = (-(-m // 128) * 128) * (-(-(q_cols // SCALE_VEC) // 4) * 4)
    ws_bytes = 2 * m * k + m * q_cols + s_bytes
    n_ws = max(2, math.ceil(3 * l2 / ws_bytes))
    return {"q_cols": q_cols, "s_bytes": s_bytes, "ws_bytes": ws_bytes, "n_ws": n_ws, "l2": l2,
            "text": f"{n_ws} rotating workspaces of {ws_bytes / 1e6:.0f} MB (> 3x the {l2 / 1e6:.0f} MB L2)"}


def pci_of(device_index: int) -> tuple[int, int, int] | None:
    try:
        import torch

        p = torch.cuda.get_device_properties(device_index)
        return int(p.pci_domain_id), int(p.pci_bus_id), int(p.pci_device_id)
    except Exception:
        return None


class ClockSampler:
    """Samples SM clock and clock-event reasons with NVML from a background
    thread (about every 0.2 ms) for the life of the process; window(t0, t1)
    summarises the samples taken between two host times (time.perf_counter).
    The GPU is found by its PCI address, so the samples are of the device
    torch uses whatever CUDA_VISIBLE_DEVICES says."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, device_index: int, period_s: float = 0.0002):
        self.period = period_s
        self.samples: list[tuple[float, int, int]] = []
        self.max_mhz = None
        self.uuid = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            pci = pci_of(device_index)
            if pci is not None:
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(f"{pci[0]:08X}:{pci[1]:02X}:{pci[2]:02X}.0")
            else:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            uuid = pynvml.nvmlDeviceGetUUID(self.handle)
            self.uuid = uuid.decode() if isinstance(uuid, bytes) else uuid
        except Exception:
            self.nvml = None
        if self.nvml:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def _run(self):
        n = self.nvml
        while not self._stop.is_set():
            try:
                mhz = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
                reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((time.perf_counter(), mhz, reasons))
                if len(self.samples) > 200000:
                    del self.samples[:100000]
            except Exception:
                pass
            time.sleep(self.period)

    def close(self):
        if self._thread:
            self._stop.set()
            self._thread.join()
            self._thread = None

    def window(self, t0: float, t1: float) -> dict:
        """Median SM clock and the reasons seen in samples taken in [t0, t1]
        (samples with the gpu_idle reason are left out unless all have it)."""
        inside = [(mhz, r) for t, mhz, r in list(self.samples) if t0 <= t <= t1]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        busy = [s for s in inside if not (s[1] & 0x1)] or inside
        seen = 0
        for _, r in busy:
            seen |= r
        return {"sm_mhz": statistics.median(s[0] for s in busy), "sm_max_mhz": self.max_mhz,
                "reasons": [name for bit, name in self.REASONS.items() if seen & bit and bit != 0x1],
                "samples": len(busy), "window_ms": (t1 - t0) * 1e3}


def bind_to_gpu_numa_node(device_index: int) -> str | None:
    """Restrict this process to the host CPUs next to its GPU (so that pinned
    host buffers are first touched on the GPU's NUMA node).  Returns the CPU
    list used, or None when the topology is unknown or binding would change
    nothing."""
    pci = pci_of(device_index)
    if pci is None:
        return None
    node_dir = pathlib.Path(f"/sys/bus/pci/devices/{pci[0]:04x}:{pci[1]:02x}:{pci[2]:02x}.0")
    try:
        text = (node_dir / "local_cpulist").read_text().strip()
    except OSError:
        return None
    cpus = set()
    for part in text.split(","):
        if "-" in part:
            a, b = part.split("-")
            cpus.update(range(int(a), int(b) + 1))
        elif part:
            cpus.add(int(part))
    have = os.sched_getaffinity(0)
    use = cpus & have
    if not use or use == have:
        return None
    os.sched_setaffinity(0, use)
    return text


def hold_stream(ms: float, mhz: int | None) -> None:
    """Keep torch's current stream busy for about `ms` (a spin kernel of
    ms x clock cycles) so that what the host queues next starts back to back."""
    import torch

    if ms > 0:
        torch.cuda._sleep(int(ms * 1e3 * (mhz or 2000)))


def timed_region(run_steps, stream, sampler, barrier, hold_ms: float) -> tuple[float, dict]:
    """barrier + synchronize, [hold, start event, run_steps(), end event],
    synchronize + barrier.  Returns (elapsed ms on `stream`, clocks sampled
    from the hold's launch to the final synchronize)."""
    import torch

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    hold_stream(hold_ms, sampler.max_mhz)
    start.record(stream)
    run_steps()
    end.record(stream)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    barrier()
    return start.elapsed_time(end), sampler.window(t0, t1)


def per_rank_summary(per_rank_ms: list[float], steps: int) -> dict:
    slow = max(range(len(per_rank_ms)), key=lambda r: per_rank_ms[r])
    fast = min(range(len(per_rank_ms)), key=lambda r: per_rank_ms[r])
    return {"per_rank_ms_per_step": [t / steps for t in per_rank_ms], "slowest_rank": slow, "fastest_rank": fast,
            "spread": per_rank_ms[slow] / per_rank_ms[fast] - 1.0}


def cpu_oracle_time(x_bits, m_rows: int, k: int, reps: int, threads: int) -> float:
    import oracle  # test infrastructure: the CPU baseline only

    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        oracle.quantize(x_bits[:m_rows], "bf16", m_rows, -(-k // SCALE_VEC) * SCALE_VEC, nthreads=threads)
        best = min(best, time.perf_counter() - t0)
    return best


def torch_recipe_time(x_bits, m_rows: int, k: int, reps: int, threads: int) -> float:
    """The recipe as torch CPU tensor code (the package's restatement of the
    reference's reference_quantize, MXFP8_quantizer.py:610-641) plus packing
    the scale bytes into the chunk layout; best of `reps`."""
    import numpy as np
    import torch

    import MXFP8_quantizer

    pkg = MXFP8_quantizer.load_package()
    torch.set_num_threads(threads)
    q_cols = -(-k // SCALE_VEC) * SCALE_VEC
    x = torch.zeros((m_rows, q_cols), dtype=torch.bfloat16)
    x[:, :k] = torch.from_numpy(np.ascontiguousarray(x_bits[:m_rows]).view(np.int16)).view(torch.bfloat16)
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        scale, _q = pkg.reference_quantize(x)
        pkg.pack_scale_bytes(scale, m_rows, q_cols)
        best = min(best, time.perf_counter() - t0)
    return best


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def host_workload(m: int, k: int, seed: int):
    import numpy as np
    import torch

    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32)
    return torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def base_line(args, world: int) -> dict:
    """The fields both arms print identically (metric, workload, config)."""
    plan = workspace_plan(args.m, args.k, l2_bytes())
    return {
        "metric": METRIC,
        "unit": "TB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: N(0,1) bf16, seeded (no dataset involved)",
        "config": {
            "workload": f"{args.m}x{args.k} bf16 -> e4m3 + ue8m0 (tcgen05 128x4 chunks) per rank; "
                        f"rank r owns rows [r*{args.m}, (r+1)*{args.m}) of a ({args.m}*N)x{args.k} matrix",
            "m_per_rank": args.m, "k": args.k, "input_dtype": "bf16", "global_m": args.m * world,
            "q_offset_bytes": args.q_offset,
            "parallelism": f"row shards of 128-row chunks x{world}, no collective",
            "l2": plan["text"],
        },
    }


def reference_arm(args, rank: int, world: int) -> None:
    """CPU implementation of the recipe, rank 0 only."""
    if rank != 0:
        return
    sys_path_oracle()
    threads = cpu_threads()
    x = host_workload(args.m, args.k, 1)
    # size each step's row sample so the whole run stays within ~2 minutes
    probe_rows = min(args.m, 1024)
    t_probe = cpu_oracle_time(x, probe_rows, args.k, 1, threads)
    per_row = t_probe / probe_rows
    budget = min(0.5, 120.0 / max(1, args.steps + args.warmup))
    rows = int(max(128, min(args.m, budget / max(per_row, 1e-9))) // 128 * 128)
    for _ in range(args.warmup):
        cpu_oracle_time(x, rows, args.k, 1, threads)
    times = [cpu_oracle_time(x, rows, args.k, 1, threads) for _ in range(args.steps)]
    total = sum(times)
    value = algo_bytes(rows, args.k) * args.steps / total / 1e12
    line = base_line(args, world)
    sample = (f"{rows}x{args.k} rows of the workload per step, {threads} threads, C restatement of the recipe "
              f"on {cpu_model()}")
    line.update({
        "impl": "reference",
        "value": value,
        "ms_per_step": total / args.steps * 1e3,
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    })
    torch_rows = min(rows, 1024)
    t = torch_recipe_time(x, torch_rows, args.k, 3, threads)
    line["cpu_baseline_torch"] = {
        "value": algo_bytes(torch_rows, args.k) / t / 1e12, "unit": "TB/s", "cores": threads, "kind": "port",
        "sample": f"{torch_rows}x{args.k} rows, best of 3, the recipe as torch CPU tensor code incl. scale packing"}
    print(json.dumps(line), flush=True)


SIDE_BY_SIDE = [
    # (m, k, dtype, cold_l2): BASELINE config 2 and the reference README's table
    (8192, 8192, "bf16", False), (8192, 8192, "bf16", True), (16384, 16384, "bf16", False),
    (16384, 16384, "fp16", False), (32768, 16384, "bf16", False), (32768, 8192, "bf16", False),
    (16384, 16384, "bf16", True), (16385, 16384, "bf16", False), (2051, 2080, "fp16", False),
    (2048, 2048, "bf16", False), (16384, 4096, "fp16", False),
    # odd K: the reference pads X on the host and times its kernel on the padded matrix;
    # this library reads the unaligned rows in place
    (8192, 8191, "bf16", False), (16384, 16383, "bf16", False),
]


def reference_kernel_arm(args, rank: int, local: int) -> None:
    """The reference's CuTeDSL kernel and this library, each through its own
    run_quantizer (same timing rule: min over 5 passes of the mean of 50
    launches after 10 warm-up launches), on the same GPU, with NVML clock
    samples taken during each arm's run.  Needs the reference module; prints
    one JSON line per configuration."""
    if rank != 0:
        return
    import importlib.util

    import torch

    import MXFP8_quantizer

    torch.cuda.set_device(local)
    arms = []
    ref_file = pathlib.Path(args.reference_path) / "MXFP8_quantizer.py"
    if ref_file.exists():
        spec = importlib.util.spec_from_file_location("reference_mxfp8_quantizer", ref_file)
        ref = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(ref)
        # one runtime for every row, so its compile cache keeps the kernel between calls
        arms.append(("reference_cutedsl", ref.build_runtime()["run_quantizer"]))
    ours = MXFP8_quantizer.load_package()
    arms.append(("b200", ours.run_quantizer))
    sampler = ClockSampler(local, period_s=0.0005)
    common = {"rows_per_cta": 8, "k_tile": 256, "seed": 0}
    for m, k, dt, cold in SIDE_BY_SIDE:
        row = {"m": m, "k": k, "input_dtype": dt, "cold_l2": cold, "device": torch.cuda.get_device_name(local),
               "gpu_uuid": sampler.uuid}
        for name, fn in arms:
            # compile / first-call work outside the sampled window, then the sampled run
            fn(m=m, k=k, input_dtype=dt, warmup_iterations=1, iterations=1, benchmark_repeats=1, cold_l2=cold,
               skip_verification=True, **common)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            r = fn(m=m, k=k, input_dtype=dt, warmup_iterations=10, iterations=50, benchmark_repeats=5, cold_l2=cold,
                   skip_verification=False, **common)
            torch.cuda.synchronize()
            clocks = sampler.window(t0, time.perf_counter())
            row[name] = {key: r[key] for key in ("effective_tb_s", "runtime_min_us", "runtime_std_us",
                                                 "verification_passed", "q_max_byte_diff", "workspace_count")}
            row[name]["clocks"] = clocks
            torch.cuda.empty_cache()
        if "reference_cutedsl" in row:
            row["speedup"] = row["b200"]["effective_tb_s"] / row["reference_cutedsl"]["effective_tb_s"]
        print(json.dumps(row), flush=True)
    sampler.close()


def cpu_model() -> str:
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def sys_path_oracle():
    import sys

    p = str(ROOT / "oracle")
    if p not in sys.path:
        sys.path.insert(0, p)


def dequantize_arm(args, pkg, capi, xs, qs, ss, launch, n_ws, m, k, s_bytes, stream, barrier, rank, world,
                   sampler) -> None:
    """Time mxfp8_dequantize (E4M3 payload + packed scales -> bf16) on this
    rank's workload: reads MK + MK/32 bytes, writes 2MK."""
    import torch

    for i in range(n_ws):
        launch(i)
    ys = [torch.empty((m, k), dtype=torch.bfloat16, device=xs[0].device) for _ in range(n_ws)]
    lib = capi.lib()
    sh = stream.cuda_stream
    args_d = [(qs[i].data_ptr(), m, k, k, ss[i].data_ptr(), s_bytes, ys[i].data_ptr(), capi.BF16, k, sh)
              for i in range(n_ws)]

    def deq(i):
        rc = lib.mxfp8_dequantize(*args_d[i])
        if rc:
            capi.check(rc, "bench dequantize")

    deq(0)
    torch.cuda.synchronize()
    # exact check against a torch decode of the same payload and scales
    dense = pkg.decode_scale_bytes(ss[0], m, k).to(torch.float32)
    scale = torch.exp2(dense - 127.0).repeat_interleave(32, dim=1)
    ref = (qs[0].view(torch.float8_e4m3fn).to(torch.float32) * scale).to(torch.bfloat16)
    if not torch.equal(ref, ys[0]):
        raise SystemExit("dequantize output differs from the torch decode")
    del dense, scale, ref
    for i in range(args.warmup):
        deq(i % n_ws)

    def steps():
        for i in range(args.steps):
            deq(i % n_ws)

    elapsed, clocks = timed_region(steps, stream, sampler, barrier, args.hold_ms)
    max_ms = pkg.shard.max_over_ranks(elapsed, device=xs[0].device)
    nbytes = m * k + s_bytes + 2 * m * k
    peak, peak_kind = measured_hbm_peak()
    achieved = nbytes / (elapsed / args.steps * 1e-3) / 1e9
    if rank == 0:
        line = base_line(args, world)
        line["metric"] = "effective TB/s of mxfp8_dequantize (MK + MK/32 read + 2MK bf16 write) / device time"
        line["config"]["workload"] = f"{m}x{k} e4m3 + ue8m0 -> bf16 per rank"
        line.update({"op": "dequantize", "value": world * nbytes / (max_ms / args.steps * 1e-3) / 1e12,
                     "ms_per_step": max_ms / args.steps, "clocks": clocks,
                     "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                                  "frac": achieved / peak, "peak_kind": peak_kind, "traffic": None,
                                  "algorithmic_bytes_per_launch": nbytes},
                     "gpu_launches": args.steps})
        print(json.dumps(line), flush=True)


def run_c5(args, pkg, rank: int, world: int, dev, barrier, sampler, steps: int) -> dict:
    """X = 131072 x 16384 bf16 N(0, 2), split by 128-row
    chunks over the ranks (strong scaling: the whole matrix is fixed).  Each
    rank generates its rows in 1024-row blocks from per-block seeds, so the
    data is the same for every rank count; it quantizes its shard into its
    slice of Q and S with no collective on the data path.  Every rank calls
    this (the timing takes collective steps)."""
    import torch

    capi = pkg._capi
    m_total, k = C5_M, C5_K
    r0, r1 = pkg.shard.row_shard(m_total, world, rank)
    m = r1 - r0
    x = torch.empty((m, k), dtype=torch.bfloat16, device=dev)
    for b0 in range(r0, r1, 1024):
        g = torch.Generator(device=dev).manual_seed(4_000_000 + b0 // 1024)
        n = min(1024, r1 - b0)
        x[b0 - r0:b0 - r0 + n] = (torch.randn((1024, k), generator=g, device=dev) * 2.0)[:n].to(torch.bfloat16)
    s_bytes = capi.scale_storage_bytes(m, k)
    q = torch.empty((m, k), dtype=torch.uint8, device=dev)
    s = torch.empty((s_bytes,), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev)
    lib = capi.lib()
    a = (x.data_ptr(), 0, m, k, k, q.data_ptr(), m, k, k, s.data_ptr(), s_bytes, st.cuda_stream)
    capi.check(lib.mxfp8_quantize(*a), "c5 launch")
    torch.cuda.synchronize()
    ver = pkg.verify_quantizer_outputs({"x": x[:1024], "q_fp8": q[:1024].view(torch.float8_e4m3fn),
                                        "s_storage_bytes": s[:capi.scale_storage_bytes(1024, k)]},
                                       1024, k, 1024, k)
    if not ver["verification_passed"] or ver["q_max_byte_diff"] != 0:
        raise SystemExit(f"c5 verification failed on rank {rank}")
    for _ in range(args.warmup):
        lib.mxfp8_quantize(*a)

    def run():
        for _ in range(steps):
            lib.mxfp8_quantize(*a)

    elapsed, clocks = timed_region(run, st, sampler, barrier, args.hold_ms)
    if capi.device_status(clear=True):
        raise SystemExit("device status word set after the c5 timed region")
    per_rank = pkg.shard.gather_over_ranks(elapsed, device=dev)
    slowest = max(per_rank) / steps
    total = algo_bytes(m_total, k)
    del x, q, s
    torch.cuda.empty_cache()
    out = {"value": total / (slowest * 1e-3) / 1e12, "unit": "TB/s", "n_gpus": world, "steps": steps,
           "warmup": args.warmup, "ms_per_step": slowest,
           "per_gpu_tb_s": algo_bytes(m, k) / (slowest * 1e-3) / 1e12, "scaling": "strong",
           "gpu_launches": steps * launches_per_call(m, k, k), "clocks_rank0": clocks,
           "verification_rank0_first_1024_rows": ver["verification_passed"],
           "workload": f"131072x16384 bf16 N(0,2), rows [{r0}, {r1}) on rank {rank} of {world}"}
    out.update(per_rank_summary(per_rank, steps))
    return out


def c5_arm(args, rank: int, world: int, local: int) -> None:
    """`--workload c5`: config 5 alone, as its own JSON line."""
    import torch
    import torch.distributed as dist

    import MXFP8_quantizer

    pkg = MXFP8_quantizer.load_package()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    sampler = ClockSampler(local)
    r = run_c5(args, pkg, rank, world, dev, barrier, sampler, max(3, min(args.steps, 200)))
    sampler.close()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        r.update({"metric": "effective TB/s of BASELINE config 5 (131072x16384 bf16 N(0,2), row-sharded), "
                            "max over ranks",
                  "higher_is_better": True, "dtype": "f32",
                  "data": "synthetic: N(0,2) bf16 from per-1024-row-block seeds",
                  "config": {"workload": "131072x16384 bf16 split by 128-row chunks",
                             "parallelism": f"row shards of 128-row chunks x{world}, no collective"}})
        print(json.dumps(r), flush=True)


def copy_ceiling(x_host, q_host, s_host, x_dev, q_dev, s_dev, steps: int, dev, barrier) -> dict:
    """The host link's ceiling for the end-to-end step: the same bytes as one
    end-to-end step (X host->device, Q and S device->host), copied from and to
    the same pinned buffers, both directions at once on two streams, steps
    serialised like the end-to-end calls.  Also each direction alone."""
    import torch

    cur = torch.cuda.current_stream(dev)
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def step(up: bool, down: bool):
        ev = torch.cuda.Event()
        ev.record(cur)
        for st in (h2d, d2h):
            st.wait_event(ev)
        if up:
            with torch.cuda.stream(h2d):
                x_dev.copy_(x_host, non_blocking=True)
        if down:
            with torch.cuda.stream(d2h):
                q_host.copy_(q_dev, non_blocking=True)
                s_host.copy_(s_dev, non_blocking=True)
        for st in (h2d, d2h):
            e = torch.cuda.Event()
            e.record(st)
            cur.wait_event(e)

    out = {}
    for name, up, down in (("both", True, True), ("h2d_only", True, False), ("d2h_only", False, True)):
        step(up, down)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        e0.record(cur)
        for _ in range(steps):
            step(up, down)
        e1.record(cur)
        torch.cuda.synchronize()
        barrier()
        out[name] = e0.elapsed_time(e1) / steps
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["b200", "reference", "reference-kernel"], default="b200")
    ap.add_argument("--reference-path", default=str(ROOT / "baseline" / "_ref"),
                    help="directory holding the reference's MXFP8_quantizer.py (reference-kernel arm)")
    ap.add_argument("--m", type=int, default=M_DEFAULT)
    ap.add_argument("--k", type=int, default=K_DEFAULT)
    ap.add_argument("--e2e-steps", type=int, default=30)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-c5", action="store_true", help="leave config 5 out of the driver line")
    ap.add_argument("--hold-ms", type=float, default=2.0,
                    help="hold the stream this long before the start event so the timed launches are queued "
                         "back to back (0: no hold)")
    ap.add_argument("--workload", choices=["c2", "c5"], default="c2",
                    help="c2: 8192x8192 per rank (weak scaling, the driver's line); "
                         "c5: the 131072x16384 N(0,2) matrix split by 128-row chunks over the ranks (strong scaling)")
    ap.add_argument("--op", choices=["quantize", "dequantize"], default="quantize",
                    help="dequantize: time mxfp8_dequantize (E4M3 + scales -> bf16) on the same workload")
    ap.add_argument("--q-offset", type=int, default=0,
                    help="place each Q this many bytes past a 16-byte boundary (the kernel's any-offset store path)")
    ap.add_argument("--profile", action="store_true",
                    help="kernel launches only (verify, warm-up, K launches): the command profiled with ncu")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if not 0 <= args.q_offset < 64:
        raise SystemExit("--q-offset must be in [0, 64)")
    if not 0 <= args.hold_ms <= 100:
        raise SystemExit("--hold-ms must be in [0, 100]")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return
    if args.impl == "reference-kernel":
        reference_kernel_arm(args, rank, local)
        return
    if args.workload == "c5":
        c5_arm(args, rank, world, local)
        return

    import torch
    import torch.distributed as dist

    import MXFP8_quantizer

    pkg = MXFP8_quantizer.load_package()
    capi = pkg._capi
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    numa_cpus = bind_to_gpu_numa_node(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    # this rank's rows of the global (m * world) x k matrix: whole 128-row chunks
    r0, r1 = pkg.shard.row_shard(args.m * world, world, rank)
    m, k = r1 - r0, args.k
    # Q geometry: K rounded up to whole scale blocks (K itself on the driver's
    # line; an odd --k runs X through the kernel's unaligned-row path)
    plan = workspace_plan(m, k, l2_bytes())
    q_cols, s_bytes, n_ws, ws_bytes = plan["q_cols"], plan["s_bytes"], plan["n_ws"], plan["ws_bytes"]
    if s_bytes != capi.scale_storage_bytes(m, q_cols):
        raise SystemExit("scale storage size disagrees with the library")
    if args.op == "dequantize" and q_cols != k:
        raise SystemExit("--op dequantize needs --k a multiple of 32")
    nbytes = algo_bytes(m, k)
    gen = torch.Generator(device=dev).manual_seed(1 + rank)
    xs = [torch.randn((m, k), generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16) for _ in range(n_ws)]
    # Q as a view args.q_offset bytes into a slightly larger buffer (0: 16-byte aligned)
    qs = [torch.empty((m * q_cols + 64,), dtype=torch.uint8, device=dev)[args.q_offset:args.q_offset + m * q_cols]
          .view(m, q_cols) for _ in range(n_ws)]
    ss = [torch.empty((s_bytes,), dtype=torch.uint8, device=dev) for _ in range(n_ws)]
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream
    lib = capi.lib()
    launch_args = [(xs[i].data_ptr(), 0, m, k, k, qs[i].data_ptr(), m, q_cols, q_cols, ss[i].data_ptr(), s_bytes, sh)
                   for i in range(n_ws)]
    sampler = ClockSampler(local)

    def launch(i):
        rc = lib.mxfp8_quantize(*launch_args[i])
        if rc:
            capi.check(rc, "bench launch")

    if args.op == "dequantize":
        dequantize_arm(args, pkg, capi, xs, qs, ss, launch, n_ws, m, k, s_bytes, stream, barrier, rank, world,
                       sampler)
        sampler.close()
        if world > 1:
            dist.destroy_process_group()
        return

    # correctness gate before timing (the reference does the same, MXFP8_quantizer.py:912-935)
    launch(0)
    torch.cuda.synchronize()
    buffers = {"x": xs[0], "q_fp8": qs[0].view(torch.float8_e4m3fn), "s_storage_bytes": ss[0]}
    ver = pkg.verify_quantizer_outputs(buffers, m, q_cols, m, k)
    if not ver["verification_passed"] or ver["q_max_byte_diff"] != 0:
        raise SystemExit(f"verification failed on rank {rank}: {ver}")

    for i in range(args.warmup):
        launch(i % n_ws)
    torch.cuda.synchronize()
    if args.profile:
        for i in range(args.steps):
            launch(i % n_ws)
        torch.cuda.synchronize()
        if capi.device_status(clear=True):
            raise SystemExit("device status word set")
        if rank == 0:
            print(json.dumps({"profile_run": True, "m": m, "k": k, "launches": 1 + args.warmup + args.steps}))
        sampler.close()
        if world > 1:
            dist.destroy_process_group()
        return

    def steps():
        for i in range(args.steps):
            launch(i % n_ws)

    elapsed_ms, clocks = timed_region(steps, stream, sampler, barrier, args.hold_ms)
    status = capi.device_status(clear=True)
    if status:
        raise SystemExit(f"device status word {status:#x} after the timed region")
    per_rank = pkg.shard.gather_over_ranks(elapsed_ms, device=dev)
    per_rank_mhz = pkg.shard.gather_over_ranks(float(clocks["sm_mhz"] or 0.0), device=dev)
    max_ms = max(per_rank)
    ms_per_step = max_ms / args.steps
    value = world * nbytes / (ms_per_step * 1e-3) / 1e12

    # kernel roofline: this rank's average launch over the timed region
    peak, peak_kind = measured_hbm_peak()
    achieved = nbytes / (elapsed_ms / args.steps * 1e-3) / 1e9
    traffic = committed_traffic(m, k)

    # end to end through the public API with host buffers: pinned X in, Q and S out
    x_host = torch.empty((m, k), dtype=torch.bfloat16, pin_memory=True)
    x_host.copy_(xs[0].cpu())
    q_host = torch.empty((m, q_cols), dtype=torch.uint8, pin_memory=True)
    s_host = torch.empty((s_bytes,), dtype=torch.uint8, pin_memory=True)
    hq = pkg.HostQuantizer(m, k, torch.bfloat16, device=dev)
    for _ in range(2):
        hq(x_host, q_host, s_host)
    torch.cuda.synchronize()

    def e2e_steps():
        for _ in range(args.e2e_steps):
            hq(x_host, q_host, s_host)

    e2e_elapsed, _ = timed_region(e2e_steps, stream, sampler, barrier, 0.0)
    e2e_ms = max(pkg.shard.gather_over_ranks(e2e_elapsed, device=dev)) / args.e2e_steps
    if not torch.equal(q_host, qs[0].cpu()) or not torch.equal(s_host, ss[0].cpu()):
        raise SystemExit("end-to-end output differs from the device-resident result")
    e2e_value = world * nbytes / (e2e_ms * 1e-3) / 1e12
    ceil_ms = copy_ceiling(x_host, q_host, s_host, hq.x, hq.q, hq.s, args.e2e_steps, dev, barrier)
    ceil_ms = {name: max(pkg.shard.gather_over_ranks(v, device=dev)) for name, v in ceil_ms.items()}
    ceiling_value = world * nbytes / (ceil_ms["both"] * 1e-3) / 1e12
    del hq
    del xs, qs, ss
    torch.cuda.empty_cache()

    c5 = None
    if not args.no_c5 and args.m == M_DEFAULT and args.k == K_DEFAULT and args.q_offset == 0:
        c5 = run_c5(args, pkg, rank, world, dev, barrier, sampler, max(3, min(args.steps, 200)))
    sampler.close()  # no GPU work below; the CPU baselines get every host thread

    cpu = cpu_torch = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys_path_oracle()
        threads = cpu_threads()
        xb = x_host.view(torch.int16).numpy().view("uint16")
        t_all = cpu_oracle_time(xb, m, k, 3, threads)
        cpu = {"value": nbytes / t_all / 1e12, "unit": "TB/s", "cores": threads, "kind": "port",
               "sample": f"the full {m}x{k} workload, best of 3, C restatement of the recipe on {cpu_model()}"}
        torch_rows = min(m, 1024)
        t_torch = torch_recipe_time(xb, torch_rows, k, 3, threads)
        cpu_torch = {"value": algo_bytes(torch_rows, k) / t_torch / 1e12, "unit": "TB/s", "cores": threads,
                     "kind": "port",
                     "sample": f"{torch_rows}x{k} rows of the workload, best of 3, the recipe as torch CPU tensor "
                               f"code (reference_quantize) incl. scale packing"}

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = base_line(args, world)
    line.update({
        "value": value,
        "ms_per_step": ms_per_step,
        "clocks": clocks,
        "timing": {"hold_ms_before_start": args.hold_ms, "events_on": "the launching stream",
                   "per_rank_sm_mhz": per_rank_mhz, **per_rank_summary(per_rank, args.steps)},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind, "traffic": traffic,
                     "algorithmic_bytes_per_launch": nbytes},
        "e2e": {"value": e2e_value, "unit": "TB/s", "h2d_bytes_per_step": 2 * m * k,
                "d2h_bytes_per_step": m * q_cols + s_bytes, "ms_per_step": e2e_ms,
                "copy_ceiling": {"value": ceiling_value, "unit": "TB/s", "ms_per_step": ceil_ms["both"],
                                 "h2d_only_ms": ceil_ms["h2d_only"], "d2h_only_ms": ceil_ms["d2h_only"],
                                 "what": "the same bytes copied between the same pinned buffers, both "
                                         "directions at once, no kernel"},
                "frac_of_copy_ceiling": e2e_value / ceiling_value,
                "host_cpus": numa_cpus or "unchanged"},
        "gpu_launches": args.steps * launches_per_call(m, k, k, q_any_offset=args.q_offset % 16 != 0),
        "verification": ver,
    })
    if c5 is not None:
        line["c5"] = c5
    if cpu is not None:
        line["cpu_baseline"] = cpu
        line["cpu_baseline_torch"] = cpu_torch
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
