"""Benchmark of the north-star op: Q4_K x Q8_K decode matvec on B200.

Workload (batch 1): one step = the three Q4_K matvecs
4096->12288, 12288->4096 and 4096->4096, each quantizing its f32 activation
to Q8_K inside the kernel.  Algorithmic bytes per matvec = packed weight bytes
N*(K/256)*144 + f32 activation K*4 + f32 output N*4; 66,224,128 B per step.

* value   -- GB/s over the timed region: K steps replayed from a CUDA graph,
             CUDA events on the capture stream, barrier + synchronize on both
             sides, max over ranks.  A step is ONE launch of the persistent
             matvec-program kernel running the three independent matvecs
             (oracle_cuda_matvec_program).  Weights rotate through a pool of 6
             sets (397 MB, > 3x the 126 MB L2), so every step reads them from HBM.
* e2e     -- the same metric through the public host-pointer C ABI call
             (oracle_cuda_host_storage_matvec, Q8_K contract) with pinned host
             x and y: each step copies x in, runs, copies y out, synchronises.
* roofline -- the program kernel (the only kernel in the timed region):
             algorithmic bytes / average launch time against MEASURED_PEAKS.json
             hbm_gbs; the same step as three separate single-matvec launches and
             each shape alone (graphs of back-to-back launches) are reported too.
* cpu_baseline -- the CPU restatement (oracle/, single thread) on a bounded
             row sample of the same matrices.

--impl reference times the CPU implementation of the path on all host
threads.  Oracle has no Q4_K decoder and no Q8_K integer dot (its storage
decoder rejects type 12), so that arm runs the C restatement of GGML's
algorithm (kind "port").  Multi-GPU (torchrun): every rank runs the full step
on its own weights (weak scaling, no collective in the data path).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
SHAPES = [(4096, 12288), (12288, 4096), (4096, 4096)]  # (K, N): K -> N
TYPE_Q4_K = 12
POOL_SETS = 6
METRIC = "Q4_K x Q8_K decode matvec GB/s"
UNIT = "GB/s"


def algorithmic_bytes(k: int, n: int) -> int:
    return n * (k // 256) * 144 + k * 4 + n * 4


STEP_BYTES = sum(algorithmic_bytes(k, n) for k, n in SHAPES)
H2D_BYTES = sum(k * 4 for k, _ in SHAPES)
D2H_BYTES = sum(n * 4 for _, n in SHAPES)


def config_block(n_gpus: int) -> dict:
    return {"workload": "config2: Q4_K x Q8_K decode matvec, batch 1, shapes 4096->12288, 12288->4096, "
                        "4096->4096 (activation quantized to Q8_K in-kernel)",
            "shapes_k_to_n": [f"{k}->{n}" for k, n in SHAPES],
            "batch": 1,
            "bytes_per_step": STEP_BYTES,
            "l2": f"weights rotate through {POOL_SETS} sets ({POOL_SETS * sum(n * (k // 256) * 144 for k, n in SHAPES) / 1e6:.0f} MB > 3x L2)",
            "parallelism": f"replicas{n_gpus}" if n_gpus > 1 else "single"}


def load_peaks() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_traffic() -> float | None:
    path = os.path.join(ROOT, "profiles", "q4k_q8k_matvec_traffic.json")
    try:
        with open(path) as f:
            return float(json.load(f)["dram_bytes_per_step"])
    except Exception:
        return None


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """Polls NVML (SM clock, throttle reasons, power) every ~2 ms while running."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, device_index: int):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._handle = None
        try:
            import pynvml as nv
            import torch
            nv.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            for i in range(nv.nvmlDeviceGetCount()):
                h = nv.nvmlDeviceGetHandleByIndex(i)
                u = nv.nvmlDeviceGetUUID(h)
                u = u.decode() if isinstance(u, bytes) else u
                if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                    self._handle = h
            if self._handle is None and nv.nvmlDeviceGetCount() == 1:
                self._handle = nv.nvmlDeviceGetHandleByIndex(0)
            self._nv = nv
            if self._handle is not None:
                self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self._handle, nv.NVML_CLOCK_SM)
        except Exception:
            self._handle = None

    def _sample(self):
        nv = self._nv
        mhz = nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM)
        try:
            reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
        except Exception:
            reasons = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._handle)
        self.samples.append((mhz, reasons))

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(0.002)

    def __enter__(self):
        if self._handle is not None:
            self._sample()
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._handle is not None:
            self._stop.set()
            self._t.join()
            self._sample()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"], "samples": 0}
        mask = 0
        for _, r in self.samples:
            mask |= r
        names = [n for bit, n in self.REASONS.items() if mask & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# ---------------------------------------------------------------- distributed plumbing

def dist_setup(n_gpus: int):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, local, world


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- CPU legs

def cpu_sample_rows(k: int, n: int, fraction: float) -> int:
    return max(1, int(n * fraction))


def time_cpu_port(weights, xs, fraction: float, threads: int) -> tuple[float, int, float]:
    """Run the restatement's Q8_K quantize + matvec over `fraction` of each
    matrix's rows on `threads` threads.  Returns (seconds, bytes, check)."""
    import oracle
    port = oracle.port()
    total_bytes = 0
    jobs = []
    for (k, n), w, x in zip(SHAPES, weights, xs):
        rows = cpu_sample_rows(k, n, fraction)
        total_bytes += rows * (k // 256) * 144 + k * 4 + rows * 4
        jobs.append((k, rows, w, x))
    results = []

    def work(k, lo, hi, w, q8):
        results.append(port.matvec_q8_k(TYPE_Q4_K, hi - lo, k, w[lo:hi], q8)[0].sum())

    t0 = time.perf_counter()
    for k, rows, w, x in jobs:
        q8 = port.quantize_q8_k(x)
        bounds = np.linspace(0, rows, threads + 1).astype(int)
        ts = [threading.Thread(target=work, args=(k, bounds[i], bounds[i + 1], w, q8))
              for i in range(threads) if bounds[i + 1] > bounds[i]]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
    dt = time.perf_counter() - t0
    return dt, total_bytes, float(np.sum(results))


def host_weights():
    from oracle_b200 import synth
    ws = [synth.weight(TYPE_Q4_K, n, k, "config2", f"W_{k}_{n}") for k, n in SHAPES]
    xs = [synth.activations(k, 1, "config2", f"x_{k}")[0] for k, _ in SHAPES]
    return ws, xs


def cpu_baseline_leg(target_seconds: float = 3.0) -> dict:
    """The whole config-2 step on one core, repeated for about target_seconds."""
    ws, xs = host_weights()
    time_cpu_port(ws, xs, 1.0, 1)  # warm
    total_t, total_b, reps = 0.0, 0, 0
    while total_t < target_seconds:
        dt, nbytes, _ = time_cpu_port(ws, xs, 1.0, 1)
        total_t += dt
        total_b += nbytes
        reps += 1
    return {"value": total_b / total_t / 1e9, "unit": UNIT, "cores": 1, "kind": "port",
            "sample": f"the full config-2 step ({STEP_BYTES / 1e6:.1f} MB) x {reps} repetitions, Q8_K quantize + "
                      f"integer dot, single-threaded C restatement (oracle/quant_oracle.c), {total_t:.1f} s"}


def reference_arm(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and rank != 0:
        return
    threads = os.cpu_count() or 1
    ws, xs = host_weights()
    dt, _, _ = time_cpu_port(ws, xs, 0.01, threads)
    # one step is a bounded sample sized for about 0.5 s on all threads
    fraction = min(1.0, 0.01 * 0.5 / max(dt, 1e-4))
    for _ in range(args.warmup):
        time_cpu_port(ws, xs, fraction, threads)
    total_t, total_b = 0.0, 0
    for _ in range(args.steps):
        dt, nb, _ = time_cpu_port(ws, xs, fraction, threads)
        total_t += dt
        total_b += nb
    value = total_b / total_t / 1e9
    sample = (f"{fraction * 100:.2f}% of the rows of each config-2 matrix per step on {threads} threads; "
              "Oracle has no Q4_K decoder or Q8_K dot (storage_decode.cpp:192-196 rejects type 12), so this "
              "is the C restatement of GGML's algorithm (oracle/quant_oracle.c)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_t / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/u4 -> f32",
            "data": "synthetic", "config": config_block(args.gpus),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm

def gpu_arm(args) -> None:
    import torch

    import oracle_b200 as ob

    rank, local, world = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ctx = ob.Context(local, flags=ob.FLAG_PDL if not args.no_pdl else 0)
    ws, xs = host_weights()
    # weight pool: set 0 is the seeded host weights; others are byte-rotations
    # of it (same distribution, distinct addresses) so every step misses L2
    pool = []
    for s in range(POOL_SETS):
        pool.append([torch.from_numpy(np.roll(w.reshape(-1), s * 144)).to(dev) for w in ws])
    x_dev = [torch.from_numpy(x).to(dev) for x in xs]
    y_dev = [torch.empty(n, dtype=torch.float32, device=dev) for _, n in SHAPES]
    stream = torch.cuda.Stream(dev)

    def step(s: int):
        # one persistent launch runs the three independent matvecs
        ctx.matvec_program([(TYPE_Q4_K, n, k, pool[s % POOL_SETS][i], x_dev[i], y_dev[i], 0)
                            for i, (k, n) in enumerate(SHAPES)], stream=stream)

    def step_separate(s: int):
        for i, (k, n) in enumerate(SHAPES):
            ctx.storage_matvec(ob.CONTRACT_Q8K, TYPE_Q4_K, n, k, pool[s % POOL_SETS][i], x_dev[i], y_dev[i],
                               stream=stream)

    # correctness gate on this box: set 0 of every shape against the restatement
    with torch.cuda.stream(stream):
        step(0)
    stream.synchronize()
    ctx.device_status()
    import oracle
    port = oracle.port()
    wants = [port.matvec_q8_k(TYPE_Q4_K, n, k, ws[i], port.quantize_q8_k(xs[i]))[0]
             for i, (k, n) in enumerate(SHAPES)]
    for i in range(len(SHAPES)):
        if not np.array_equal(y_dev[i].cpu().numpy().view(np.uint32), wants[i].view(np.uint32)):
            raise SystemExit("GPU result differs from the restatement; refusing to report a number")
    want = wants[2]

    # graph of one pass over the pool (POOL_SETS steps)
    launches0 = ctx.launch_count()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        for s in range(POOL_SETS):
            step(s)
    stream.synchronize()
    with torch.cuda.graph(graph, stream=stream):
        for s in range(POOL_SETS):
            step(s)
    launches_per_step = (ctx.launch_count() - launches0) // (2 * POOL_SETS)
    # the remaining K mod POOL_SETS steps run from a second graph, so exactly K
    # steps are timed (and exactly W warmed up)
    rem = args.steps % POOL_SETS
    tail = None
    if rem:
        tail = torch.cuda.CUDAGraph()
        with torch.cuda.graph(tail, stream=stream):
            for s in range(rem):
                step(s)
    # graph replays go to the current stream: make that the capture stream,
    # so the events below bracket exactly the replayed kernels
    with torch.cuda.stream(stream):
        for _ in range(args.warmup // POOL_SETS):
            graph.replay()
        for s in range(args.warmup % POOL_SETS):
            step(s)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    with sampler, torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(args.steps // POOL_SETS):
            graph.replay()
        if tail is not None:
            tail.replay()
        end.record(stream)
        torch.cuda.synchronize()
    steps_timed = args.steps
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    ctx.device_status()
    value = world * steps_timed * STEP_BYTES / (ms / 1e3) / 1e9

    # the same step as three separate launches (one kernel per matvec)
    gsep = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gsep, stream=stream):
        for s in range(POOL_SETS):
            step_separate(s)
    with torch.cuda.stream(stream):
        gsep.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(20):
            gsep.replay()
        b.record(stream)
        torch.cuda.synchronize()
    sep_us = a.elapsed_time(b) * 1e3 / (20 * POOL_SETS)
    del gsep

    # per-shape launch durations, graphs of back-to-back single-matvec launches
    per_shape = []
    reps = 60
    for i, (k, n) in enumerate(SHAPES):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for r in range(reps):
                ctx.storage_matvec(ob.CONTRACT_Q8K, TYPE_Q4_K, n, k, pool[r % POOL_SETS][i], x_dev[i], y_dev[i],
                                   stream=stream)
        with torch.cuda.stream(stream):
            g.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(5):
                g.replay()
            b.record(stream)
            torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1e3 / (5 * reps)
        per_shape.append({"shape": f"{k}->{n}", "us_per_launch": us,
                          "gbs": algorithmic_bytes(k, n) / (us * 1e-6) / 1e9})
        del g
    # the timed region holds nothing but the program kernel (one launch per step)
    achieved = STEP_BYTES / (ms / steps_timed * 1e-3) / 1e9
    peak, peak_kind = load_peaks()

    # e2e through the host-pointer C ABI with pinned buffers
    x_pin = [torch.from_numpy(x).pin_memory() for x in xs]
    y_pin = [torch.empty(n, dtype=torch.float32).pin_memory() for _, n in SHAPES]
    x_np = [t.numpy() for t in x_pin]
    y_np = [t.numpy() for t in y_pin]

    def e2e_step():
        for i, (k, n) in enumerate(SHAPES):
            ctx.host_storage_matvec(ob.CONTRACT_Q8K, TYPE_Q4_K, n, k, ws[i], x_np[i], y_np[i])

    for _ in range(max(3, args.warmup // 100)):
        e2e_step()
    e2e_steps = max(10, min(args.steps, 2000))
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e_value = world * e2e_steps * STEP_BYTES / e2e_s / 1e9
    if not np.array_equal(y_np[2].view(np.uint32), want.view(np.uint32)):
        raise SystemExit("host-path result differs from the restatement")

    cpu = cpu_baseline_leg() if (rank == 0 and world == 1 and not args.no_cpu) else None
    traffic = load_traffic()
    if rank == 0:
        clocks = sampler.summary()
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps_timed,
                "warmup": args.warmup, "ms_per_step": ms / steps_timed, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "int8 x u4 -> int32, f32 combine",
                "data": "synthetic (seeded; BASELINE config-2 distributions)", "config": config_block(world),
                "gpu_launches": launches_per_step * steps_timed,
                "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": H2D_BYTES,
                        "d2h_bytes_per_step": D2H_BYTES,
                        "how": "oracle_cuda_host_storage_matvec (Q8_K contract) per shape, pinned host x/y, "
                               "wall clock over synchronous calls"},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                             "traffic": traffic, "kernel": "matvec_program_kernel (3 Q4_K x Q8_K ops per launch)",
                             "separate_launches": {"us_per_step": sep_us,
                                                   "gbs": STEP_BYTES / (sep_us * 1e-6) / 1e9},
                             "per_shape_single_launch": per_shape},
                "cpu_baseline": cpu, "clocks": clocks, "pdl": not args.no_pdl}
        print(json.dumps(line), flush=True)
    del graph, tail
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=12000)
    ap.add_argument("--warmup", type=int, default=600)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-pdl", action="store_true", help="launch without programmatic dependent launch")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args)
    else:
        gpu_arm(args)


if __name__ == "__main__":
    main()
