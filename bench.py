"""Benchmark of the north-star op: Q4_K x Q8_K decode matvec on B200.

Default workload (batch 1): one step = the three Q4_K
matvecs 4096->12288, 12288->4096 and 4096->4096, each quantizing its f32
activation to Q8_K in the call.  Algorithmic bytes per matvec = packed weight
bytes + f32 activation K*4 + f32 output N*4; 66,224,128 B per step.
--workload config3 (Q6_K LM head 4096->151936) and config1 (Q8_0 4096x4096,
Oracle's f32 contract) print the same line for those configurations.

* value   -- GB/s over the timed region: K steps replayed from a CUDA graph,
             CUDA events on the capture stream, barrier + synchronize on both
             sides, max over ranks.  A step is ONE launch of the persistent
             matvec-program kernel running the three independent matvecs
             (oracle_cuda_matvec_program).  Weights rotate through a pool of 10
             sets (661 MB, > 3x the 126 MB L2), so every step reads them from HBM.
* e2e     -- the same metric through the public host-pointer C ABI call
             (oracle_cuda_host_matvec_program, Q8_K contract) with pinned host
             x and y and registered weights (rotating over the same sets): each
             step copies x in, runs, copies y out, synchronises.
* roofline -- the program kernel (the only kernel in the timed region):
             algorithmic bytes / average launch time against MEASURED_PEAKS.json
             hbm_gbs; the same step as three separate single-matvec launches and
             each shape alone (graphs of back-to-back launches) are reported too.
* cpu_baseline -- the CPU restatement (oracle/, single thread) on a bounded
             row sample of the same matrices.

--impl reference times the CPU implementation of the path on all host
threads.  Oracle has no Q4_K decoder and no Q8_K integer dot (its storage
decoder rejects type 12), so that arm runs the C restatement of GGML's
algorithm (kind "port").  Multi-GPU (torchrun, one process per GPU): every
matrix is row-sharded over the ranks and each step ends with one NCCL
all-gather of the packed outputs (strong scaling: the whole job processes the
same matrices at every N; oracle_b200/shard.py).
--workload config4 times the prefill dequant-GEMM (TFLOP/s, tensor roofline).
--workload config5 times greedy decoding of the synthetic Qwen3.5-style hybrid
decoder (tokens/s; its tokens are checked against Oracle's own decode loop).
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
TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K = 8, 12, 14
CONTRACT_F32, CONTRACT_Q8K = 0, 1
UNIT = "GB/s"
BLOCK = {TYPE_Q8_0: (32, 34), TYPE_Q4_K: (256, 144), TYPE_Q6_K: (256, 210)}


def product_library_mapped() -> bool:
    """Whether this process has mapped the product library (liboracle_cuda.so).
    The reference arm must not: it times only the CPU implementation."""
    try:
        with open("/proc/self/maps") as f:
            return "liboracle_cuda.so" in f.read()
    except OSError:
        return False


def print_reference_line(line: dict) -> None:
    """The reference arm's JSON line, after checking that nothing of the
    product was loaded into this process."""
    mapped = product_library_mapped()
    if mapped:
        raise SystemExit("reference arm: liboracle_cuda.so is mapped into the reference process")
    line["product_library_mapped"] = mapped
    print(json.dumps(line), flush=True)


def weight_bytes(qtype: int, k: int, n: int) -> int:
    be, bb = BLOCK[qtype]
    return n * (k // be) * bb


def algorithmic_bytes(qtype: int, k: int, n: int) -> int:
    """Packed weight bytes + f32 activation read + f32 output written."""
    return weight_bytes(qtype, k, n) + k * 4 + n * 4


class Workload:
    """One step of a benchmark configuration: a list of matvecs (qtype, K, N)."""

    def __init__(self, name, metric, description, ops, contract, pool_sets, program, cpu_kind, dtype,
                 steps_per_launch=1):
        self.steps_per_launch = steps_per_launch
        self.name, self.metric, self.description = name, metric, description
        self.ops, self.contract, self.pool_sets, self.program = ops, contract, pool_sets, program
        self.cpu_kind, self.dtype = cpu_kind, dtype
        self.step_bytes = sum(algorithmic_bytes(t, k, n) for t, k, n in ops)
        self.h2d = sum(k * 4 for _, k, _ in ops)
        self.d2h = sum(n * 4 for _, _, n in ops)

    def config(self, n_gpus: int) -> dict:
        wb = sum(weight_bytes(t, k, n) for t, k, n in self.ops)
        return {"workload": self.description, "shapes_k_to_n": [f"{k}->{n}" for _, k, n in self.ops], "batch": 1,
                "bytes_per_step": self.step_bytes,
                "l2": f"weights rotate through {self.pool_sets} sets ({self.pool_sets * wb / 1e6:.0f} MB > 3x L2)",
                "parallelism": (f"tp{n_gpus}: rows sharded over {n_gpus} GPUs, outputs all-gathered every step "
                                "(inside the matvec kernel over NVLink, or one NCCL all-gather with --exchange nccl)"
                                if n_gpus > 1 else "single")}


WORKLOADS = {
    "config2": Workload(
        "config2", "Q4_K x Q8_K decode matvec GB/s",
        "config2: Q4_K x Q8_K decode matvec, batch 1, shapes 4096->12288, 12288->4096, 4096->4096 "
        "(each step's activations quantized to Q8_K in the launch); one GPU: one launch per matvec, "
        "chained by programmatic dependent launch (the one-launch matvec program is timed beside it); "
        "several GPUs: one matvec-program launch per step with the all-gather inside the kernel",
        [(TYPE_Q4_K, 4096, 12288), (TYPE_Q4_K, 12288, 4096), (TYPE_Q4_K, 4096, 4096)], CONTRACT_Q8K, 10, True,
        "port", "int8 x u4 -> int32, f32 combine", steps_per_launch=1),
    "config3": Workload(
        "config3", "Q6_K x Q8_K LM-head matvec GB/s",
        "config3: Q6_K x Q8_K LM-head matvec 4096->151936, batch 1", [(TYPE_Q6_K, 4096, 151936)], CONTRACT_Q8K, 2,
        False, "port", "int8 x u6 -> int32, f32 combine"),
    "config1": Workload(
        "config1", "Q8_0 f32-contract matvec GB/s",
        "config1: Q8_0 4096x4096 dequant-matvec against f32 x, Oracle's sequential f32 sum (bit-identical)",
        [(TYPE_Q8_0, 4096, 4096)], CONTRACT_F32, 8, False, "reference", "f32"),
}


class GemmWorkload:
    """prefill dequant-GEMMs Y = X . dequant(W)^T on the
    tensor cores; a step is one GEMM per (K, N) shape at M tokens."""

    name = "config4"
    metric = "Q4_K prefill dequant-GEMM TFLOP/s"
    unit = "TFLOP/s"
    dtype = "bf16 x bf16 -> f32 (tcgen05)"
    pool_sets = 3

    def __init__(self, m: int = 512, shapes=((4096, 12288), (12288, 4096)), extra_m=(2048,)):
        self.m, self.shapes, self.extra_m = m, list(shapes), list(extra_m)
        self.step_flops = sum(2 * m * k * n for k, n in self.shapes)
        self.h2d = sum(m * k * 4 for k, _ in self.shapes)
        self.d2h = sum(m * n * 4 for _, n in self.shapes)
        self.description = (f"config4: Q4_K prefill dequant-GEMM, M={m} tokens x (4096->12288, 12288->4096); W "
                            "tiles dequantized to bf16 in shared memory, X rounded to bf16, f32 accumulation in TMEM")

    def config(self, n_gpus: int) -> dict:
        wb = sum(weight_bytes(TYPE_Q4_K, k, n) for k, n in self.shapes)
        return {"workload": self.description, "m_tokens": self.m,
                "shapes_k_to_n": [f"{k}->{n}" for k, n in self.shapes], "flops_per_step": self.step_flops,
                "l2": f"weights rotate through {self.pool_sets} sets ({self.pool_sets * wb / 1e6:.0f} MB > L2)",
                "parallelism": f"replicas{n_gpus}" if n_gpus > 1 else "single"}


def load_peaks() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_tensor_peak() -> tuple[float, str]:
    """Dense bf16 TFLOP/s: the sustained figure (the timed loop runs for
    seconds under the power cap), else the fallback."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops_sustained"]), "measured bf16_tflops_sustained"
    except Exception:
        return 1400.0, "fallback sustained"


def load_traffic(wl: Workload):
    """DRAM bytes per step of the dominant kernel from the committed ncu capture."""
    path = os.path.join(ROOT, "profiles", f"{wl.name}_traffic.json")
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

def synth_activation(wl: Workload, k: int, slot: int) -> np.ndarray:
    """Activation of width k for step slot `slot` > 0 of a launch (seeded, N(0,1))."""
    from oracle_b200 import synth
    return synth.activations(k, 1, wl.name, f"x_{k}_slot{slot}")[0]


def host_weights(wl: Workload):
    from oracle_b200 import synth
    ws = [synth.weight(t, n, k, wl.name, f"W_{k}_{n}") for t, k, n in wl.ops]
    xs = [synth.activations(k, 1, wl.name, f"x_{k}")[0] for _, k, _ in wl.ops]
    return ws, xs


def time_cpu(wl: Workload, ws, xs, fraction: float, threads: int) -> tuple[float, int]:
    """Run `fraction` of every matrix's rows of one step on `threads` host
    threads with the CPU implementation (ctypes releases the GIL).  config2/3:
    the C restatement's Q8_K quantize + integer dot; config1: the reference's
    own compiled reference_storage_matvec.  Returns (seconds, bytes)."""
    import oracle
    port = oracle.port()
    ref = oracle.ref() if wl.cpu_kind == "reference" else None
    jobs, total = [], 0
    for (t, k, n), w, x in zip(wl.ops, ws, xs):
        rows = max(1, int(n * fraction))
        total += weight_bytes(t, k, rows) + k * 4 + rows * 4
        jobs.append((t, k, rows, w, x))

    def work(t, k, lo, hi, w, xin):
        if ref is not None:
            ref.storage_matvec(t, hi - lo, k, w[lo:hi], xin)
        else:
            port.matvec_q8_k(t, hi - lo, k, w[lo:hi], xin)

    t0 = time.perf_counter()
    for t, k, rows, w, x in jobs:
        xin = x if ref is not None else port.quantize_q8_k(x)
        bounds = np.linspace(0, rows, threads + 1).astype(int)
        th = [threading.Thread(target=work, args=(t, k, bounds[i], bounds[i + 1], w, xin))
              for i in range(threads) if bounds[i + 1] > bounds[i]]
        for h in th:
            h.start()
        for h in th:
            h.join()
    return time.perf_counter() - t0, total


def cpu_what(wl: Workload) -> str:
    if wl.cpu_kind == "reference":
        return "Oracle's own reference_storage_matvec compiled from the reference sources (oracle/_ref)"
    return ("the C restatement of GGML's Q8_K quantize + integer dot (oracle/quant_oracle.c); Oracle has no "
            "Q4_K decoder and no Q8_K dot (storage_decode.cpp:192-196 rejects type 12)")


def cpu_baseline_leg(wl: Workload, target_seconds: float = 10.0) -> dict:
    """One core, a bounded row sample of the step, about target_seconds."""
    ws, xs = host_weights(wl)
    dt, _ = time_cpu(wl, ws, xs, 0.02, 1)
    fraction = min(1.0, 0.02 * (target_seconds / 4) / max(dt, 1e-4))
    total_t, total_b, reps = 0.0, 0, 0
    while total_t < target_seconds and reps < 1000:
        dt, nb = time_cpu(wl, ws, xs, fraction, 1)
        total_t += dt
        total_b += nb
        reps += 1
    return {"value": total_b / total_t / 1e9, "unit": UNIT, "cores": 1, "kind": wl.cpu_kind,
            "sample": f"{fraction * 100:.1f}% of the rows of every {wl.name} matrix x {reps} repetitions "
                      f"({total_b / 1e6:.0f} MB in {total_t:.1f} s, single thread): {cpu_what(wl)}"}


def reference_arm(args, wl: Workload) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and rank != 0:
        return
    threads = os.cpu_count() or 1
    ws, xs = host_weights(wl)
    dt, _ = time_cpu(wl, ws, xs, 0.05, threads)
    # one step is a bounded sample: about 0.5 s on all threads, less when
    # many steps are asked for, so that the whole run stays near two minutes
    per_step = min(0.5, 120.0 / max(1, args.steps + args.warmup))
    fraction = min(1.0, max(1e-4, 0.05 * per_step / max(dt, 1e-4)))
    for _ in range(args.warmup):
        time_cpu(wl, ws, xs, fraction, threads)
    total_t, total_b = 0.0, 0
    for _ in range(args.steps):
        dt, nb = time_cpu(wl, ws, xs, fraction, threads)
        total_t += dt
        total_b += nb
    value = total_b / total_t / 1e9
    sample = f"{fraction * 100:.2f}% of the rows of every {wl.name} matrix per step on {threads} threads: {cpu_what(wl)}"
    line = {"impl": "reference", "metric": wl.metric, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_t / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": wl.dtype,
            "data": "synthetic", "config": wl.config(args.gpus),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": wl.cpu_kind, "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print_reference_line(line)


# ---------------------------------------------------------------- GPU arm

def gpu_arm(args, wl: Workload) -> None:
    import torch

    import oracle_b200 as ob

    rank, local, world = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ctx = ob.Context(local, flags=ob.FLAG_PDL if not args.no_pdl else 0)
    ws, xs = host_weights(wl)
    # N > 1: every matrix is row-sharded (rank r owns an equal contiguous row
    # range); each step ends with ONE NCCL all-gather of the packed per-rank
    # outputs, after which every rank holds every output (oracle_b200/shard.py)
    from oracle_b200.shard import PackPlan
    plan = PackPlan([n for _, _, n in wl.ops], world, rank)
    local_ops = [(t, k, sh.local_rows) for (t, k, _), sh in zip(wl.ops, plan.shards)]
    # weight pool: set 0 is the seeded host weights; the others are rotations
    # by whole blocks (same distribution, distinct addresses), so no step finds
    # its weights in L2
    # (set s = this rank's rows of the full matrix rolled by s blocks, so every
    # set is a whole matrix the CPU checker can reproduce at any rank count)
    pool = []
    for s in range(wl.pool_sets):
        pool.append([torch.from_numpy(np.ascontiguousarray(
            sh.weight_slice(np.roll(w.reshape(-1), s * BLOCK[t][1]).reshape(w.shape)))).to(dev)
            for w, sh, (t, _, _) in zip(ws, plan.shards, wl.ops)])
    # P steps per launch: step slot p of a launch has its own activations
    # (slot 0: the seeded ones) and its own outputs
    P = wl.steps_per_launch
    xs_sets = [xs] + [[synth_activation(wl, k, p) for _, k, _ in wl.ops] for p in range(1, P)]
    x_sets = [[torch.from_numpy(x).to(dev) for x in xset] for xset in xs_sets]
    x_dev = x_sets[0]
    # N > 1, Q8_K contract: the all-gather is fused into the matvec program
    # (rows stored into every peer's gather buffer over NVLink, CUDA IPC);
    # --exchange nccl (or the f32 contract) uses one NCCL all-gather instead
    fused = world > 1 and args.exchange == "fused" and wl.contract == CONTRACT_Q8K
    group = None
    if fused:
        import torch.distributed as dist
        group = ob.PeerGroup(ctx, rank, world, (P * world * plan.pack_len * 4 + 15) // 16 * 16)
        handles = [None] * world
        dist.all_gather_object(handles, group.handle)
        group.connect(handles)
        region = group.tensor()
        gathered_sets = [region[p * world * plan.pack_len:(p + 1) * world * plan.pack_len] for p in range(P)]
        y_packs = [g[rank * plan.pack_len:(rank + 1) * plan.pack_len] for g in gathered_sets]
    else:
        y_packs = [torch.empty(plan.pack_len, dtype=torch.float32, device=dev) for _ in range(P)]
        gathered_sets = [torch.empty(world * plan.pack_len, dtype=torch.float32, device=dev) if world > 1 else None
                         for _ in range(P)]
    gathered, y_pack = gathered_sets[0], y_packs[0]
    y_sets = [[yp[o:o + sh.local_rows] for o, sh in zip(plan.offsets, plan.shards)] for yp in y_packs]
    y_dev = y_sets[0]
    stream = torch.cuda.Stream(dev)

    def exchange():
        if world > 1 and not fused:
            import torch.distributed as dist
            dist.all_gather_into_tensor(gathered, y_pack)

    def launch(s0: int, count: int):
        """Steps s0 .. s0+count-1 (count <= P): with a program, ONE persistent
        launch runs all their (independent) matvecs back to back."""
        # one GPU: one single-matvec launch per op (programmatic dependent launch
        # chains them); the matvec program, which runs them in one persistent
        # launch, is timed beside it.  Several GPUs: the program (its all-gather
        # runs inside the kernel) or, with --exchange nccl, the program + NCCL
        if not (fused or (wl.program and world > 1)):
            for s in range(s0, s0 + count):
                step_separate(s)
            return
        ops_ = []
        for s in range(s0, s0 + count):
            ws_, p = pool[s % wl.pool_sets], s % P
            ops_ += [(t, n, k, ws_[i], x_sets[p][i], y_sets[p][i], 0) for i, (t, k, n) in enumerate(local_ops)]
        if fused:
            ctx.matvec_program_allgather(group, ops_, stream=stream)
        else:
            ctx.matvec_program(ops_, stream=stream)
            if world > 1:
                import torch.distributed as dist
                for p in sorted({s % P for s in range(s0, s0 + count)}):
                    dist.all_gather_into_tensor(gathered_sets[p], y_packs[p])

    def steps(s0: int, count: int):
        for a in range(s0, s0 + count, P):
            launch(a, min(P, s0 + count - a))

    def step_separate(s: int):
        ws_ = pool[s % wl.pool_sets]
        for i, (t, k, n) in enumerate(local_ops):
            ctx.storage_matvec(wl.contract, t, n, k, ws_[i], x_dev[i], y_dev[i], stream=stream)
        exchange()

    def outputs(p: int = 0) -> list:
        if world > 1:
            return plan.unpack(gathered_sets[p].cpu().numpy())
        return [y.cpu().numpy() for y in y_sets[p]]

    # correctness gate on this box: the first launch (steps 0 .. P-1, weight
    # sets 0 .. P-1, activation slots 0 .. P-1), every op against the CPU checker
    with torch.cuda.stream(stream):
        steps(0, P)
    stream.synchronize()
    ctx.device_status()
    import oracle
    port = oracle.port()
    wants = []
    for p in range(P):
        got = outputs(p)
        for i, (t, k, n) in enumerate(wl.ops):
            w_host = np.roll(ws[i].reshape(-1), p * BLOCK[t][1]).reshape(ws[i].shape) if p % wl.pool_sets else ws[i]
            x_host = xs_sets[p][i]
            if wl.contract == CONTRACT_Q8K:
                want = port.matvec_q8_k(t, n, k, w_host, port.quantize_q8_k(x_host))[0]
            else:
                want = port.storage_matvec_f32(t, n, k, w_host, x_host)[0]
            if p == 0:
                wants.append(want)
            if not np.array_equal(got[i].view(np.uint32), want.view(np.uint32)):
                raise SystemExit("GPU result differs from the CPU checker; refusing to report a number")

    # graph of one pass over the pool (pool_sets steps); K mod pool_sets more from a tail graph
    launches0 = ctx.launch_count()
    with torch.cuda.stream(stream):
        steps(0, wl.pool_sets)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        steps(0, wl.pool_sets)
    launches_per_pass = (ctx.launch_count() - launches0) / 2
    launches_per_step = launches_per_pass / wl.pool_sets
    rem = args.steps % wl.pool_sets
    tail = None
    if rem:
        tail = torch.cuda.CUDAGraph()
        with torch.cuda.graph(tail, stream=stream):
            steps(0, rem)
    # graph replays go to the current stream: make that the capture stream, so
    # the events below bracket exactly the replayed kernels
    with torch.cuda.stream(stream):
        for _ in range(args.warmup // wl.pool_sets):
            graph.replay()
        steps(0, args.warmup % wl.pool_sets)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    with sampler, torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(args.steps // wl.pool_sets):
            graph.replay()
        if tail is not None:
            tail.replay()
        end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    ctx.device_status()
    steps_timed = args.steps
    # whole-job bytes: the full matrices, whatever the rank count (strong scaling)
    value = steps_timed * wl.step_bytes / (ms / 1e3) / 1e9
    # the timed region holds nothing but the step's kernels (and, N > 1, the all-gather)
    achieved = wl.step_bytes / world / (ms / steps_timed * 1e-3) / 1e9
    peak, peak_kind = load_peaks()

    extra = {}
    if wl.program and world == 1:
        # the same step as ONE matvec-program launch (the three matvecs in one persistent kernel)
        def step_program(s: int):
            ws_, p = pool[s % wl.pool_sets], s % P
            ctx.matvec_program([(t, n, k, ws_[i], x_sets[p][i], y_sets[p][i], 0) for i, (t, k, n) in
                                enumerate(local_ops)], stream=stream)

        with torch.cuda.stream(stream):
            step_program(0)  # sizes the context's scratch outside the capture
        stream.synchronize()
        gsep = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gsep, stream=stream):
            for s in range(wl.pool_sets):
                step_program(s)
        with torch.cuda.stream(stream):
            gsep.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(20):
                gsep.replay()
            b.record(stream)
            torch.cuda.synchronize()
        sep_us = a.elapsed_time(b) * 1e3 / (20 * wl.pool_sets)
        extra["program_launch"] = {"us_per_step": sep_us, "gbs": wl.step_bytes / (sep_us * 1e-6) / 1e9}
        del gsep
        if P > 1:
            # the same steps, one program launch each
            g1 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g1, stream=stream):
                for s in range(wl.pool_sets):
                    launch(s, 1)
            with torch.cuda.stream(stream):
                g1.replay()
                torch.cuda.synchronize()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(20):
                    g1.replay()
                b.record(stream)
                torch.cuda.synchronize()
            one_us = a.elapsed_time(b) * 1e3 / (20 * wl.pool_sets)
            extra["one_step_per_launch"] = {"us_per_step": one_us, "gbs": wl.step_bytes / (one_us * 1e-6) / 1e9}
            del g1
        per_op = []
        reps = 60
        for i, (t, k, n) in enumerate(wl.ops):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for r in range(reps):
                    ctx.storage_matvec(wl.contract, t, n, k, pool[r % wl.pool_sets][i], x_dev[i], y_dev[i],
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
            per_op.append({"shape": f"{k}->{n}", "us_per_launch": us, "gbs": algorithmic_bytes(t, k, n) / (us * 1e-6) / 1e9})
            del g
        extra["per_shape_single_launch"] = per_op

    # e2e: N = 1 through the host-pointer C ABI (the drop-in call) with pinned
    # buffers; N > 1 pinned x copied in on every rank, the sharded step with
    # its all-gather, the whole output copied out, synchronised every step
    x_pin = [torch.from_numpy(x).pin_memory() for x in xs]
    x_np = [t.numpy() for t in x_pin]
    if world == 1:
        y_pin = [torch.empty(n, dtype=torch.float32).pin_memory() for _, _, n in wl.ops]
        y_np = [t.numpy() for t in y_pin]

        # the weight sets (the device pool's host bytes: set s is every matrix
        # rolled by s blocks, so the step's weights do not sit in L2) are
        # registered once, as the adapter does for a mapped GGUF tensor
        # (immutable bytes): the calls then read their HBM copies
        ws_host = [[np.ascontiguousarray(np.roll(w.reshape(-1), s * BLOCK[t][1])) for w, (t, _, _) in zip(ws, wl.ops)]
                   for s in range(wl.pool_sets)]
        for wset in ws_host:
            for (t, k, n), w in zip(wl.ops, wset):
                ctx.register_host_weight(t, n, k, w)
        if wl.contract == CONTRACT_Q8K:
            host_steps = [ctx.prepare_host_program([(t, n, k, wset[i], x_np[i], y_np[i])
                                                    for i, (t, k, n) in enumerate(wl.ops)])
                          for wset in ws_host]

            def e2e_step(s=0):
                host_steps[s % wl.pool_sets]()

            e2e_how = ("oracle_cuda_host_program_run: the step's matvecs prepared once per weight set "
                       "(oracle_cuda_host_program_create, registered weights rotating over the pool's sets), each "
                       "call copying pinned host x in and y out around one launch and one synchronize; wall clock "
                       "over synchronous calls")
        else:
            def e2e_step(s=0):
                wset = ws_host[s % wl.pool_sets]
                for i, (t, k, n) in enumerate(wl.ops):
                    ctx.host_storage_matvec(wl.contract, t, n, k, wset[i], x_np[i], y_np[i])

            e2e_how = ("oracle_cuda_host_storage_matvec per matvec, pinned host x/y, registered weights rotating "
                       "over the pool's sets; wall clock over synchronous calls")
        e2e_d2h = wl.d2h
    else:
        g_pin = torch.empty(world * plan.pack_len, dtype=torch.float32).pin_memory()

        def e2e_step(s=0):
            with torch.cuda.stream(stream):
                for i in range(len(wl.ops)):
                    x_dev[i].copy_(x_pin[i], non_blocking=True)
                launch(s % wl.pool_sets, 1)
                g_pin.copy_(gathered, non_blocking=True)
            stream.synchronize()

        e2e_how = ("pinned x copied in on every rank, row-sharded step with its all-gather "
                   f"({'in the matvec kernel' if fused else 'NCCL'}), every rank copies the whole output out, "
                   "synchronised each step; wall clock, max over ranks")
        e2e_d2h = world * plan.pack_len * 4

    for _ in range(3):
        e2e_step()
    e2e_steps = max(10, min(args.steps, 2000))
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for s in range(e2e_steps):
        e2e_step(s)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e_value = e2e_steps * wl.step_bytes / e2e_s / 1e9
    e2e_step(0)  # the checked result: weight set 0, the seeded weights
    e2e_out = [y_np[i] for i in range(len(wl.ops))] if world == 1 else plan.unpack(g_pin.numpy())
    for i in range(len(wl.ops)):
        if not np.array_equal(e2e_out[i].view(np.uint32), wants[i].view(np.uint32)):
            raise SystemExit("end-to-end result differs from the CPU checker")

    cpu = cpu_baseline_leg(wl) if (rank == 0 and world == 1 and not args.no_cpu) else None
    if rank == 0:
        kernel = ("matvec_program_kernel" if wl.program and world > 1 else
                  "matvec_q80_split_kernel (lane per row, sequential f32)" if wl.contract == CONTRACT_F32 else
                  "stream_rows_kernel<MatvecQ8KConsumer>")
        line = {"metric": wl.metric, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps_timed,
                "warmup": args.warmup, "ms_per_step": ms / steps_timed, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": wl.dtype,
                "data": f"synthetic (seeded; BASELINE {wl.name} distributions)", "config": wl.config(world),
                "gpu_launches": int(round(launches_per_step * steps_timed)),
                "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": e2e_d2h,
                        "how": e2e_how},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                             "traffic": load_traffic(wl), "kernel": kernel, **extra},
                "cpu_baseline": cpu, "clocks": sampler.summary(), "pdl": not args.no_pdl,
                "exchange": ("fused all-gather in the matvec kernel (NVLink stores to CUDA-IPC gather buffers)"
                             if fused else "NCCL all_gather_into_tensor" if world > 1 else None)}
        print(json.dumps(line), flush=True)
    del graph, tail
    torch.cuda.synchronize()
    barrier(world)  # no peer still writes into this rank's gather buffer
    if group is not None:
        group.close()
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ---------------------------------------------------------------- prefill GEMM (config 4)

def gemm_host(wl: GemmWorkload, m: int):
    from oracle_b200 import synth
    ws = [synth.weight(TYPE_Q4_K, n, k, "config4", f"W_{k}_{n}") for k, n in wl.shapes]
    xs = [synth.activations(k, m, "config4", f"X_{k}_{m}") for k, _ in wl.shapes]
    return ws, xs


def gemm_cpu(wl: GemmWorkload, ws, xs, samples: int, threads: int, seed: int) -> tuple[float, float]:
    """`samples` output elements of every shape by the C restatement (f32
    operands, f64 sums) on `threads` host threads; returns (seconds, flops)."""
    import oracle
    port = oracle.port()
    rng = np.random.default_rng(seed)
    jobs = []
    for (k, n), w, x in zip(wl.shapes, ws, xs):
        mi = rng.integers(0, x.shape[0], samples)
        ni = np.sort(rng.integers(0, n, samples))
        jobs.append((k, n, w, x, mi, ni))
    t0 = time.perf_counter()
    for k, n, w, x, mi, ni in jobs:
        parts = np.array_split(np.arange(samples), threads)
        th = [threading.Thread(target=port.gemm_sampled, args=(TYPE_Q4_K, n, k, w, x, mi[p], ni[p], 0))
              for p in parts if len(p)]
        for h in th:
            h.start()
        for h in th:
            h.join()
    return time.perf_counter() - t0, float(sum(2 * k * samples for k, _ in wl.shapes))


def gemm_cpu_baseline(wl: GemmWorkload, ws, xs, target_seconds: float = 10.0) -> dict:
    dt, fl = gemm_cpu(wl, ws, xs, 64, 1, 1)
    samples = max(64, int(64 * (target_seconds / 3) / max(dt, 1e-4)))
    total_t, total_f, reps = 0.0, 0.0, 0
    while total_t < target_seconds and reps < 100:
        dt, fl = gemm_cpu(wl, ws, xs, samples, 1, 2 + reps)
        total_t += dt
        total_f += fl
        reps += 1
    return {"value": total_f / total_t / 1e12, "unit": "TFLOP/s", "cores": 1, "kind": "port",
            "sample": f"{reps} x {samples} sampled output elements of each config4 shape (M={wl.m}), single "
                      "thread: the C restatement's f32-operand dot per element (oracle/quant_oracle.c "
                      "oq_gemm_sampled); Oracle has no prefill GEMM (it ingests prompts one matvec at a time)"}


def gemm_reference_arm(args, wl: GemmWorkload) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and rank != 0:
        return
    threads = os.cpu_count() or 1
    ws, xs = gemm_host(wl, wl.m)
    dt, _ = gemm_cpu(wl, ws, xs, 256 * threads, threads, 1)
    per_step = min(0.5, 120.0 / max(1, args.steps + args.warmup))
    samples = max(threads, int(256 * threads * per_step / max(dt, 1e-4)))
    for i in range(args.warmup):
        gemm_cpu(wl, ws, xs, samples, threads, 100 + i)
    total_t, total_f = 0.0, 0.0
    for i in range(args.steps):
        dt, fl = gemm_cpu(wl, ws, xs, samples, threads, 1000 + i)
        total_t += dt
        total_f += fl
    value = total_f / total_t / 1e12
    line = {"impl": "reference", "metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_t / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (CPU)",
            "data": "synthetic", "config": wl.config(args.gpus),
            "cpu_baseline": {"value": value, "unit": wl.unit, "cores": threads, "kind": "port",
                             "sample": f"{samples} sampled output elements per shape per step on {threads} threads"},
            "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print_reference_line(line)


def gemm_arm(args, wl: GemmWorkload) -> None:
    import torch

    import oracle
    import oracle_b200 as ob

    rank, local, world = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ctx = ob.Context(local)
    port = oracle.port()
    ws, xs = gemm_host(wl, wl.m)
    pool = [[torch.from_numpy(np.roll(w.reshape(-1), s * 144)).to(dev) for w in ws] for s in range(wl.pool_sets)]
    x_dev = [torch.from_numpy(x.reshape(-1)).to(dev) for x in xs]
    y_dev = [torch.empty(wl.m * n, dtype=torch.float32, device=dev) for _, n in wl.shapes]
    stream = torch.cuda.Stream(dev)

    def step(s: int):
        for i, (k, n) in enumerate(wl.shapes):
            ctx.prefill_gemm(TYPE_Q4_K, n, k, pool[s % wl.pool_sets][i], x_dev[i], wl.m, y_dev[i], stream=stream)

    def gate(ys, ws_, xs_, m):
        rng = np.random.default_rng(7)
        for (k, n), y, w, x in zip(wl.shapes, ys, ws_, xs_):
            mi, ni = rng.integers(0, m, 400), rng.integers(0, n, 400)
            ref = port.gemm_sampled(TYPE_Q4_K, n, k, w, x, mi, ni, 1)
            scale = port.gemm_sampled(TYPE_Q4_K, n, k, w, x, mi, ni, 2)
            got = y.cpu().numpy().reshape(m, n)[mi, ni]
            if not np.all(np.abs(got - ref) <= 1e-4 * scale + 1e-6):
                raise SystemExit("GPU GEMM differs from the CPU checker; refusing to report a number")

    with torch.cuda.stream(stream):
        step(0)
    stream.synchronize()
    ctx.device_status()
    gate(y_dev, ws, xs, wl.m)

    launches0 = ctx.launch_count()
    with torch.cuda.stream(stream):
        for s in range(wl.pool_sets):
            step(s)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for s in range(wl.pool_sets):
            step(s)
    launches_per_step = (ctx.launch_count() - launches0) // (2 * wl.pool_sets)
    rem = args.steps % wl.pool_sets
    tail = None
    if rem:
        tail = torch.cuda.CUDAGraph()
        with torch.cuda.graph(tail, stream=stream):
            for s in range(rem):
                step(s)
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup // wl.pool_sets)):
            graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    with sampler, torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(args.steps // wl.pool_sets):
            graph.replay()
        if tail is not None:
            tail.replay()
        end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    ctx.device_status()
    value = world * args.steps * wl.step_flops / (ms / 1e3) / 1e12
    achieved = wl.step_flops / (ms / args.steps * 1e-3) / 1e12
    peak, peak_kind = load_tensor_peak()

    # each shape alone, and at the larger token counts
    per_shape = []
    for m in [wl.m] + wl.extra_m:
        ws_m, xs_m = (ws, xs) if m == wl.m else gemm_host(wl, m)
        xm = [torch.from_numpy(x.reshape(-1)).to(dev) for x in xs_m]
        ym = [torch.empty(m * n, dtype=torch.float32, device=dev) for _, n in wl.shapes]
        for i, (k, n) in enumerate(wl.shapes):
            with torch.cuda.stream(stream):
                ctx.prefill_gemm(TYPE_Q4_K, n, k, pool[0][i], xm[i], m, ym[i], stream=stream)
            stream.synchronize()
            if m != wl.m:
                rng = np.random.default_rng(11)
                mi, ni = rng.integers(0, m, 200), rng.integers(0, n, 200)
                ref = port.gemm_sampled(TYPE_Q4_K, n, k, ws_m[i], xs_m[i], mi, ni, 1)
                scale = port.gemm_sampled(TYPE_Q4_K, n, k, ws_m[i], xs_m[i], mi, ni, 2)
                got = ym[i].cpu().numpy().reshape(m, n)[mi, ni]
                if not np.all(np.abs(got - ref) <= 1e-4 * scale + 1e-6):
                    raise SystemExit(f"GPU GEMM differs from the CPU checker at M={m}")
            reps = 3 * wl.pool_sets
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for r in range(reps):
                    ctx.prefill_gemm(TYPE_Q4_K, n, k, pool[r % wl.pool_sets][i], xm[i], m, ym[i], stream=stream)
            with torch.cuda.stream(stream):
                g.replay()
                torch.cuda.synchronize()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(10):
                    g.replay()
                b.record(stream)
                torch.cuda.synchronize()
            us = a.elapsed_time(b) * 1e3 / (10 * reps)
            per_shape.append({"m": m, "shape": f"{k}->{n}", "us": us,
                              "tflops": 2 * m * k * n / (us * 1e-6) / 1e12})
            del g
        del xm, ym

    # e2e: pinned host X in, GEMMs, host Y out, synchronous per step
    x_pin = [torch.from_numpy(x.reshape(-1)).pin_memory() for x in xs]
    y_pin = [torch.empty(wl.m * n, dtype=torch.float32).pin_memory() for _, n in wl.shapes]

    def e2e_step():
        for i, (k, n) in enumerate(wl.shapes):
            x_dev[i].copy_(x_pin[i], non_blocking=True)
            ctx.prefill_gemm(TYPE_Q4_K, n, k, pool[0][i], x_dev[i], wl.m, y_dev[i],
                             stream=torch.cuda.current_stream())
            y_pin[i].copy_(y_dev[i], non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for _ in range(3):
        e2e_step()
    e2e_steps = 50
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e_value = world * e2e_steps * wl.step_flops / e2e_s / 1e12
    gate([y.cuda() for y in y_pin], ws, xs, wl.m)

    cpu = gemm_cpu_baseline(wl, ws, xs) if (rank == 0 and world == 1 and not args.no_cpu) else None
    if rank == 0:
        line = {"metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": wl.dtype,
                "data": "synthetic (seeded; BASELINE config4 distributions)", "config": wl.config(world),
                "gpu_launches": launches_per_step * args.steps,
                "e2e": {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": wl.h2d,
                        "d2h_bytes_per_step": wl.d2h,
                        "how": "pinned host X copied in, oracle_cuda_prefill_gemm, Y copied out, synchronised "
                               "every step, weights resident"},
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                             "frac": achieved / peak, "peak_source": peak_kind, "traffic": load_traffic(wl),
                             "kernel": "gemm_q4k_bf16_kernel (+ convert_bf16_kernel, 1 per GEMM)",
                             "per_shape": per_shape},
                "cpu_baseline": cpu, "clocks": sampler.summary()}
        print(json.dumps(line), flush=True)
    del graph, tail
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ---------------------------------------------------------------- config 5: the hybrid decoder

class DecoderWorkload:
    """greedy decoding of the synthetic Qwen3.5-style hybrid
    model (oracle_b200/qwen35.py CONFIG5, Q4_K_M, 4.95 GB of weights) from a
    seeded 128-token prompt, batch 1.  A step is one decode token: one replay
    of the captured step graph (oracle_b200/decoder.py)."""
    name = "config5"
    metric = "batch-1 decode tokens/s (Qwen3.5-style hybrid, Q4_K_M)"
    unit = "tokens/s"
    prompt_len = 128
    n_new = 256
    dtype = "f32 activations, Q8_K x Q4_K/Q6_K integer dots"

    def __init__(self, batch: int = 1):
        from oracle_b200 import qwen35
        self.cfg = qwen35.CONFIG5
        self.specs = qwen35.tensor_specs(self.cfg)
        self.batch = batch
        if batch > 1:
            self.metric = f"batch-{batch} decode tokens/s (Qwen3.5-style hybrid, Q4_K_M)"

    def config(self, n_gpus: int) -> dict:
        c = self.cfg
        return {"workload": "config5: synthetic Qwen3.5-style hybrid decoder, 32 blocks (24 Gated DeltaNet + 8 "
                            "gated GQA attention), hidden 4096, FFN 12288, vocab 151936, Q4_K_M, greedy",
                "batch": self.batch, "prompt_tokens": self.prompt_len, "new_tokens": self.n_new,
                "kv_capacity": c.context,
                "contract": "q8k",
                "parallelism": "single GPU" if n_gpus == 1 else
                f"tp{n_gpus}: heads sharded (Gated DeltaNet value heads, attention query heads, FFN columns, "
                f"vocabulary rows per GPU); output projection and ffn_down as canonical-order partial sums "
                f"exchanged over NVLink inside the matvec programs, 2 cross-GPU dependencies per block",
                "l2": "no flush needed: each step streams 4.7 GB of weights (> 37x the 126 MB L2)"}

    def step_bytes(self, position: int, batch: int = 1) -> int:
        """Algorithmic HBM bytes of one decode step at a cache length: every
        projection's packed weights (once, whatever the batch), one embedding
        row per sequence, and per sequence each recurrent state read and
        written once, the conv histories, and the KV rows read by attention."""
        from oracle_b200 import qwen35
        c = self.cfg
        total = 0
        for name, qtype, dims, _, _ in self.specs:
            be, bb = qwen35.BLOCK[qtype]
            n = int(np.prod(dims)) // be * bb
            if name == "token_embd.weight":
                n = n // dims[1] * batch
            total += n
        recurrent = sum(not c.is_attention(i) for i in range(c.layers))
        attention = c.layers - recurrent
        per_seq = recurrent * (2 * c.value_heads * c.state_size * c.state_size * 4 + 2 * c.conv_channels * 4 * 4)
        per_seq += attention * (position + 1) * 2 * c.kv_width * 4
        return total + batch * per_seq


def decoder_host_model(wl: DecoderWorkload):
    from oracle_b200 import qwen35
    tensors = qwen35.synthetic_model(wl.cfg, "q4_k_m", "config5")
    rng = np.random.default_rng(5150)
    prompt = rng.integers(0, wl.cfg.vocab, wl.prompt_len).astype(np.uint32)
    return tensors, prompt


def decoder_cpu_leg(wl: DecoderWorkload, tensors, prompt, n_prompt: int = 2, n_new: int = 2):
    """Oracle's decode loop (oracle/ref_qwen35.cpp, Q8_K checker build) on the
    same model: greedy tokens for a short prompt, and its speed."""
    import oracle
    r = oracle.Qwen35Reference("q8k", tensors=tensors, manifest=wl.cfg.manifest(), admit_q4k=True,
                               max_tokens=n_prompt + n_new + 1)
    t0 = time.perf_counter()
    toks = r.greedy(prompt[:n_prompt], n_new)
    s = time.perf_counter() - t0
    forwards = n_prompt + n_new - 1
    r.close()
    return toks, forwards / s, forwards, s


def decoder_reference_arm(args, wl: DecoderWorkload) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    tensors, prompt = decoder_host_model(wl)
    forwards = max(2, min(args.steps, 4))
    _, tps, n, s = decoder_cpu_leg(wl, tensors, prompt, n_prompt=1, n_new=forwards)
    cpu = {"value": tps, "unit": wl.unit, "cores": 1, "kind": "reference",
           "sample": f"{n} decode steps of the full config-5 model from a 1-token prompt",
           "note": "Oracle's execute_qwen35_reference_token + greedy Sampler compiled from its sources "
                   "(single-threaded); Q4_K/Q6_K projections through the C restatement of GGML's Q8_K dot, "
                   "since Oracle's own decoder rejects Q4_K"}
    line = {"impl": "reference", "metric": wl.metric, "value": tps, "unit": wl.unit, "n_gpus": args.gpus,
            "steps": n, "warmup": 0, "ms_per_step": s * 1e3 / n, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded Q4_K_M weights)",
            "config": wl.config(1), "cpu_baseline": cpu,
            "e2e": {"value": tps, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print_reference_line(line)


def batch_prompts(wl: DecoderWorkload, prompt: np.ndarray) -> np.ndarray:
    """Sequence 0 gets the batch-1 prompt; sequence b > 0 a prompt seeded 5150 + b."""
    rows = [prompt] + [np.random.default_rng(5150 + b).integers(0, wl.cfg.vocab, wl.prompt_len).astype(np.uint32)
                       for b in range(1, wl.batch)]
    return np.stack(rows)


def decoder_batch_arm(args, wl: DecoderWorkload) -> None:
    """Batched decoding (oracle_b200/batch_decoder.py): B sequences in lockstep,
    every projection's weights streamed once per step for all of them."""
    import torch

    import oracle_b200 as ob
    from oracle_b200.batch_decoder import BatchDecoder

    if args.gpus != 1:
        raise SystemExit("batched decoding runs on one GPU (replicas for more)")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ctx = ob.Context(0)
    tensors, prompt = decoder_host_model(wl)
    prompts = batch_prompts(wl, prompt)
    B = wl.batch
    max_new = max(wl.n_new, args.warmup + args.steps + 1)
    if wl.prompt_len + max_new > wl.cfg.context:
        raise SystemExit("warm-up + timed steps exceed the KV cache capacity")
    dec = BatchDecoder(ctx, wl.cfg, tensors, B, capacity=wl.cfg.context, max_new=max_new)

    # gate: sequence 0's greedy tokens on a short prompt equal Oracle's decode loop's
    cpu = None
    if not args.no_cpu:
        want, tps, n, s = decoder_cpu_leg(wl, tensors, prompt)
        got = dec.generate(prompts[:, :2], 2)
        if not np.array_equal(got[0], want):
            raise SystemExit(f"GPU tokens {got[0].tolist()} differ from the CPU reference {want.tolist()}")
        cpu = {"value": tps, "unit": "tokens/s", "cores": 1, "kind": "reference",
               "sample": f"{n} decode steps (2-token prompt, 2 new tokens) of the full config-5 model, one sequence",
               "note": "Oracle's execute_qwen35_reference_token + greedy Sampler compiled from its sources "
                       "(single-threaded, one sequence per call: a batch costs B times this); tokens identical "
                       "to the GPU's sequence 0"}

    dec.start(prompts)
    launches = dec.launches_per_step()
    dec.start(prompts)
    with torch.cuda.stream(dec.stream):
        for _ in range(wl.prompt_len + args.warmup):
            dec.graph.replay()
    dec.stream.synchronize()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(0)
    with sampler, torch.cuda.stream(dec.stream):
        start.record(dec.stream)
        for _ in range(args.steps):
            dec.graph.replay()
        end.record(dec.stream)
        dec.stream.synchronize()
    ms = start.elapsed_time(end)
    ctx.device_status()
    value = B * args.steps / (ms / 1e3)
    ms_step = ms / args.steps
    mid = wl.prompt_len + args.warmup + args.steps // 2
    step_bytes = wl.step_bytes(mid, B)
    peak, peak_kind = load_peaks()
    dec.start(prompts)
    with torch.cuda.stream(dec.stream):
        for _ in range(wl.prompt_len):
            dec.graph.replay()
    proj_bytes, proj_ms, _ = dec.profile_projections()
    proj_gbs = proj_bytes / (proj_ms * 1e-3) / 1e9

    # e2e: B host prompts in, BatchDecoder.generate, B x n_new host tokens out
    dec.generate(prompts, 8)
    t0 = time.perf_counter()
    toks = dec.generate(prompts, wl.n_new)
    e2e_s = time.perf_counter() - t0
    forwards = wl.prompt_len + wl.n_new - 1
    line = {"metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded Q4_K_M weights and prompts)",
            "config": wl.config(1), "gpu_launches": launches * args.steps,
            "e2e": {"value": B * wl.n_new / e2e_s, "unit": wl.unit, "h2d_bytes_per_step": 4 * B,
                    "d2h_bytes_per_step": 4 * B,
                    "how": f"BatchDecoder.generate: {B} host prompts of {wl.prompt_len} tokens in, {B} x {wl.n_new} "
                           f"greedy tokens out ({forwards} graph replays); value = generated tokens / wall time",
                    "first_tokens_seq0": toks[0, :8].tolist()},
            "roofline": {"bound": "hbm", "achieved": proj_gbs, "peak": peak, "unit": "GB/s",
                         "frac": proj_gbs / peak, "peak_source": peak_kind, "traffic": None,
                         "kernel": "matvec_batch_kernel (the step's batched projections, one uncaptured step timed "
                                   "with CUDA events around each call)",
                         "projection_ms_per_step": proj_ms, "projection_bytes_per_step": proj_bytes,
                         "step_bytes": step_bytes, "step_achieved": step_bytes / (ms_step * 1e-3) / 1e9,
                         "step_frac": step_bytes / (ms_step * 1e-3) / 1e9 / peak, "launches_per_step": launches},
            "cpu_baseline": cpu, "clocks": sampler.summary()}
    print(json.dumps(line), flush=True)
    dec.close()
    del dec
    ctx.close()


def decoder_arm(args, wl: DecoderWorkload) -> None:
    import torch

    import oracle_b200 as ob
    from oracle_b200.decoder import Qwen35Decoder

    rank, local, world = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ctx = ob.Context(local)
    tensors, prompt = decoder_host_model(wl)
    max_new = max(wl.n_new, args.warmup + args.steps + 1)

    def exchange(handle):
        import torch.distributed as dist
        hs = [None] * world
        dist.all_gather_object(hs, handle)
        return hs

    # several GPUs: heads sharded (each rank its own heads, FFN columns and
    # vocabulary rows; partial sums exchanged inside the matvec programs); the
    # job decodes ONE sequence
    if world > 1:
        from oracle_b200.tp_decoder import HeadShardedDecoder
        dec = HeadShardedDecoder(ctx, wl.cfg, tensors, rank, world, exchange, capacity=wl.cfg.context,
                                 max_new=max_new, device=local)
    else:
        dec = Qwen35Decoder(ctx, wl.cfg, tensors, contract="q8k", capacity=wl.cfg.context, max_new=max_new,
                            device=local)
    if wl.prompt_len + max_new > wl.cfg.context:
        raise SystemExit("warm-up + timed steps exceed the KV cache capacity")

    # gate: the GPU's greedy tokens on a short prompt equal Oracle's decode loop's
    cpu, want = None, None
    if rank == 0 and not args.no_cpu:
        want, tps, n, s = decoder_cpu_leg(wl, tensors, prompt)
        cpu = {"value": tps, "unit": wl.unit, "cores": 1, "kind": "reference",
               "sample": f"{n} decode steps (2-token prompt, 2 new tokens) of the full config-5 model",
               "note": "Oracle's execute_qwen35_reference_token + greedy Sampler compiled from its sources "
                       "(single-threaded); Q4_K/Q6_K projections through the C restatement of GGML's Q8_K "
                       "dot, since Oracle's own decoder rejects Q4_K; tokens identical to the GPU's"}
    if not args.no_cpu:
        barrier(world)  # rank 0 ran the CPU leg: every rank's first step starts together
        got = dec.generate(prompt[:2], 2)
        if rank == 0 and not np.array_equal(got, want):
            raise SystemExit(f"GPU tokens {got.tolist()} differ from the CPU reference {want.tolist()}")
        barrier(world)

    # timed region: decode steps after the 128-token prompt
    dec.start(prompt)
    launches = dec.launches_per_step()
    dec.start(prompt)
    with torch.cuda.stream(dec.stream):
        for _ in range(wl.prompt_len + args.warmup):
            dec.graph.replay()
    dec.stream.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    with sampler, torch.cuda.stream(dec.stream):
        start.record(dec.stream)
        for _ in range(args.steps):
            dec.graph.replay()
        end.record(dec.stream)
        dec.stream.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    ctx.device_status()
    value = args.steps / (ms / 1e3)  # one sequence, whatever the number of GPUs
    mid = wl.prompt_len + args.warmup + args.steps // 2
    step_bytes = wl.step_bytes(mid)
    peak, peak_kind = load_peaks()
    ms_step = ms / args.steps

    # the matvec programs' share: one uncaptured step with events around each projection call
    dec.start(prompt)
    with torch.cuda.stream(dec.stream):
        for _ in range(wl.prompt_len):
            dec.graph.replay()
    proj_bytes, proj_ms, _ = dec.profile_projections()
    proj_gbs = proj_bytes / (proj_ms * 1e-3) / 1e9  # this rank's weight bytes (1/N of the model)

    # e2e: host prompt in, Qwen35Decoder.generate, host tokens out
    dec.generate(prompt, 8)
    barrier(world)
    t0 = time.perf_counter()
    toks = dec.generate(prompt, wl.n_new)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    forwards = wl.prompt_len + wl.n_new - 1
    if rank == 0:
        line = {"metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded Q4_K_M weights and prompt)",
                "config": wl.config(world), "gpu_launches": launches * args.steps,
                "e2e": {"value": wl.n_new / e2e_s, "unit": wl.unit, "h2d_bytes_per_step": 4,
                        "d2h_bytes_per_step": 4,
                        "how": f"{type(dec).__name__}.generate: 128-token host prompt in, {wl.n_new} greedy tokens out "
                               f"({forwards} graph replays, prompt ingested token by token as Oracle does); "
                               f"value = generated tokens / wall time",
                        "forward_steps_per_s": forwards / e2e_s, "first_tokens": toks[:8].tolist()},
                "roofline": {"bound": "hbm", "achieved": proj_gbs, "peak": peak, "unit": "GB/s",
                             "frac": proj_gbs / peak, "peak_source": peak_kind, "traffic": None,
                             "kernel": "matvec_program_kernel (the step's projections, one uncaptured step "
                                       "timed with CUDA events around each program call)",
                             "projection_ms_per_step": proj_ms, "projection_bytes_per_step": proj_bytes,
                             "step_bytes": step_bytes, "step_achieved": step_bytes / world / (ms_step * 1e-3) / 1e9,
                             "step_frac": step_bytes / world / (ms_step * 1e-3) / 1e9 / peak,
                             "launches_per_step": launches},
                "cpu_baseline": cpu, "clocks": sampler.summary()}
        print(json.dumps(line), flush=True)
    barrier(world)
    dec.close()
    del dec
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
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["config4", "config5"], default="config2")
    ap.add_argument("--no-pdl", action="store_true", help="launch without programmatic dependent launch")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--batch", type=int, default=1, help="config5: sequences decoded together (1..16)")
    ap.add_argument("--exchange", choices=["fused", "nccl"], default="fused",
                    help="N > 1: all-gather inside the matvec kernel (fused) or one NCCL all-gather per step")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "config5":
        wl5 = DecoderWorkload(args.batch)
        if args.impl == "reference":
            decoder_reference_arm(args, wl5)
        else:
            (decoder_batch_arm if args.batch > 1 else decoder_arm)(args, wl5)
        return
    if args.workload == "config4":
        wl = GemmWorkload()
        (gemm_reference_arm if args.impl == "reference" else gemm_arm)(args, wl)
        return
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        reference_arm(args, wl)
    else:
        gpu_arm(args, wl)


if __name__ == "__main__":
    main()
