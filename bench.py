"""Benchmark of the Pearl mining hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the headline configuration): one mined int8 noisy GEMM,
M = N = K = 8192, R = 128, seeded int7 operands, int32 accumulation, fused
transcript hashing, keyed BLAKE3 and a difficulty check whose target yields
~1e-6 hits per hash tile.  One step = noise_gen + the noising of both
operands (noise_A and noise_B in one launch, as noisy_gemm(run_noising_A/B=
True) runs it) + the mined GEMM (transcript, BLAKE3, target compare,
denoise, bf16 C) for one GEMM; each step uses a fresh pair of noise seeds
(another point of the nonce space).  Under torchrun every rank mines its own
seeds (nonce-space sharding, no collective on the data path; weak scaling)
and only hit counts are reduced after timing.

metric: effective TOPS = 2*M*N*K per GEMM / time (noise and denoise work not
counted, as in the reference's TOPS figure); hashed tiles/s = M*N/128 per
GEMM / time.

--impl reference times the reference's CPU path on the host cores: the C
restatement in oracle/ (the Rust miner zk-pow/src/ffi/mine.rs cannot be built
here: no cargo), each step a bounded sample of hash tiles of the same GEMM.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M = N = K = 8192
R = 128
HASH_TILE = 128  # elements per protocol hash tile (2 x 64)
TARGET_FRACTION = 1e-6  # expected hits per hash tile
# Kernels of this implementation launched per step (noise_gen 1, the fused
# noising of A and B 1, mined GEMM 1).
LAUNCHES_PER_STEP = 3


def target_value(frac: float) -> int:
    return int(frac * (1 << 256))


class BenchProblem:
    """Device buffers of one noisy GEMM laid out as the reference's callers
    lay them out (miner/vllm-miner/src/vllm_miner/gemm_operators.py:68-333):
    seeded int7 operands, the noise factors noise_gen fills, the noised
    operands, the half denoise factors and C."""

    def __init__(self, m, n, k, r, seed, device):
        g = torch.Generator().manual_seed(seed)
        self.m, self.n, self.k, self.r = m, n, k, r
        self.A = torch.randint(-64, 64, (m, k), generator=g, dtype=torch.int8).to(device)
        self.B = torch.randint(-64, 64, (n, k), generator=g, dtype=torch.int8).to(device)
        self.A_scales = torch.full((m,), 1.0 / 128, dtype=torch.float32, device=device)
        self.B_scales = torch.full((n,), 1.0 / 128, dtype=torch.float32, device=device)
        e = lambda *shape, dt=torch.int8: torch.empty(*shape, dtype=dt, device=device)  # noqa: E731
        self.noise = dict(EAL=e(m, r), EBR=e(n, r), EAR_R_major=e(k, r), EBL_R_major=e(k, r),
                          EAR_K_major=e(r, k), EBL_K_major=e(r, k), EAL_fp16=e(m, r, dt=torch.float16),
                          EBR_fp16=e(n, r, dt=torch.float16))
        self.out = dict(ApEA=e(m, k), BpEB=e(n, k), AxEBL_fp16=e(m, r, dt=torch.float16),
                        EARxBpEB_fp16=e(n, r, dt=torch.float16), C=e(m, n, dt=torch.bfloat16))


def bind_to_gpu_numa_node(dev: torch.device) -> str | None:
    """Restrict this process to the CPUs of the GPU's own NUMA node, so the
    pinned host buffers of the e2e leg (first touched by this process) sit
    on the node whose PCIe root serves the GPU.  Returns the node and CPU
    list used, or why nothing was changed."""
    try:
        props = torch.cuda.get_device_properties(dev)
        bus = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        base = f"/sys/bus/pci/devices/{bus}"
        node = int(open(f"{base}/numa_node").read().strip())
        if node < 0:
            return f"none: {bus} reports no NUMA node"
        cpulist = open(f"/sys/devices/system/node/node{node}/cpulist").read().strip()
        cpus = set()
        for part in cpulist.split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        os.sched_setaffinity(0, cpus)
        return f"node {node}: {cpulist}"
    except (AttributeError, OSError, ValueError) as e:
        return f"none: {type(e).__name__}: {e}"


def signal_buffers(pg, device):
    header = torch.zeros(pg.get_host_signal_header_size(), dtype=torch.int8, pin_memory=True)
    sync = torch.zeros(pg.get_host_signal_sync_size(), dtype=torch.int8, device=device)
    return header, sync


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return json.load(open(p))
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0,
            "fallback": True}


def ncu_traffic() -> dict | None:
    p = os.path.join(ROOT, "profiles", "traffic.json")
    return json.load(open(p)) if os.path.exists(p) else None


class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = os.path.join("/tmp", f"pb2_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9 and f[1].isdigit():
                rows.append(f)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [int(r[1]) for r in rows]
        loaded = [s for s in sm if s > 500] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": int(rows[0][2]),
                "reasons": reasons, "samples": len(rows)}


def setup_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        if args.impl == "ours":
            torch.cuda.set_device(local)
        dist.init_process_group("nccl" if args.impl == "ours" else "gloo",
                                timeout=datetime.timedelta(seconds=120))
    return world, rank, local


# ------------------------------------------------------------------ ours ---
def run_ours(args, world, rank, local):
    import pearl_b200 as pg
    from pearl_b200 import shard

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    all_cpus = os.sched_getaffinity(0)
    numa = bind_to_gpu_numa_node(dev)
    p = BenchProblem(M, N, K, R, seed=1000 + rank, device=dev)
    # A fresh pair of noise seeds every step: every rank mines its own points
    # of the nonce space (shard.rank_job_key), all resident before timing.
    n_keys = args.warmup + args.steps
    base = bytes(range(32))
    keys_a = torch.tensor([list(shard.rank_job_key(base, rank, 2 * i)) for i in range(n_keys)],
                          dtype=torch.uint8).to(dev)
    keys_b = torch.tensor([list(shard.rank_job_key(base, rank, 2 * i + 1)) for i in range(n_keys)],
                          dtype=torch.uint8).to(dev)
    target = pg.make_pow_target_tensor(target_value(TARGET_FRACTION), dev)
    header, sync = signal_buffers(pg, dev)
    hits = torch.zeros(1024, 12, dtype=torch.uint32, device=dev)
    stream = torch.cuda.current_stream(dev)
    ev_main = []
    factors = {k: v for k, v in p.noise.items() if k not in ("EAL", "EBR")}

    def step(i, record=False):
        # host_signal_sync is zeroed once before the timed loop, so hit_count
        # accumulates over the steps (the header keeps the first hit).
        ka, kb = keys_a[i % n_keys], keys_b[i % n_keys]
        pg.noise_gen(R=R, key_A=ka, key_B=kb, **p.noise)
        # The noising step of noisy_gemm(run_noising_A/B=True), issued apart
        # so that the events below bracket the mined GEMM alone.
        pg.noise_AB(p.A, p.noise["EAL"], p.out["AxEBL_fp16"], p.out["ApEA"],
                    p.B, p.noise["EBR"], p.out["EARxBpEB_fp16"], p.out["BpEB"], **factors)
        if record:
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        pg.noisy_gemm(A=p.A, B=p.B, A_scales=p.A_scales, B_scales=p.B_scales,
                      host_signal_header_pinned=header, host_signal_sync=sync, pow_target=target,
                      pow_key=ka.view(torch.uint32), run_noising_A=False, run_noising_B=False,
                      hits=hits, **p.noise, **p.out)
        if record:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record(stream)
            ev_main.append((e0, e1))

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    err = pg.get_host_signal_sync_fields(sync)["error"]
    if err:
        raise RuntimeError(f"device reported error {err}")
    sync.zero_()
    barrier(world)
    clocks = ClockSampler(dev.index if dev.index is not None else 0)
    clocks.start()
    time.sleep(0.3)
    torch.cuda.synchronize(dev)
    barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        step(args.warmup + i, record=True)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    main_ms = sum(a.elapsed_time(b) for a, b in ev_main) / len(ev_main)
    local_hits = int(pg.get_host_signal_sync_fields(sync)["hit_count"])
    total_hits = local_hits
    if world > 1:
        # The only cross-rank traffic: the slowest rank's time and the
        # winning proofs, gathered to rank 0 after the timed region.
        ms = shard.max_over_ranks(ms, dev)
        gathered = shard.gather_hits(hits, min(local_hits, hits.shape[0]))
        total_hits = None if gathered is None else int(gathered.shape[0])

    # ---- end to end through the public API with host buffers -------------
    e2e = None
    if args.e2e_steps > 0:
        e2e = run_e2e(args, p, keys_a, keys_b, target, header, sync, dev, world)
        e2e["host_numa_binding"] = numa
    os.sched_setaffinity(0, all_cpus)  # the CPU baseline below uses every host core

    # ---- live cuBLAS int8 reference point (rank 0) ------------------------
    cublas = None
    if rank == 0:
        try:
            for _ in range(3):
                torch._int_mm(p.A, p.B.t())
            torch.cuda.synchronize(dev)
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record(stream)
            for _ in range(10):
                torch._int_mm(p.A, p.B.t())
            b.record(stream)
            torch.cuda.synchronize(dev)
            cublas = 2 * M * N * K / (a.elapsed_time(b) / 10 * 1e-3) / 1e12
        except Exception:  # noqa: BLE001
            cublas = None

    if rank != 0:
        return None
    ops = 2.0 * M * N * K
    tiles = M * N / HASH_TILE
    step_s = ms / args.steps * 1e-3
    peaks = measured_peaks()
    # The mined GEMM is timed inside a short region (steps x ~0.6 ms) at the
    # full SM clock, so its denominator is the burst figure; the sustained
    # one (a seconds-long loop under the power cap) is given beside it.
    peak_int8 = 2.0 * peaks["bf16_tflops"]
    peak_int8_sustained = 2.0 * peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    achieved = ops / (main_ms * 1e-3) / 1e12
    traffic = ncu_traffic()
    line = {
        "metric": "effective TOPS (mined int8 noisy GEMM with fused transcript hashing)",
        "value": round(world * ops / step_s / 1e12, 2),
        "unit": "TOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic (seeded int7 operands, fresh noise seeds per step)",
        "config": {"workload": (f"pearl-gemm noisy_gemm M=N={M} K={K} R=128, target 1e-6 hits/hash tile"
                                if K != 8192 else "pearl-gemm noisy_gemm M=N=K=8192 R=128, target 1e-6 hits/hash tile"),
                   "m": M, "n": N, "k": K, "r": R, "hash_tile": "2x64",
                   "l2": "inputs larger than L2: A,B,ApEA,BpEB,C = 384 MiB per step > 126 MB",
                   "parallelism": f"nonce-space shards x{world}"},
        "hashed_tiles_per_s": round(world * tiles / step_s, 1),
        "hits": total_hits,
        "expected_hits": round(world * args.steps * tiles * TARGET_FRACTION, 2),
        "main_kernel_ms": round(main_ms, 4),
        "e2e": e2e,
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "roofline": {
            "kernel": "noisy_gemm_kernel<reduce,denoise> (tcgen05 kind::i8 + transcript + BLAKE3)",
            "bound": "tensor",
            "achieved": round(achieved, 1),
            "peak": round(peak_int8, 1),
            "unit": "TOPS",
            "frac": round(achieved / peak_int8, 4),
            "peak_source": ("2 x measured burst bf16 of MEASURED_PEAKS.json (B200 dense int8 = 2 x bf16)"
                            + (" [fallback figure]" if peaks.get("fallback") else "")),
            "frac_of_sustained": round(achieved / peak_int8_sustained, 4),
            "peak_sustained": round(peak_int8_sustained, 1),
            "cublas_int8_live_tops": round(cublas, 1) if cublas else None,
            "traffic": traffic.get("main_kernel_dram_bytes_per_launch") if traffic else None,
        },
        "clocks": clk,
    }
    # The CPU baseline is timed at N = 1 only: under torchrun the host cores
    # are shared by every rank's process.
    line["cpu_baseline"] = (cpu_baseline(budget_s=args.cpu_budget)
                            if world == 1 and args.cpu_budget > 0 and K == 8192 else None)
    return line


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def run_e2e(args, p, keys_a, keys_b, target, header, sync, dev, world):
    """Same metric through the public calls a miner makes (noise_gen +
    noisy_gemm with in-kernel noising), with every step's A and B copied from
    pinned host memory and its result (sync word + hit list) read back, all
    inside the timed region.  Two device buffer sets let step i+1's copies
    (on their own stream) overlap step i's GEMM."""
    import pearl_b200 as pg
    from pearl_b200 import shard

    hostA = p.A.cpu().pin_memory()
    hostB = p.B.cpu().pin_memory()
    hit_host = torch.zeros(64, 12, dtype=torch.uint32).pin_memory()
    sync_host = torch.zeros(16, dtype=torch.int8).pin_memory()
    hits = torch.zeros(64, 12, dtype=torch.uint32, device=dev)
    stream = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(dev)
    bufs = [(p.A, p.B), (torch.empty_like(p.A), torch.empty_like(p.B))]
    copied = [torch.cuda.Event() for _ in bufs]
    consumed = [torch.cuda.Event() for _ in bufs]
    steps = max(1, min(args.steps, args.e2e_steps))

    def issue_copy(i):
        b = i % 2
        if i >= 2:
            copy_stream.wait_event(consumed[b])  # step i-2 is done with the buffers
        with torch.cuda.stream(copy_stream):
            bufs[b][0].copy_(hostA, non_blocking=True)
            bufs[b][1].copy_(hostB, non_blocking=True)
            copied[b].record(copy_stream)

    def compute(i):
        b = i % 2
        A, B = bufs[b]
        stream.wait_event(copied[b])
        sync.zero_()
        ka, kb = keys_a[i % len(keys_a)], keys_b[i % len(keys_b)]
        pg.noise_gen(R=R, key_A=ka, key_B=kb, **p.noise)
        pg.noisy_gemm(A=A, B=B, A_scales=p.A_scales, B_scales=p.B_scales,
                      host_signal_header_pinned=header, host_signal_sync=sync, pow_target=target,
                      pow_key=ka.view(torch.uint32), hits=hits, **p.noise, **p.out)
        consumed[b].record(stream)
        sync_host.copy_(sync, non_blocking=True)
        hit_host.copy_(hits, non_blocking=True)

    def run(n):
        issue_copy(0)
        for i in range(n):
            if i + 1 < n:
                issue_copy(i + 1)
            compute(i)

    run(3)
    torch.cuda.synchronize(dev)
    barrier(world)
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record(stream)
    copy_stream.wait_event(a)  # the copies belong to the timed region too
    run(steps)
    b.record(stream)
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b)
    if world > 1:
        ms = shard.max_over_ranks(ms, dev)
    step_s = ms / steps * 1e-3
    return {"value": round(world * 2.0 * M * N * K / step_s / 1e12, 2), "unit": "TOPS",
            "h2d_bytes_per_step": 2 * M * K, "d2h_bytes_per_step": 16 + hit_host.numel() * 4,
            "steps": steps, "ms_per_step": round(ms / steps, 4),
            "path": "pearl_b200.noise_gen + pearl_b200.noisy_gemm (run_noising_A/B) from pinned host A,B; "
                    "next step's copies overlap this step's GEMM"}


# ------------------------------------------------------- CPU reference ----
class CpuProblem:
    """The headline GEMM prepared for the oracle: operands, noise, noised
    operands (the per-GEMM O(MK) part is timed once and amortized).

    Both CPU legs (the repo arm's cpu_baseline and the --impl reference arm)
    time the same kind of sample: whole windows of WINDOW consecutive hash
    tiles (16 rows of hash tiles across all of N) at fixed, evenly spread
    offsets, in the same order, so the two figures measure one rate."""

    WINDOW = 2048

    def __init__(self, seed=1000):
        import numpy as np

        from oracle import oracle as O
        self.O = O
        g = torch.Generator().manual_seed(seed)
        A = torch.randint(-64, 64, (M, K), generator=g, dtype=torch.int8).numpy()
        B = torch.randint(-64, 64, (N, K), generator=g, dtype=torch.int8).numpy()
        self.key_a = np.random.default_rng(seed + 1000).integers(0, 256, 32, dtype=np.uint8).tobytes()
        self.key_b = np.random.default_rng(seed + 2000).integers(0, 256, 32, dtype=np.uint8).tobytes()
        t = time.perf_counter()
        prob = O.noisy_problem(A, B, self.key_a, self.key_b, R)
        self.noise_s = time.perf_counter() - t
        self.ApEA, self.BpEB = prob.ApEA, prob.BpEB
        self.total_tiles = O.num_hash_tiles(M, N)
        self.windows = self.total_tiles // self.WINDOW
        self.target = target_value(TARGET_FRACTION)
        self.next = 0

    def window_time(self, count: int) -> float:
        """Seconds for the next `count` windows of the fixed sequence."""
        secs = 0.0
        for _ in range(count):
            start = ((self.next * 37) % self.windows) * self.WINDOW
            self.next += 1
            t = time.perf_counter()
            self.O.mine_tiles(self.ApEA, self.BpEB, R, self.key_a, self.target, start, start + self.WINDOW)
            secs += time.perf_counter() - t
        return secs

    def gemm_seconds(self, tiles: int, secs: float) -> float:
        return self.noise_s + secs / tiles * self.total_tiles


def cpu_baseline(budget_s: float = 12.0) -> dict:
    from oracle import oracle as O
    cp = CpuProblem()
    per = cp.window_time(1)  # also warms the thread pool
    count = max(1, min(cp.windows, int(budget_s / max(per, 1e-6))))
    secs = cp.window_time(count)
    tiles = count * cp.WINDOW
    gemm_s = cp.gemm_seconds(tiles, secs)
    return {"value": round(2.0 * M * N * K / gemm_s / 1e12, 6), "unit": "TOPS",
            "cores": O.num_threads(), "kind": "port",
            "hashed_tiles_per_s": round(cp.total_tiles / gemm_s, 1),
            "sample": (f"{tiles} of {cp.total_tiles} hash tiles of the 8192^3 GEMM ({count} fixed windows of "
                       f"{cp.WINDOW}, full K, {secs:.1f}s) + full noise/noising ({cp.noise_s:.2f}s), "
                       f"extrapolated per tile"),
            "cpu": cpu_model()}


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args, world, rank):
    if rank != 0:
        return None
    from oracle import oracle as O
    cp = CpuProblem()
    per = cp.window_time(1)  # also warms the thread pool
    # size the per-step sample so the whole run stays within ~args.ref_budget seconds
    per_step = max(1, int(args.ref_budget / max(1, args.steps + args.warmup) / max(per, 1e-6)))
    for _ in range(args.warmup):
        cp.window_time(per_step)
    secs = sum(cp.window_time(per_step) for _ in range(args.steps))
    tiles = per_step * cp.WINDOW * args.steps
    gemm_s = cp.gemm_seconds(tiles, secs)
    value = round(2.0 * M * N * K / gemm_s / 1e12, 6)
    sample = (f"{per_step} fixed windows of {cp.WINDOW} hash tiles (full K) per step of the 8192^3 GEMM, "
              f"amortized noise/noising ({cp.noise_s:.2f}s per GEMM); GEMM time extrapolated per tile")
    return {
        "impl": "reference",
        "metric": "effective TOPS (mined int8 noisy GEMM with fused transcript hashing)",
        "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(secs / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded int7 operands)",
        "config": {"workload": "pearl-gemm noisy_gemm M=N=K=8192 R=128, target 1e-6 hits/hash tile",
                   "m": M, "n": N, "k": K, "r": R,
                   "implementation": "oracle/pearl_oracle.c: C restatement of zk-pow/src/ffi/mine.rs "
                                     "(Rust toolchain absent, reference miner not buildable)"},
        "hashed_tiles_per_s": round(cp.total_tiles / gemm_s, 1),
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": O.num_threads(), "kind": "port",
                         "sample": sample, "cpu": cpu_model()},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------- other workloads
def _time_steps(fn, steps, warmup, dev, world):
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize(dev)
    barrier(world)
    stream = torch.cuda.current_stream(dev)
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record(stream)
    for i in range(steps):
        fn(warmup + i)
    b.record(stream)
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b)
    if world > 1:
        from pearl_b200 import shard
        ms = shard.max_over_ranks(ms, dev)
    return ms / steps


def _line(args, world, name, ops_per_step, ms, extra, mined_gemms):
    step_s = ms * 1e-3
    return {"metric": "effective TOPS (mined int8 noisy GEMM with fused transcript hashing)",
            "value": round(world * ops_per_step / step_s / 1e12, 2), "unit": "TOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded int7 weights / bf16 activations, random routing)",
            "config": {"workload": name, "mined_gemms_per_step": mined_gemms, **extra},
            "e2e": None, "cpu_baseline": None}


def run_workload(args, world, rank, local):
    """The other workloads (the default line is the 8192^3 GEMM): timed through the
    operators a miner calls, one step = one pass of the workload."""
    from pearl_b200 import miner as MN
    from pearl_b200 import shard
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    g = torch.Generator().manual_seed(77 + rank)
    base = bytes(range(32))
    job = lambda i: MN.MiningJob(shard.rank_job_key(base, rank, i), target_value(TARGET_FRACTION))  # noqa: E731
    if args.workload == "gemm16384":
        m, n, k = 16384, 8192, 8192
        A = torch.randint(-64, 64, (m, k), generator=g, dtype=torch.int8).to(dev)
        B = torch.randint(-64, 64, (n, k), generator=g, dtype=torch.int8).to(dev)
        sa = torch.full((m,), 1 / 128, device=dev)
        sb = torch.full((n,), 1 / 128, device=dev)
        done = []

        def step(i):
            C, mined = MN.pearl_gemm_noisy(A, B, sa, sb, torch.bfloat16, job(i))
            done.append(mined)
            if len(done) > 8:
                MN.release_header(done.pop(0).host_signal_header_pinned)
        ms = _time_steps(step, args.steps, args.warmup, dev, world)
        return _line(args, world, "16384 x 8192 x 8192 int8 mined GEMM with "
                     "commitment (tensor_hash A,B), noise_gen, noising, transcript, BLAKE3",
                     2.0 * m * n * k, ms, {"m": m, "n": n, "k": k, "r": R}, 1) if rank == 0 else None
    if args.workload == "fp8_16384":
        # The FP8 extension of the mined contraction on the 16384 x 8192 x
        # 8192 shape: normal(0,1) E4M3 operands with per-tensor scales.
        import pearl_b200 as pg
        m, n, k = 16384, 8192, 8192
        gdev = torch.Generator(device=dev).manual_seed(91 + rank)
        A8 = torch.randn(m, k, generator=gdev, device=dev).to(torch.float8_e4m3fn)
        B8 = torch.randn(n, k, generator=gdev, device=dev).to(torch.float8_e4m3fn)
        sa = torch.full((1,), 1 / 16, device=dev)
        sb = torch.full((1,), 1 / 16, device=dev)
        C = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        header, sync = signal_buffers(pg, dev)
        target = pg.make_pow_target_tensor(target_value(TARGET_FRACTION), dev)
        keys = [torch.tensor(list(shard.rank_job_key(base, rank, i)), dtype=torch.uint8).to(dev).view(torch.uint32)
                for i in range(8)]

        def step(i):
            pg.fp8.mined_gemm_fp8(A8, B8, sa, sb, C, header, sync, target, keys[i % 8])
        ms = _time_steps(step, args.steps, args.warmup, dev, world)
        if rank != 0:
            return None
        line = _line(args, world, "FP8 E4M3 mined GEMM M=16384 N=K=8192 (per-tensor scales, transcript over "
                     "f32 accumulators, BLAKE3, target compare; no noise)", 2.0 * m * n * k, ms,
                     {"m": m, "n": n, "k": k, "r": R, "operands": "float8_e4m3fn normal(0,1)"}, 1)
        line["dtype"] = "fp8_e4m3"
        line["metric"] = "effective TFLOPS (mined FP8 E4M3 GEMM with fused transcript hashing)"
        line["unit"] = "TFLOPS"
        line["roofline"] = {"kernel": "noisy_gemm_kernel<kind::f8f6f4>", "bound": "tensor",
                            "achieved": line["value"], "peak": round(2.0 * measured_peaks()["bf16_tflops"], 1),
                            "unit": "TFLOPS", "frac": round(line["value"] / (2.0 * measured_peaks()["bf16_tflops"]), 4),
                            "peak_source": "2 x measured burst bf16 (B200 dense FP8 = 2 x bf16)", "traffic": None}
        return line
    if args.workload in ("llama", "llama_decode"):
        tokens = 8192 if args.workload == "llama" else 256
        hidden, mlp, layers = 4096, 14336, 32
        shapes = [("qkv", 6144, hidden), ("o", hidden, hidden), ("gate_up", 2 * mlp, hidden),
                  ("down", hidden, mlp)]

        class Layer:
            pass
        w = {}
        for name, n_out, k_in in shapes:  # one weight per projection, reused by the 32 layers
            L = Layer()
            L.weight = torch.randint(-63, 64, (n_out, k_in), generator=g, dtype=torch.int8).to(dev)
            L.weight_scale = (torch.rand(n_out, 1, generator=g) / 64).to(dev)
            w[name] = L
        xs = {k_in: torch.randn(tokens, k_in, generator=g).to(torch.bfloat16).to(dev)
              for _, _, k_in in shapes}
        lin = MN.PearlLinear(True, MN.MiningConfig(), None)

        def step(i):
            lin.job = job(i)
            for _ in range(layers):
                for name, n_out, k_in in shapes:
                    lin.apply_weights(w[name], xs[k_in])
            for mnd in lin.mined:
                MN.release_header(mnd.host_signal_header_pinned)
            lin.mined.clear()
        graphed = False
        if tokens < 1024:
            # The decode step runs as one CUDA graph, as vLLM runs its decode
            # batches: 128 quantize + GEMM pairs would otherwise be launched
            # from Python one by one, and the GPU would wait on the host.
            for i in range(2):
                step(i)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step(0)
            step = lambda i: graph.replay()  # noqa: E731
            graphed = True
        ms = _time_steps(step, args.steps, args.warmup, dev, world)
        ops = layers * sum(2.0 * tokens * n_out * k_in for _, n_out, k_in in shapes)
        mined = layers * len(shapes) if tokens >= 1024 else 0
        if rank != 0:
            return None
        line = _line(args, world, f"Llama-3-8B linear layers x32 through PearlLinear.apply_weights "
                     f"({tokens} tokens: {'mined' if mined else 'vanilla int8'} branch, int7 quantization "
                     f"included)", ops, ms, {"tokens": tokens, "hidden": hidden, "mlp": mlp,
                                             "layers": layers, "cuda_graph": graphed}, mined)
        if not mined:
            # The decode step streams every weight once per layer: 218 MB of
            # int8 weights per layer (more than the 126 MB L2, so each GEMM
            # reads its weight from HBM even though the synthetic layers
            # share one weight per projection).
            wbytes = layers * sum(n_out * k_in for _, n_out, k_in in shapes)
            peak = measured_peaks()["hbm_gbs"]
            achieved = wbytes / (ms * 1e-3) / 1e9
            line["roofline"] = {"kernel": "whole decode step (weight streaming)", "bound": "hbm",
                                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                                "frac": round(achieved / peak, 4), "traffic": None,
                                "algorithmic_bytes_per_step": wbytes}
        return line
    if args.workload == "moe":
        E, tokens, top_k, N, K = 8, 16384, 2, 2 * 14336, 4096
        A = torch.randint(-64, 64, (tokens, K), generator=g, dtype=torch.int8).to(dev)
        sa = (torch.rand(tokens, 1, generator=g) / 64).to(dev)
        w1 = torch.randint(-64, 64, (E, N, K), generator=g, dtype=torch.int8).to(dev)
        w1s = (torch.rand(E, N, generator=g) / 64).to(dev)
        ids = torch.stack([torch.randperm(E, generator=g)[:top_k] for _ in range(tokens)]).to(torch.int32).to(dev)
        out = torch.empty(tokens * top_k, N, dtype=torch.bfloat16, device=dev)

        def step(i):
            _, res = MN.moe_gemm1(A, sa, ids, w1, w1s, job(i), out=out)
            for mnd in res.per_expert.values():
                MN.release_header(mnd.host_signal_header_pinned)
        ms = _time_steps(step, args.steps, args.warmup, dev, world)
        return _line(args, world, "Mixtral-8x7B MoE GEMM1 (8 experts, 16384 tokens, top-2, "
                     "N=2x14336, K=4096), routing + commitment + one mined GEMM per expert",
                     2.0 * tokens * top_k * N * K, ms, {"experts": E, "tokens": tokens, "top_k": top_k,
                                                         "n": N, "k": K}, E) if rank == 0 else None
    raise SystemExit(f"unknown workload {args.workload}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=40)
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--ref-budget", type=float, default=90.0)
    ap.add_argument("--workload", default="gemm8192",
                    choices=["gemm8192", "gemm16384", "llama", "llama_decode", "moe", "fp8_16384"],
                    help="gemm8192 (default) is the headline GEMM; the others are the larger "
                         "configs 3-5 measured through the miner-facing operators")
    ap.add_argument("--k", type=int, default=8192,
                    help="K of the default GEMM workload (8192 is the headline; a smaller K gives the "
                         "small case the full ncu sections are captured on)")
    args = ap.parse_args()
    global K
    K = args.k
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = setup_dist(args)
    try:
        if args.impl == "reference":
            line = run_reference(args, world, rank)
        else:
            line = (run_ours(args, world, rank, local) if args.workload == "gemm8192"
                    else run_workload(args, world, rank, local))
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
