"""Benchmark of the preemptible persistent-GEMM runtime (one JSON line).

Workload: a persistent fp32 SGEMM background task,
M=N=K=4096, 128x128 output tiles, K-tile 32, at full residency, while an
urgent fp32 256x256x256 GEMM (uniform[-1,1]) is injected by the host at a
uniformly random time inside every 1 ms period.  Inputs come from the
reference's generator (srand(21)/rand(), src/persistent.cu:132-135);
synthetic, no dataset involved.

A step is one launch of the persistent kernel: it drains background tiles
(task t computes tile t mod 1024) while `--events-per-step` urgent GEMMs are
injected by the host (flag stored with cudaMemcpyAsync on a high-priority
control stream); the launch is bounded and ends by itself.  value = the
background GEMM's TFLOP/s over the timed steps (FLOPs of completed tiles /
CUDA-event time of the launches, summed over ranks and divided by the max
over ranks); latency_us holds the urgent preemption latencies of all timed
events.  e2e = the same metric through the public API with host buffers:
apk_gemm over pinned host A, B -> C (H2D + drain + D2H), with the plain copy
ceiling of the same buffers beside it.

Every rank also runs the configs[4] leg (`config4`): 2^20 heterogeneous bf16
GEMM tasks from one seed, LPT-sharded over the ranks, each rank draining its
shard undisturbed and under a 2 kHz Poisson urgent stream; exactly-once over
the union of shards, corrupted half-tiles and urgent claims are checked on
the host after timing.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    python bench.py --case drain-f32|drain-bf16|tasks-bf16 [...]   # one small case, for ncu

Definitions of the latency keys: preempt = host store of the yield flag ->
host sees the device's claim ack (mapped memory, host clock, no clock
mapping); urgent_done = host store -> host sees the last urgent item's ack;
dev_* = globaltimer intervals from the first CTA to observe the flag
(claim after it, spread of observations, done after claim);
device_set.* = CTA 0 sets the flag on a schedule, so set -> claim / last
observer / done share one clock (the reference's primary instrument,
src/yield.cu:186-195).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M = N = K = 4096
U = 256
METRIC = "urgent-task p50/p99 preempt latency (us); background GEMM TFLOPS (% of peak)"
SMS_B200 = 148
# DRAM bytes (read + write) per 128x128x4096 tile of the warp-specialized
# fp32 kernel: one ncu capture of a 4096^3 drain (1024 tiles) measured
# 350.1 MB read + 53.0 MB written, i.e. 403.1 MB / 1024 tiles.  Command:
#   ncu --set full --clock-control none -k regex:sgemm_ws -s 1 -c 1 \
#       python bench.py --case drain-f32 --n 4096
# A constant, so a stale value shows up beside the profile it came from
# rather than silently; re-capture after any change to the kernel.
F32WS_DRAM_BYTES_PER_TILE = 393618
# DRAM bytes (read + write) per TFLOP of the configs[4] task kernel: one ncu
# capture of a 2^16-task list of the same generator measured 70.97 GB read +
# 94.84 GB written for 87.50 TFLOP.  Traffic grows with the work, so a full
# shard's launch is scaled by its TFLOP.  Command:
#   ncu --set full --clock-control none -k regex:gemm_bf16_persistent -s 1 -c 1 \
#       python bench.py --case tasks-bf16 --tasks 65536 --reps 2
C4_DRAM_BYTES_PER_TFLOP = (70.97e9 + 94.84e9) / 87.50


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--events-per-step", type=int, default=200)
    ap.add_argument("--period-us", type=float, default=1000.0)
    ap.add_argument("--no-extras", action="store_true", help="skip overhead/baseline/cpu legs")
    ap.add_argument("--no-config4", action="store_true", help="skip the configs[4] task-queue leg")
    ap.add_argument("--config4-tasks", type=int, default=1 << 20)
    # one small case for profilers (ncu): a few bounded launches, no timing contract
    ap.add_argument("--case", default=None, choices=["drain-f32", "drain-bf16", "tasks-bf16"])
    ap.add_argument("--n", type=int, default=0, help="--case drain-*: n^3 background")
    ap.add_argument("--reps", type=int, default=0, help="--case: launches")
    ap.add_argument("--poll", default="stage", choices=("off", "boundary", "stage"))
    ap.add_argument("--kernel", default="auto", help="--case drain-f32: auto|ws|sync; drain-bf16: auto|pair|single")
    ap.add_argument("--tasks", type=int, default=1 << 16, help="--case tasks-bf16: task count")
    return ap.parse_args()


# ---------------------------------------------------------------- clocks
def measured_peaks() -> dict:
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return {}


def pct(v, q):
    v = sorted(v)
    return v[min(int(q * len(v)), len(v) - 1)] if v else None


def r3(x):
    return None if x is None else round(float(x), 3)


# ---------------------------------------------------------------- dist
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        # control plane only (barriers, max/sum of per-rank results, the
        # exactly-once union after timing): the timed path has no
        # collective, each rank drains its own work
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def allgather_obj(world, obj):
    if world == 1:
        return [obj]
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


# ---------------------------------------------------------------- cpu legs
def numa_local_cpus(pci_bus_id: str):
    """The CPUs this process may use on the NUMA node of the GPU at this PCI
    address (sysfs local_cpulist), or None when unknown."""
    try:
        dom, rest = pci_bus_id.split(":", 1)
        path = "/sys/bus/pci/devices/%04x:%s/local_cpulist" % (int(dom, 16), rest.lower())
        with open(path) as f:
            spec = f.read().strip()
        cpus = set()
        for part in spec.split(","):
            a, _, b = part.partition("-")
            cpus.update(range(int(a), int(b or a) + 1))
        cpus &= os.sched_getaffinity(0)
    except (OSError, ValueError, AttributeError):
        return None
    return cpus or None


def host_cores() -> int:
    """Host threads this process may run on (set explicitly: torchrun exports
    OMP_NUM_THREADS=1, which must not decide the all-cores figure)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_desc():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def ref_loop_rows(oracle, A, B, rows):
    """The reference's float64 host loop (src/persistent.cu:221-227) as
    shipped: one thread, i-k-j order, on the first `rows` rows of A."""
    return oracle.gemm_f64_rows(A, B, 0, rows)


def size_rows(fn, target_s, lo=8):
    """Rows of the 4096^3 product that take about target_s through fn."""
    rows = lo
    while True:
        t = time.perf_counter()
        fn(rows)
        dt = time.perf_counter() - t
        if dt > 0.3 or rows >= M:
            break
        rows = min(M, rows * 4)
    return int(min(M, max(lo, rows * target_s / max(dt, 1e-3))))


def cpu_single_core(oracle, A, B, target_s=8.0):
    """(TFLOP/s, rows, seconds) of the reference's loop on one core."""
    rows = size_rows(lambda r: ref_loop_rows(oracle, A, B, r), target_s)
    t = time.perf_counter()
    ref_loop_rows(oracle, A, B, rows)
    dt = time.perf_counter() - t
    return 2.0 * rows * N * K / dt / 1e12, rows, dt


def cpu_all_cores(oracle, A, B, target_s=4.0):
    """The same loop row-parallel (OpenMP) on every host thread this process
    may use: a labelled side figure, not the baseline."""
    import numpy as np
    th = host_cores()
    run = lambda r: oracle.gemm_f64_omp(np.ascontiguousarray(A[:r]), B, th)  # noqa: E731
    rows = size_rows(run, target_s, lo=th)
    t = time.perf_counter()
    run(rows)
    dt = time.perf_counter() - t
    return 2.0 * rows * N * K / dt / 1e12, rows, th, dt


def run_reference(args, world, rank):
    """Reference arm: the reference's CPU implementation of the path (its
    float64 host GEMM, src/persistent.cu:221-227, as the oracle port) exactly
    as shipped -- single-threaded -- on a row band of the configs[1] product
    per step.  The same single-core measurement at every N: rank 0 runs it,
    the other ranks exit without work.  The OpenMP all-cores form is
    reported beside it under all_cores."""
    if rank != 0:
        return
    import oracle
    A, B = oracle.gen_uniform(M, N, K, 21)
    # size one step to ~2 s of single-core work so K+W steps end in minutes
    rows = size_rows(lambda r: ref_loop_rows(oracle, A, B, r), 2.0)
    for _ in range(args.warmup):
        ref_loop_rows(oracle, A, B, rows)
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        ref_loop_rows(oracle, A, B, rows)
        times.append(time.perf_counter() - t)
    tot = sum(times)
    val = 2.0 * rows * N * K * len(times) / tot / 1e12
    allc, arows, th, adt = cpu_all_cores(oracle, A, B)
    sample = f"{rows} of {M} rows of the 4096^3 float64 product per step, one thread"
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": tot / len(times) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (srand(21)/rand() uniform[-1,1], src/persistent.cu:132-135)",
        "config": {"workload": "configs[1] background GEMM fp32 4096^3 through the reference's float64 host "
                               "loop (src/persistent.cu:221-227), row band per step",
                   "rows_per_step": rows, "M": M, "N": N, "K": K,
                   "ranks": "rank 0 alone, the same single-core measurement at every N"},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": 1, "kind": "port", "sample": sample,
                         "cpu": cpu_desc()},
        "all_cores": {"value": allc, "unit": "TFLOP/s", "cores": th, "kind": "port",
                      "sample": f"{arows} rows, OpenMP row-parallel, {adt:.1f} s"},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- cases
def run_case(args):
    """One small bounded case for a profiler: --reps launches of one drain
    (fp32 or bf16 n^3 background, or a configs[4] task list), each printing
    its launch time.  Under ncu skip the first launch (`-s 1`) so the
    captured one runs with warm tensor maps and caches; the launches are
    bounded, so a serialised capture never waits for a host flag."""
    import apk_b200
    if args.case == "tasks-bf16":
        import numpy as np
        from apk_b200.runtime import POOL, gen_tasks
        tasks, n_chk = gen_tasks(args.tasks, 21)
        flops = float((2.0 * tasks["m"].astype(np.float64) * tasks["n"] * tasks["k"]).sum())
        A = apk_b200.fill_normal_bf16((POOL["a_rows"], POOL["a_cols"]), 101)
        B = apk_b200.fill_normal_bf16((POOL["b_rows"], POOL["b_cols"]), 102)
        Au = apk_b200.fill_normal_bf16((256, 256), 31)
        Bu = apk_b200.fill_normal_bf16((256, 256), 32)
        with apk_b200.Context(dtype="bf16", poll=args.poll, urgent_split_k=1,
                              bf16_kernel=args.kernel if args.kernel != "auto" else "auto") as c:
            c.set_task_pool(A, B, POOL["c_rows"], POOL["c_cols"])
            c.set_urgent(Au, Bu)
            nw = c.set_tasks(tasks, n_chk)
            for _ in range(args.reps or 3):
                c.launch(nw)
                c.wait(120)
                st = c.run_stats()
                print("tasks-bf16 %d tasks poll=%s: %.3f ms, %.1f TFLOP/s, %d halves" % (
                    args.tasks, args.poll, st["launch_ms"], flops / st["launch_ms"] / 1e9, st["tiles_done"]),
                    flush=True)
        return
    bf16 = args.case == "drain-bf16"
    n = args.n or (6144 if bf16 else 4096)
    reps = args.reps or (3 if bf16 else 2)
    if bf16:
        A = apk_b200.fill_normal_bf16((n, n), 21)
        B = apk_b200.fill_normal_bf16((n, n), 22)
        Au = apk_b200.fill_normal_bf16((256, 256), 31)
        Bu = apk_b200.fill_normal_bf16((256, 256), 32)
        kw = {"dtype": "bf16", "bf16_kernel": args.kernel}
    else:
        A, B = apk_b200.fill_uniform(n, n, n, 21)
        Au, Bu = apk_b200.fill_uniform(256, 256, 256, 99)
        kw = {"dtype": "f32", "f32_kernel": args.kernel}
    with apk_b200.Context(poll=args.poll, urgent_split_k=1, **kw) as c:
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        info = c.info
        tiles = (n // info["tile_m"]) * (-(-n // info["tile_n"]))
        for _ in range(reps):
            c.launch(tiles)
            c.wait(60)
            st = c.run_stats()
            print("%s %d^3 poll=%s: %.3f ms, %.1f TFLOP/s, %d tiles" % (
                args.case, n, args.poll, st["launch_ms"], 2.0 * n ** 3 / st["launch_ms"] / 1e9,
                st["tiles_done"]), flush=True)


# ---------------------------------------------------------------- extras
def device_set_latency(apk_b200, dev, A, B, Au, Bu, bg_tasks, events=200):
    """configs[1] with the reference's primary instrument: CTA 0 sets the
    flag at scheduled globaltimer instants (src/yield.cu:186-195), so set,
    observation, claim and completion share one clock."""
    with apk_b200.Context(device=dev, poll="stage", set_mode="device", max_events=events + 8) as c:
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        r = c.run_latency(events=events, period_us=1000, seed=7, warmup_events=10, settle_ms=2.0,
                          bg_tasks=bg_tasks)
    return {"n": r["n"], "unclaimed": r["unclaimed"], "claim_p50": r3(r["claim_p50_us"]),
            "claim_p99": r3(r["claim_p99_us"]), "last_obs_p50": r3(r["last_obs_p50_us"]),
            "last_obs_p99": r3(r["last_obs_p99_us"]), "done_p50": r3(r["done_p50_us"]),
            "done_p99": r3(r["done_p99_us"])}


def bf16_config2(apk_b200, np, dev):
    """bf16 8192^3, N(0,1) rounded to bf16, K-tile 64:
    throughput of the uninterrupted drain, then a drain with device-set
    yields at random pipeline stages whose output must be bitwise identical
    to the uninterrupted one."""
    n = 8192
    A = apk_b200.fill_normal_bf16((n, n), 21)
    B = apk_b200.fill_normal_bf16((n, n), 22)
    Au = apk_b200.fill_normal_bf16((256, 256), 31)
    Bu = apk_b200.fill_normal_bf16((256, 256), 32)
    peak = measured_peaks().get("bf16_tflops", 1590.0)
    with apk_b200.Context(device=dev, dtype="bf16", poll="stage", urgent_split_k=1) as c:
        ms = []
        for _ in range(6):
            C0 = c.gemm(A, B)
            ms.append(c.run_stats()["launch_ms"])
    med = statistics.median(ms[1:])
    tf = 2.0 * n ** 3 / (med / 1e3) / 1e12
    nev = 40
    with apk_b200.Context(device=dev, dtype="bf16", poll="stage", set_mode="device", urgent_split_k=1,
                          max_events=64) as c:
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_device_events((np.arange(nev, dtype=np.int64) + 1) * 25_000)
        info = c.info
        c.launch((n // info["tile_m"]) * (n // info["tile_n"]))
        c.wait(60)
        C = c.read_output()
        ev = c.read_events()
        st = c.run_stats()
    fired = int(np.count_nonzero(ev["set_ns"][:nev]))
    cl = [(ev["claim_ns"][e] - ev["set_ns"][e]) / 1e3 for e in range(fired) if ev["claimer"][e]]
    dn = [(ev["done_ns"][e] - ev["set_ns"][e]) / 1e3 for e in range(fired) if ev["done_ns"][e]]
    y = max(int(st["yields"]), 1)
    out = {"tflops": r3(tf), "pct_of_peak": r3(tf / peak * 100.0), "fired": fired, "ckpts": int(st["yields"]),
           "bitwise": bool(np.array_equal(C.view(np.uint32), C0.view(np.uint32))),
           "claim_p50": r3(pct(cl, 0.5)), "done_p50": r3(pct(dn, 0.5)),
           "spill_us": r3(st["ckpt_spill_ns"] / y / 1e3), "restore_us": r3(st["ckpt_restore_ns"] / y / 1e3),
           # TMEM <-> slab bandwidth of one checkpoint (a CTA pair's 512 KB)
           "spill_gbs": r3(st["ckpt_spill_bytes"] / max(st["ckpt_spill_ns"], 1)),
           "restore_gbs": r3(st["ckpt_restore_bytes"] / max(st["ckpt_restore_ns"], 1))}
    # the same drain as 256x128 jobs: the yielding accumulator parked in its
    # TMEM buffer against spilled to the slab (urgent done latency, rate)
    for kern in ("narrow", "narrow_spill"):
        with apk_b200.Context(device=dev, dtype="bf16", poll="stage", set_mode="device", urgent_split_k=1,
                              max_events=64, bf16_kernel=kern) as c:
            c.set_background(A, B)
            c.set_urgent(Au, Bu)
            c.schedule_device_events((np.arange(nev, dtype=np.int64) + 1) * 25_000)
            info = c.info
            c.launch((n // info["tile_m"]) * (n // info["tile_n"]))
            c.wait(60)
            Cn = c.read_output()
            ev = c.read_events()
            st = c.run_stats()
        fired = int(np.count_nonzero(ev["set_ns"][:nev]))
        dn = [(ev["done_ns"][e] - ev["set_ns"][e]) / 1e3 for e in range(fired) if ev["done_ns"][e]]
        cl = [(ev["claim_ns"][e] - ev["set_ns"][e]) / 1e3 for e in range(fired) if ev["claimer"][e]]
        out[kern] = {"tflops": r3(st["bg_tflops"]), "ckpts": int(st["yields"]), "parks": int(st["parks"]),
                     "claim_p50": r3(pct(cl, 0.5)), "done_p50": r3(pct(dn, 0.5)), "done_p99": r3(pct(dn, 0.99)),
                     "bitwise": bool(np.array_equal(Cn.view(np.uint32), C0.view(np.uint32)))}
    return out


# ---------------------------------------------------------------- our arm
def run_ours(args, world, rank, local):
    import numpy as np

    import apk_b200
    from apk_b200.clocks import ClockSampler, gpu_identity

    dev = local
    A, B = apk_b200.fill_uniform(M, N, K, 21)
    Au, Bu = apk_b200.fill_uniform(U, U, U, 99)
    ctx = apk_b200.Context(device=dev, poll="stage", set_mode="host_memcpy",
                           max_events=max(args.events_per_step, 16))
    info = ctx.info
    ctx.set_background(A, B)
    ctx.set_urgent(Au, Bu)
    # Every step is a bounded launch sized from the measured drain rate to
    # cover the injection schedule (+10%): it ends by itself, so no step
    # depends on a host action to terminate.
    ctx.launch(info["grid"] * 12)
    ctx.wait(60)
    cal = ctx.run_stats()
    ms_per_task = cal["launch_ms"] / cal["tiles_done"]
    settle_ms = 2.0
    step_ms = settle_ms + args.events_per_step * args.period_us / 1e3
    bg_tasks = int(step_ms * 1.10 / ms_per_task) + info["grid"]

    LAT_KEYS = ("rt_claim", "rt_done", "claim_after_first_obs", "spread", "done_after_claim")

    def one_step():
        # host-set events; no clock calibration: host round trips (host clock)
        # and device-clock intervals anchored on the first observer
        ctx.run_latency(events=args.events_per_step, period_us=args.period_us, seed=21 + rank,
                        warmup_events=0, settle_ms=settle_ms, bg_tasks=bg_tasks, probe_reps=0)
        st = ctx.run_stats()
        ev = ctx.read_events()
        n = ev["n_injected"]
        hs, ha, hd = ev["host_set_ns"][:n], ev["host_ack_ns"][:n], ev["host_done_ns"][:n]
        cl, dn, who = ev["claim_ns"][:n], ev["done_ns"][:n], ev["claimer"][:n]
        obs = ev["obs_ns"][:n]
        lat = {k: [] for k in LAT_KEYS}
        lat["unclaimed"] = lat["anomalies"] = 0
        for e in range(n):
            if who[e] == 0:
                lat["unclaimed"] += 1
                continue
            if ha[e]:
                lat["rt_claim"].append((ha[e] - hs[e]) / 1e3)
            if hd[e]:
                lat["rt_done"].append((hd[e] - hs[e]) / 1e3)
            o = obs[e]
            seen = o[o > 0]
            first = seen.min()
            lat["claim_after_first_obs"].append((cl[e] - first) / 1e3)
            if dn[e]:
                lat["done_after_claim"].append((dn[e] - cl[e]) / 1e3)
            if seen.size == o.size:
                lat["spread"].append((o.max() - first) / 1e3)
            else:
                lat["anomalies"] += 1
        return st, lat

    for _ in range(args.warmup):
        one_step()

    clocks = ClockSampler(dev)
    barrier(world)
    clocks.start()
    flops = 0.0
    tiles = 0
    launch_ms = []
    lats = {k: [] for k in LAT_KEYS}
    lats["unclaimed"] = lats["anomalies"] = 0
    yields = 0
    for _ in range(args.steps):
        st, lat = one_step()
        flops += st["bg_flops"]
        tiles += st["tiles_done"]
        launch_ms.append(st["launch_ms"])
        yields += st["yields"]
        for k in lats:
            lats[k] = lats[k] + lat[k]
    barrier(world)
    clk = clocks.stop()

    # e2e through the public API with pinned host buffers, allocated by this
    # rank while it runs on its GPU's NUMA node, so the pages land there
    # (the previous CPU set is restored for the rest of the run)
    gpu = gpu_identity(local)
    near = numa_local_cpus(gpu.get("pci_bus_id", ""))
    prev = os.sched_getaffinity(0) if near else None
    try:
        if near:
            os.sched_setaffinity(0, near)
        hA = apk_b200.pinned_empty((M, K), np.float32)
        hB = apk_b200.pinned_empty((K, N), np.float32)
        hC = apk_b200.pinned_empty((M, N), np.float32)
        hA[:] = 0
        hB[:] = 0
        hC[:] = 0
    finally:
        if prev:
            os.sched_setaffinity(0, prev)

    hA[:] = A
    hB[:] = B
    for _ in range(2):
        ctx.gemm(hA, hB, hC)
    barrier(world)  # every rank's copies contend for the host at once, as in the timed steps
    e2e_t = []
    for _ in range(max(3, args.steps)):
        t = time.perf_counter()
        ctx.gemm(hA, hB, hC)
        e2e_t.append(time.perf_counter() - t)
    e2e_tf = 2.0 * M * N * K / statistics.median(e2e_t) / 1e12
    # the copy ceiling: the same buffers and copy streams, no kernel, all
    # ranks at once (PCIe and host memory are shared between the GPUs)
    barrier(world)
    cp = ctx.probe_copy(hA, hB, hC, reps=5)
    # single-pass kernel time: one 4096^3 drain with the operands resident
    ctx.set_background(A, B)
    ctx.launch((M // info["tile_m"]) * (N // info["tile_n"]))
    ctx.wait(60)
    one_pass = ctx.run_stats()

    extras = {}
    if not args.no_extras:
        on_ms, off_ms = ctx.run_overhead(info["grid"] * 12, reps=3)
        extras["poll_cost_pct"] = r3((on_ms / off_ms - 1.0) * 100.0)
        base = ctx.run_baseline(1024, trials=20, seed=21)
        extras["no_preempt_us"] = {"p50": r3(pct(list(base), 0.5)), "p99": r3(pct(list(base), 0.99))}
    ctx.close()
    if not args.no_extras:
        extras["device_set"] = device_set_latency(apk_b200, dev, A, B, Au, Bu, bg_tasks)
        extras["bf16_config2"] = bf16_config2(apk_b200, np, dev)

    c4 = None
    if not args.no_config4:
        from apk_b200 import config4
        barrier(world)  # the shards drain concurrently on all GPUs
        c4_res, ex0, ex1 = config4.run_rank(dev, world, rank, args.config4_tasks)
        counts = config4.union_counts(world, ex0, ex1)
        c4_all = allgather_obj(world, c4_res)
        if rank == 0:
            c4 = config4.summarize(c4_all, counts, args.config4_tasks)
            # by GPU time the configs[4] drains are the run's dominant kernel
            # (the one-CTA bf16 task kernel): its roofline per GPU, against
            # the sustained tensor peak (a ~1.6 s drain runs at the power cap)
            per_gpu = c4["tflops_undisturbed"] / world
            peak_s = measured_peaks().get("bf16_tflops_sustained", 1400.0)
            c4["roofline"] = {"bound": "tensor", "achieved": r3(per_gpu), "peak": peak_s, "unit": "TFLOP/s",
                              "frac": r3(per_gpu / peak_s),
                              "traffic": r3(C4_DRAM_BYTES_PER_TFLOP * c4["pflop"] * 1e3 / world),
                              "kernel": "bf16::gemm_bf16_persistent<POLL_STAGE,DRAIN,oracle,STD64> (task list)"}

    res = {"flops": flops, "launch_s": sum(launch_ms) / 1e3, "lats": lats, "clk": clk,
           "e2e_tf": e2e_tf, "copy": cp, "extras": extras, "info": info, "yields": yields,
           "one_pass_ms": one_pass["launch_ms"], "one_pass_tiles": one_pass["tiles_done"],
           "tiles": tiles, "launch_ms": launch_ms}
    allr = allgather_obj(world, res)
    if rank != 0:
        return
    tot_flops = sum(r["flops"] for r in allr)
    tmax = max(r["launch_s"] for r in allr)
    value = tot_flops / tmax / 1e12
    L = {k: [] for k in LAT_KEYS}
    unclaimed = anomalies = 0
    for r in allr:
        for k in L:
            L[k] += r["lats"][k]
        unclaimed += r["lats"]["unclaimed"]
        anomalies += r["lats"]["anomalies"]
    clk = allr[0]["clk"]
    sm_mhz = clk.get("sm_mhz") or 1965.0
    fp32_peak_clock = SMS_B200 * 128 * 2 * sm_mhz * 1e6 / 1e12
    # the dominant kernel's launches inside the timed region (rank 0): the
    # algorithmic FLOPs of the tiles they completed / their summed
    # CUDA-event durations, i.e. FLOPs per launch / average launch time
    r0 = allr[0]
    nl = max(1, len(r0["launch_ms"]))
    achieved = 2.0 * 128 * 128 * K * r0["tiles"] / (sum(r0["launch_ms"]) / 1e3) / 1e12
    one_drain = 2.0 * 128 * 128 * K * r0["one_pass_tiles"] / (r0["one_pass_ms"] / 1e3) / 1e12
    gemm_flop = 2.0 * M * N * K
    # e2e ceiling: a call moves A, B in and C out, so no call ends before
    # both directions' copies have (measured together, every rank at once)
    copy_ceiling = sum(gemm_flop / (r["copy"]["both_ms"] / 1e3) / 1e12 for r in allr)
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": tmax * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "gpu_launches": args.steps,
        "config": {"workload": "configs[1]: fp32 4096^3 persistent SGEMM background, 128x128 tiles, K-tile 32, "
                               "full residency; urgent fp32 256^3 host-injected once per 1 ms",
                   "events_per_step": args.events_per_step, "grid": r0["info"]["grid"],
                   "ctas_per_sm": r0["info"]["ctas_per_sm"], "poll": "stage", "set": "host_memcpy",
                   "urgent_split_k": 8, "l2": "inputs > L2 (A+B+C 192 MB)",
                   "parallelism": f"{world} ranks, no collectives; configs[1] per rank, configs[4] sharded"},
        "roofline": {"bound": "fp32_fma", "achieved": achieved, "peak": fp32_peak_clock, "unit": "TFLOP/s",
                     "frac": achieved / fp32_peak_clock,
                     "traffic": F32WS_DRAM_BYTES_PER_TILE * r0["tiles"] / nl,
                     "peak_source": f"148 SMs x 128 lanes x 2 x {sm_mhz:.0f} MHz (sampled); no FP32 figure "
                                    "in MEASURED_PEAKS.json",
                     "kernel": "f32ws::sgemm_ws<POLL_STAGE,DRAIN>", "launches": nl,
                     "tiles_per_launch": r0["tiles"] / nl, "one_drain_tflops": r3(one_drain)},
        "clocks": clk,
        "e2e": {"value": sum(r["e2e_tf"] for r in allr), "unit": "TFLOP/s",
                "h2d_bytes_per_step": 2 * M * K * 4, "d2h_bytes_per_step": M * N * 4,
                "copy_ceiling": r3(copy_ceiling), "numa_local": bool(near),
                "copy_ms": {k: r3(r0["copy"][k]) for k in ("h2d_ms", "d2h_ms", "both_ms")}},
        "gpu": gpu,
        "extras": allr[0]["extras"],
    }
    if world == 1 and not args.no_extras:
        try:
            import oracle
            Ao, Bo = oracle.gen_uniform(M, N, K, 21)
            v, rows, dt = cpu_single_core(oracle, Ao, Bo)
            line["cpu_baseline"] = {"value": v, "unit": "TFLOP/s", "cores": 1, "kind": "port",
                                    "sample": f"{rows} of {M} rows of the 4096^3 float64 product ({dt:.1f} s), "
                                              "the reference's loop single-threaded as shipped",
                                    "cpu": cpu_desc()}
            va, ra, th, dta = cpu_all_cores(oracle, Ao, Bo)
            line["cpu_all_cores"] = {"value": va, "unit": "TFLOP/s", "cores": th, "kind": "port",
                                     "sample": f"{ra} rows, OpenMP row-parallel ({dta:.1f} s)"}
        except Exception as e:  # the GPU number stands without it
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    if c4 is not None:
        line["config4"] = {k: (r3(v) if isinstance(v, float) else v) for k, v in c4.items()}
    line["latency_us"] = {
        "events": len(L["claim_after_first_obs"]) + unclaimed, "unclaimed": unclaimed, "anomalies": anomalies,
        "preempt_p50": r3(pct(L["rt_claim"], 0.5)), "preempt_p99": r3(pct(L["rt_claim"], 0.99)),
        "urgent_done_p50": r3(pct(L["rt_done"], 0.5)), "urgent_done_p99": r3(pct(L["rt_done"], 0.99)),
        "dev_claim_p50": r3(pct(L["claim_after_first_obs"], 0.5)),
        "dev_claim_p99": r3(pct(L["claim_after_first_obs"], 0.99)),
        "dev_spread_p50": r3(pct(L["spread"], 0.5)), "dev_spread_p99": r3(pct(L["spread"], 0.99)),
        "dev_done_p50": r3(pct(L["done_after_claim"], 0.5)), "dev_done_p99": r3(pct(L["done_after_claim"], 0.99)),
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.case:
        run_case(args)
        return
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
