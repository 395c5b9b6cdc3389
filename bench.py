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
control stream), then the host stops it.  value = the
background GEMM's TFLOP/s over the timed steps (FLOPs of completed tiles /
CUDA-event time of the launches, summed over ranks and divided by the max
over ranks); the urgent preemption latencies of all timed events are
reported beside it.  e2e = the same metric through the public API with
host buffers: apk_gemm over pinned host A, B -> C (H2D + drain + D2H).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--events-per-step", type=int, default=200)
    ap.add_argument("--period-us", type=float, default=1000.0)
    ap.add_argument("--no-extras", action="store_true", help="skip overhead/baseline/cpu legs")
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


# ---------------------------------------------------------------- dist
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        # control plane only (barriers, max/sum of per-rank results): the
        # timed path has no collective, each rank drains its own shard
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
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
def cpu_gemm_sample(target_s: float = 8.0):
    """The reference's float64 loop (oracle port of src/persistent.cu:221-227),
    row-parallel on every host thread, on a row band of the 4096^3 workload
    sized to about target_s seconds.  Returns (TFLOP/s, rows, threads, secs)."""
    import oracle
    A, B = oracle.gen_uniform(M, N, K, 21)
    th = oracle.max_threads()
    import numpy as np
    rows = max(th, 8)
    while True:
        t = time.perf_counter()
        _ = oracle_gemm_band(oracle, A, B, rows, th)
        dt = time.perf_counter() - t
        if dt > 0.5 or rows >= M:
            break
        rows = min(M, rows * 4)
    rows = int(min(M, max(th, rows * target_s / max(dt, 1e-3))))
    t = time.perf_counter()
    oracle_gemm_band(oracle, A, B, rows, th)
    dt = time.perf_counter() - t
    del np
    return 2.0 * rows * N * K / dt / 1e12, rows, th, dt


def oracle_gemm_band(oracle, A, B, rows, th):
    import numpy as np
    Ab = np.ascontiguousarray(A[:rows])
    return oracle.gemm_f64_omp(Ab, B, th)


def cpu_desc():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def run_reference(args, world, rank):
    """Reference arm: the reference's own CPU implementation of the path (its
    float64 host GEMM, as the oracle port) on all host threads."""
    if rank != 0:
        return
    import oracle
    A, B = oracle.gen_uniform(M, N, K, 21)
    th = oracle.max_threads()
    # size one step to ~2 s of work so K+W steps end within a few minutes
    rows = max(th, 16)
    t = time.perf_counter()
    oracle_gemm_band(oracle, A, B, rows, th)
    dt = time.perf_counter() - t
    rows = int(min(M, max(th, rows * 2.0 / max(dt, 1e-3))))
    for _ in range(args.warmup):
        oracle_gemm_band(oracle, A, B, rows, th)
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        oracle_gemm_band(oracle, A, B, rows, th)
        times.append(time.perf_counter() - t)
    tot = sum(times)
    val = 2.0 * rows * N * K * len(times) / tot / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": tot / len(times) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (srand(21)/rand() uniform[-1,1], src/persistent.cu:132-135)",
        "config": {"workload": "configs[1] background GEMM fp32 4096^3 as the reference's float64 host "
                               "loop (src/persistent.cu:221-227), row band per step",
                   "rows_per_step": rows, "M": M, "N": N, "K": K},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": th, "kind": "port",
                         "sample": f"{rows} of {M} rows of the 4096^3 product per step, OpenMP row-parallel",
                         "cpu": cpu_desc()},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- extras
def device_set_latency(apk_b200, np, dev, A, B, Au, Bu, bg_tasks, events=200):
    """configs[1] with the reference's primary instrument: CTA 0 sets the
    flag at scheduled globaltimer instants (src/yield.cu:186-195), so set,
    observation, claim and completion share one clock."""
    with apk_b200.Context(device=dev, poll="stage", set_mode="device", max_events=events + 8) as c:
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        r = c.run_latency(events=events, period_us=1000, seed=7, warmup_events=10, settle_ms=2.0,
                          bg_tasks=bg_tasks)
    keys = ("n", "unclaimed", "anomalies", "claim_p50_us", "claim_p99_us", "last_obs_p50_us",
            "last_obs_p99_us", "done_p50_us", "done_p99_us", "bg_tflops")
    return {k: r[k] for k in keys}


def bf16_config2(apk_b200, np, dev):
    """bf16 8192^3, N(0,1) rounded to bf16, K-tile 64 (the
    reference's shape is 256x128 tiles in a 4-stage ring; this kernel runs
    256x256 tiles in a 3-stage ring of the same 192 KB): throughput of the
    uninterrupted drain, then a drain with device-set yields at random
    pipeline stages whose output must be bitwise identical to the
    uninterrupted one."""
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
    mid = sum(1 for e in range(fired) if ev["claimer"][e] and ev["claim_site"][e] > 0)
    return {"tflops_median": tf, "pct_of_measured_peak": tf / peak * 100.0, "peak_tflops": peak,
            "ms_median": med, "yield_run": {
                "events_fired": fired, "checkpoints": st["yields"], "mid_pipeline_claims": mid,
                "bitwise_equal_to_uninterrupted": bool(np.array_equal(C.view(np.uint32), C0.view(np.uint32))),
                "claim_p50_us": pct(cl, 0.5), "claim_p99_us": pct(cl, 0.99),
                "done_p50_us": pct(dn, 0.5), "done_p99_us": pct(dn, 0.99),
                "tflops_with_yields": st["bg_tflops"], "checkpoint": ckpt_stats(st)}}


def ckpt_stats(st):
    """Checkpoint traffic of a bf16 yield run: bytes moved between TMEM and
    the slab, mean CTA wall time per checkpoint and the CTA's GB/s."""
    y = max(int(st["yields"]), 1)
    out = {}
    for k in ("spill", "restore"):
        b, ns = int(st[f"ckpt_{k}_bytes"]), int(st[f"ckpt_{k}_ns"])
        out[f"{k}_bytes"] = b
        out[f"{k}_us_mean"] = ns / y / 1e3
        out[f"{k}_gbs_per_cta"] = b / ns if ns > 0 else None
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
    wall0 = time.perf_counter()
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
            lats[k] = lats[k] + lat[k] if isinstance(lats[k], list) else lats[k] + lat[k]
    wall = time.perf_counter() - wall0
    barrier(world)
    clk = clocks.stop()

    # e2e through the public API with pinned host buffers
    hA = apk_b200.pinned_empty((M, K), np.float32)
    hB = apk_b200.pinned_empty((K, N), np.float32)
    hC = apk_b200.pinned_empty((M, N), np.float32)
    hA[:] = A
    hB[:] = B
    for _ in range(2):
        ctx.gemm(hA, hB, hC)
    e2e_t = []
    for _ in range(max(3, args.steps)):
        t = time.perf_counter()
        ctx.gemm(hA, hB, hC)
        e2e_t.append(time.perf_counter() - t)
    e2e_tf = 2.0 * M * N * K / statistics.median(e2e_t) / 1e12
    # single-pass kernel time for the roofline: one 4096^3 drain with the
    # operands already resident (apk_gemm from host memory streams them in
    # while the kernel runs, so its launch time includes the transfers)
    ctx.set_background(A, B)
    ctx.launch((M // info["tile_m"]) * (N // info["tile_n"]))
    ctx.wait(60)
    one_pass = ctx.run_stats()

    extras = {}
    if not args.no_extras:
        on_ms, off_ms = ctx.run_overhead(info["grid"] * 12, reps=3)
        extras["poll_cost_pct"] = (on_ms / off_ms - 1.0) * 100.0
        extras["drain_ms_poll_on"] = on_ms
        extras["drain_ms_poll_off"] = off_ms
        base = ctx.run_baseline(1024, trials=20, seed=21)
        extras["no_preemption_e2e_us"] = {"p50": pct(list(base), 0.5), "p99": pct(list(base), 0.99)}
    ctx.close()
    if not args.no_extras:
        extras["device_set"] = device_set_latency(apk_b200, np, dev, A, B, Au, Bu, bg_tasks)
        extras["bf16_config2"] = bf16_config2(apk_b200, np, dev)

    res = {"flops": flops, "launch_s": sum(launch_ms) / 1e3, "lats": lats, "wall": wall, "clk": clk,
           "e2e_tf": e2e_tf, "extras": extras, "info": info, "yields": yields,
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
    fp32_peak_nominal = SMS_B200 * 128 * 2 * 1965e6 / 1e12
    fp32_peak_clock = SMS_B200 * 128 * 2 * sm_mhz * 1e6 / 1e12
    per_gpu = value / world
    # the dominant kernel's launches inside the timed region (rank 0): the
    # algorithmic FLOPs of the tiles they completed / their summed
    # CUDA-event durations, i.e. FLOPs per launch / average launch time
    r0 = allr[0]
    achieved = 2.0 * 128 * 128 * K * r0["tiles"] / (sum(r0["launch_ms"]) / 1e3) / 1e12
    one_drain = 2.0 * 128 * 128 * K * r0["one_pass_tiles"] / (r0["one_pass_ms"] / 1e3) / 1e12
    # DRAM bytes per launch: the ncu capture's per-tile traffic (read + write)
    # scaled to the average tiles of a timed launch
    traffic = None
    tp = os.path.join(ROOT, "profiles", "sgemm_f32_ws_4096.md")
    if os.path.exists(tp):
        for ln in open(tp):
            if ln.startswith("dram_bytes_per_tile:"):
                traffic = float(ln.split(":", 1)[1]) * r0["tiles"] / max(1, len(r0["launch_ms"]))
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": tmax * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "configs[1]: persistent fp32 SGEMM 4096^3 background, 128x128 tiles, K-tile 32, "
                               "full residency; urgent fp32 256^3 injected by the host (flag via cudaMemcpyAsync) at a "
                               "uniform time in every 1 ms period",
                   "M": M, "N": N, "K": K, "urgent": [U, U, U], "events_per_step": args.events_per_step,
                   "period_us": args.period_us, "grid": allr[0]["info"]["grid"],
                   "ctas_per_sm": allr[0]["info"]["ctas_per_sm"], "poll": "stage", "set": "host_memcpy",
                   "urgent_split_k": 8, "l2": "inputs larger than L2: A+B+C = 192 MB > 126 MB",
                   "parallelism": f"{world} independent replicas (no collectives)"},
        "latency_us": {
            "events": len(L["claim_after_first_obs"]) + unclaimed, "unclaimed": unclaimed, "anomalies": anomalies,
            "preempt_p50": pct(L["rt_claim"], 0.5), "preempt_p99": pct(L["rt_claim"], 0.99),
            "urgent_done_p50": pct(L["rt_done"], 0.5), "urgent_done_p99": pct(L["rt_done"], 0.99),
            "device_claim_after_first_observer_p50": pct(L["claim_after_first_obs"], 0.5),
            "device_claim_after_first_observer_p99": pct(L["claim_after_first_obs"], 0.99),
            "device_observation_spread_p50": pct(L["spread"], 0.5),
            "device_observation_spread_p99": pct(L["spread"], 0.99),
            "device_done_after_claim_p50": pct(L["done_after_claim"], 0.5),
            "device_done_after_claim_p99": pct(L["done_after_claim"], 0.99),
            "definition": "preempt = host store of the yield flag -> host sees the device's claim ack (the "
                          "first popper of the urgent work, acked through mapped memory), host clock, no "
                          "clock mapping; urgent_done = host store -> host sees the last urgent item's ack; "
                          "device_* are globaltimer intervals from the first CTA to observe the flag "
                          "(src/yield.cu:148-153); extras.device_set measures set->claim in one clock",
        },
        "bg_pct_of_fp32_peak": {"nominal_1965MHz": per_gpu / fp32_peak_nominal * 100.0,
                                "at_measured_clock": per_gpu / fp32_peak_clock * 100.0},
        "yields": sum(r["yields"] for r in allr),
        "roofline": {"bound": "fp32_fma", "achieved": achieved, "peak": fp32_peak_clock, "unit": "TFLOP/s",
                     "frac": achieved / fp32_peak_clock, "traffic": traffic,
                     "peak_source": f"148 SMs x 128 FP32 lanes x 2 x {sm_mhz:.0f} MHz (median SM clock sampled "
                                    "under load); MEASURED_PEAKS.json has no FP32 CUDA-core figure",
                     "kernel": "apk::f32ws::sgemm_ws<POLL_STAGE, DRAIN>: the timed steps' bounded launches "
                               "(4096^3 background tiles under urgent injections)",
                     "launches": len(r0["launch_ms"]), "tiles_per_launch": r0["tiles"] / max(1, len(r0["launch_ms"])),
                     "one_drain_tflops": one_drain},
        "e2e": {"value": sum(r["e2e_tf"] for r in allr), "unit": "TFLOP/s",
                "h2d_bytes_per_step": 2 * M * K * 4, "d2h_bytes_per_step": M * N * 4,
                "path": "apk_gemm with pinned host A, B -> C: A row panels and B column panels stream in "
                        "(interleaved) while the persistent kernel runs, C blocks stream back as they finish"},
        "gpu_launches": args.steps,
        "clocks": clk,
        "gpu": gpu_identity(local),
        "extras": allr[0]["extras"],
    }
    if rank == 0 and world == 1 and not args.no_extras:
        try:
            v, rows, th, dt = cpu_gemm_sample()
            line["cpu_baseline"] = {"value": v, "unit": "TFLOP/s", "cores": th, "kind": "port",
                                    "sample": f"{rows} of {M} rows of the 4096^3 float64 product "
                                              f"({dt:.1f} s), OpenMP row-parallel restatement of "
                                              "src/persistent.cu:221-227", "cpu": cpu_desc()}
        except Exception as e:  # the GPU number stands without it
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
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
