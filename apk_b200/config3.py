"""the scaling surface of the preemptible persistent GEMM.

    python -m apk_b200.config3 [--events 600] [--warmup 100] [--dtype f32|bf16|both]

Cells: resident CTAs per SM {1, 2, 4, 8} x K-tile {32, 64, 128} x shape
{4096^3, 16384x1024x4096}, fp32 and bf16, operands uniform[-1,1] from the
reference generator (bf16: the same values rounded to nearest even).  Each
feasible cell

* times ABAB-interleaved bounded drains with per-stage polling vs polling
  off in the same library (throughput cost of the poll, src/yield.cu:670-711);
* runs a bounded background drain while CTA 0 sets the yield flag at
  uniform-random instants, one per 1 ms (device-set events, the reference's
  primary instrument, src/yield.cu:186-195), discards the warm-up events
  (src/yield.cu:340) and reports on the device clock: set -> claim (yield
  latency), set -> last CTA observation (flag-propagation time) and
  set -> urgent done;
* compares that drain's TFLOP/s with an undisturbed drain of the same
  tasks run just before it (preemption cost).  Both last about a second, so
  both run at the clock the 1 kW power cap allows under sustained load (bf16
  settles near 1.4 GHz); the short ABAB drains of the poll cost run at burst
  clocks.  SM clocks and throttle reasons are sampled during each.

Every cell has a geometry: 4 and 8 fp32 CTAs per SM run 64x128 and 32x128
tiles, 2 / 4 / 8 bf16 CTAs run 256x128 / 128x128 / 64x128 tiles with one
TMEM buffer each, and the K-tile is the K depth between two yield sites,
moved through each kernel's own ring slots.  A cell whose CTAs would not
all fit on an SM is reported with the occupancy limit instead of numbers.  One JSON line per cell, then a
summary table.  Each cell runs in a process of its own, so that no cell's
timing depends on the device allocations and kernels of the cells before
it.
"""
from __future__ import annotations

import argparse
import json
import math
import subprocess
import sys

CTAS = (1, 2, 4, 8)
KTILES = (32, 64, 128)
SHAPES = ((4096, 4096, 4096), (16384, 1024, 4096))
URGENT = 256


def _operands(apk_b200, dtype, M, N, K):
    A, B = apk_b200.fill_uniform(M, N, K, 21)
    Au, Bu = apk_b200.fill_uniform(URGENT, URGENT, URGENT, 99)
    if dtype == "bf16":
        A, B, Au, Bu = (apk_b200.round_bf16(x) for x in (A, B, Au, Bu))
    return A, B, Au, Bu


def geometry(dtype, cps):
    """The tile geometry each cell runs (the runtime picks it from
    ctas_per_sm; restated here for the report)."""
    if dtype == "f32":
        return {1: "128x128 tiles, 128-thread CTAs", 2: "128x128 tiles, two workers per 384-thread CTA",
                4: "64x128 tiles, 64-thread CTAs", 8: "32x128 tiles, 32-thread CTAs"}[cps]
    return {1: "256x512 tiles on CTA pairs (K-tile >= 64) / 256x256 (K-tile 32)",
            2: "256x128 tiles, 256 TMEM columns", 4: "128x128 tiles, 128 TMEM columns",
            8: "64x128 tiles, 64 TMEM columns"}[cps]


def _infeasible_reason(dtype, cps, kt, info):
    """None when the cell runs as asked; else why the runtime could not place
    cps CTAs of the cell's geometry on an SM (its occupancy limit)."""
    if info is not None and info["ctas_per_sm"] != cps:
        return f"{cps} CTAs/SM: at most {info['max_ctas_per_sm']} of this geometry fit ({geometry(dtype, cps)})"
    return None


def run_cell(apk_b200, dtype, cps, kt, shape, events, warmup, seed, operands):
    from apk_b200.clocks import ClockSampler
    M, N, K = shape
    cell = {"dtype": dtype, "ctas_per_sm": cps, "k_tile": kt, "shape": [M, N, K]}
    # fp32 urgent items are one K-tile each (configs[1]: split-K 8 at K-tile 32)
    split = URGENT // kt if dtype == "f32" else 1
    with apk_b200.Context(dtype=dtype, ctas_per_sm=cps, k_tile=kt, poll="stage", set_mode="device",
                          max_events=events + 8, urgent_split_k=split) as c:
        info = c.info
        reason = _infeasible_reason(dtype, cps, kt, info)
        if reason:
            cell["infeasible"] = reason
            return cell
        A, B, Au, Bu = operands
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        tiles = (M // info["tile_m"]) * (-(-N // info["tile_n"]))
        # enough whole drains per timed launch for ~5 ms of work
        rate = 40e12 if dtype == "f32" else 1.0e15
        per = max(1, math.ceil(5e-3 * rate / (2.0 * M * N * K)))
        ms_poll, ms_off = c.run_overhead(tiles * per, reps=5)
        flops = 2.0 * M * N * K * per
        drain_ms = ms_off / per
        # the preempted drain must outlast the event schedule
        horizon_ms = 2.0 + events * 1.0 + 5.0
        bg_tasks = tiles * max(1, math.ceil(horizon_ms * 1.5 / drain_ms))
        clk = ClockSampler(c.cfg.device)
        clk.start()
        c.schedule_device_events([])
        c.launch(bg_tasks)
        c.wait(120)
        calm = c.run_stats()
        clk_calm = clk.stop()
        clk = ClockSampler(c.cfg.device)
        clk.start()
        r = c.run_latency(events=events, period_us=1000, seed=seed, warmup_events=warmup, settle_ms=2.0,
                          bg_tasks=bg_tasks, probe_reps=0)
        clk_pre = clk.stop()
        yields = c.run_stats()["yields"]
    cell.update({
        "grid": info["grid"], "tile": [info["tile_m"], info["tile_n"]], "stages": info["stages"],
        "slot_k": info["slot_k"], "yield_site_every_slots": kt // info["slot_k"],
        "kernel": ("warp-specialized (2 workers per 384-thread CTA)" if info["threads_per_cta"] == 384 else
                   f"{info['threads_per_cta']}-thread CTAs"),
        "urgent_split_k": split,
        "tflops_poll_off": flops / (ms_off / 1e3) / 1e12,
        "tflops_poll_stage": flops / (ms_poll / 1e3) / 1e12,
        "poll_cost_pct": (ms_poll / ms_off - 1.0) * 100.0,
        "events": r["n"], "unclaimed": r["unclaimed"], "anomalies": r["anomalies"],
        "yield_latency_p50_us": r["claim_p50_us"], "yield_latency_p99_us": r["claim_p99_us"],
        "flag_propagation_p50_us": r["last_obs_p50_us"], "flag_propagation_p99_us": r["last_obs_p99_us"],
        "urgent_done_p50_us": r["done_p50_us"], "urgent_done_p99_us": r["done_p99_us"],
        "tflops_sustained_undisturbed": calm["bg_tflops"], "tflops_under_preemption": r["bg_tflops"],
        "checkpoints": yields,
        "preemption_cost_pct": (1.0 - r["bg_tflops"] / calm["bg_tflops"]) * 100.0,
        "clocks_undisturbed": clk_calm, "clocks_preempted": clk_pre,
    })
    return cell


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--events", type=int, default=600)
    ap.add_argument("--warmup", type=int, default=100)
    ap.add_argument("--dtype", default="both", choices=("f32", "bf16", "both"))
    ap.add_argument("--seed", type=int, default=3)
    ap.add_argument("--cell", default=None, help="dtype,ctas,k_tile,M,N,K: run one cell in this process")
    args = ap.parse_args()

    if args.cell:
        import apk_b200
        d, cps, kt, M, N, K = args.cell.split(",")
        shape = (int(M), int(N), int(K))
        cell = run_cell(apk_b200, d, int(cps), int(kt), shape, args.events, args.warmup, args.seed,
                        _operands(apk_b200, d, *shape))
        print(json.dumps(cell), flush=True)
        return

    from apk_b200.clocks import gpu_identity
    print(json.dumps({"gpu": gpu_identity(0)}), flush=True)
    dtypes = ("f32", "bf16") if args.dtype == "both" else (args.dtype,)
    cells = []
    for dtype in dtypes:
        for shape in SHAPES:
            for cps in CTAS:
                for kt in KTILES:
                    spec = ",".join(map(str, (dtype, cps, kt) + shape))
                    out = subprocess.run(
                        [sys.executable, "-m", "apk_b200.config3", "--cell", spec, "--events", str(args.events),
                         "--warmup", str(args.warmup), "--seed", str(args.seed)],
                        capture_output=True, text=True)
                    if out.returncode != 0:
                        raise RuntimeError(f"cell {spec} failed:\n{out.stdout}\n{out.stderr}")
                    cell = json.loads(out.stdout.strip().splitlines()[-1])
                    cells.append(cell)
                    print(json.dumps(cell), flush=True)
    ran = [c for c in cells if "infeasible" not in c]
    print(f"# configs[3]: {len(ran)} of {len(cells)} cells ran")
    print("# dtype shape            CTAs/SM K-tile  TFLOP/s  poll%  yield p50/p99 us  propagation p50/p99 us"
          "  done p50 us  sustained TFLOP/s (MHz)  preempt%")
    for c in ran:
        print("# %-5s %-16s %7d %6d %8.1f %6.2f %7.2f / %-7.2f %9.2f / %-9.2f %9.2f %11.1f (%4.0f) %8.2f" % (
            c["dtype"], "x".join(map(str, c["shape"])), c["ctas_per_sm"], c["k_tile"], c["tflops_poll_off"],
            c["poll_cost_pct"], c["yield_latency_p50_us"], c["yield_latency_p99_us"],
            c["flag_propagation_p50_us"], c["flag_propagation_p99_us"], c["urgent_done_p50_us"],
            c["tflops_sustained_undisturbed"], c["clocks_undisturbed"]["sm_mhz"] or 0, c["preemption_cost_pct"]))


if __name__ == "__main__":
    main()
