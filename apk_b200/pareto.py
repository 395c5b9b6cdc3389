"""Reserved capacity versus cooperative hand-off (the reference's A3
experiment, scripts/pareto.sh and src/urgent_baseline.cu:152-175).

    python -m apk_b200.pareto [--trials 100] [--events 300]

Background: the configs[1] fp32 4096^3 persistent drain.  Urgent job: an
fp32 GEMM of U 128x128 tiles (U = 1, 4, 16: 128x128, 256x256, 512x512
outputs, K = 256), uniform[-1,1] from the reference generator.

* Reserved arm: the background runs on the full-residency grid minus R
  CTAs (R = 0, 1, 2, 4, 8, 16, 32; R = 0 is the no-preemption baseline); the
  urgent job is a separate kernel of U CTAs on a max-priority stream
  launched at U(0.2, 0.8) of the drain.  y: host arrival -> urgent done
  (host clock); x: the background's TFLOP/s with R slots held out.
* Priority arm (cluster launch control): the background grid is one CTA
  per task, scheduled by CLC work stealing with nothing held out; the urgent
  kernel is launched on the max-priority stream as in the reserved arm.
  While it waits the hardware declines the background's requests, CTAs exit
  at their next tile boundary and it takes their SMs.
* Cooperative arm: the full grid polls every stage; the host stores the
  yield flag once per 1 ms at a uniform offset and the urgent tiles are
  popped by the CTAs that observe it (split-K 1: U items).  y: host store ->
  host sees the last urgent item's done ack (host clock, the same endpoints
  as the reserved arm); x: background TFLOP/s under the injections.

One JSON line per point, then a summary table.
"""
from __future__ import annotations

import argparse
import json

RESERVE = (0, 1, 2, 4, 8, 16, 32)
URGENT_TILES = (1, 4, 16)
SIDE = {1: 128, 4: 256, 16: 512}


def _pct(v, q):
    v = sorted(v)
    return v[min(int(q * len(v)), len(v) - 1)] if v else float("nan")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--trials", type=int, default=100)
    ap.add_argument("--events", type=int, default=300)
    ap.add_argument("--bg-tasks", type=int, default=4096)
    args = ap.parse_args()

    import apk_b200
    from apk_b200.clocks import gpu_identity

    print(json.dumps({"gpu": gpu_identity(0)}), flush=True)
    A, B = apk_b200.fill_uniform(4096, 4096, 4096, 21)
    urgent = {u: apk_b200.fill_uniform(SIDE[u], SIDE[u], 256, 99) for u in URGENT_TILES}
    rows = []
    for u in URGENT_TILES:
        Au, Bu = urgent[u]
        with apk_b200.Context(poll="off", urgent_split_k=1) as c:
            c.set_background(A, B)
            c.set_urgent(Au, Bu)
            for r in RESERVE:
                e2e, tf = c.run_reserved(args.bg_tasks, r, args.trials, seed=21)
                row = {"arm": "reserved", "urgent_tiles": u, "reserve": r, "bg_tflops": tf,
                       "e2e_p50_us": _pct(e2e, 0.5), "e2e_p99_us": _pct(e2e, 0.99), "trials": len(e2e)}
                rows.append(row)
                print(json.dumps(row), flush=True)
        with apk_b200.Context(poll="off", urgent_split_k=1, scheduler="clc") as c:
            c.set_background(A, B)
            c.set_urgent(Au, Bu)
            e2e, tf = c.run_reserved(args.bg_tasks, 0, args.trials, seed=21)
            row = {"arm": "clc_priority", "urgent_tiles": u, "reserve": 0, "bg_tflops": tf,
                   "e2e_p50_us": _pct(e2e, 0.5), "e2e_p99_us": _pct(e2e, 0.99), "trials": len(e2e)}
            rows.append(row)
            print(json.dumps(row), flush=True)
        with apk_b200.Context(poll="stage", set_mode="host_memcpy", urgent_split_k=1,
                              max_events=args.events + 8) as c:
            c.set_background(A, B)
            c.set_urgent(Au, Bu)
            lat = c.run_latency(events=args.events, period_us=1000, seed=7, warmup_events=0, settle_ms=2.0,
                                probe_reps=0)
            row = {"arm": "cooperative", "urgent_tiles": u, "reserve": 0, "bg_tflops": lat["bg_tflops"],
                   "e2e_p50_us": lat["rt_done_p50_us"], "e2e_p99_us": lat["rt_done_p99_us"],
                   "claim_p50_us": lat["rt_claim_p50_us"], "claim_p99_us": lat["rt_claim_p99_us"],
                   "events": lat["n"], "unclaimed": lat["unclaimed"]}
            rows.append(row)
            print(json.dumps(row), flush=True)
    print("# arm          U   R   bg TFLOP/s   urgent e2e p50 / p99 us")
    for r in rows:
        print("# %-11s %3d %3d %10.1f   %10.1f / %.1f" % (r["arm"], r["urgent_tiles"], r["reserve"],
                                                      r["bg_tflops"], r["e2e_p50_us"], r["e2e_p99_us"]))


if __name__ == "__main__":
    main()
