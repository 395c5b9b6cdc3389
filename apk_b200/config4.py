"""the scheduler oracle under multi-GPU.

    python -m apk_b200.config4 [--tasks 1048576]                 # one GPU
    torchrun --nproc-per-node N -m apk_b200.config4 [--tasks ...] # N GPUs

A queue of bf16 GEMM tasks (m, n log-uniform in [128, 2048] to multiples of
128, k log-uniform in [256, 4096] to multiples of 64, N(0,1) operands) is
generated from one seed on every rank and statically sharded (LPT by
2*m*n*k); each GPU drains its own shard with its own persistent kernel --
no collective, no peer access in the data path.  Every rank runs its shard
three times: a warm-up drain, an undisturbed drain, then a drain with urgent
256^3 GEMMs arriving as a Poisson stream (2 kHz per GPU) injected by the
host.  Arrivals are scheduled over the first 80% of the undisturbed drain's
time, so each lands while the rank's CTAs are still draining.  Verdicts:

* exactly once: the ranks' per-tile execution counters of both measured
  drains, summed over ranks (host side, after the timed runs), are 1 for
  every global 256x128 half-tile;
* zero corrupted outputs: every half-tile's checksum sum(c^2) is bitwise
  equal between the undisturbed and the preempted drain, and every urgent
  output's checksum equals the first one's;
* aggregate TFLOP/s = sum of the ranks' task FLOPs / the slowest rank's
  CUDA-event launch time.

The bounded-run verdict restates the reference's oracle run
(src/yield.cu:576-667: every task executed once, every event's urgent work
executed U times, every event claimed).  torch.distributed (gloo) is used
only to gather results on the host after the timed drains.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics

ARRIVAL_SPAN = 0.8  # arrivals are scheduled over this fraction of the drain


def run_rank(local: int, world: int, rank: int, n_tasks: int = 1 << 20, seed: int = 21, rate_hz: float = 2000.0,
             narrow_k: int = 0):
    """Drain this rank's shard undisturbed and under Poisson urgent arrivals.
    Returns (result dict, exec counts of the undisturbed drain, of the
    preempted drain) -- the counts are int32 arrays over every global
    half-tile, zero outside this rank's shard when the shard is clean."""
    import numpy as np

    import apk_b200
    from apk_b200.runtime import POOL, gen_tasks, shard_tasks

    tasks, n_chk = gen_tasks(n_tasks, seed)
    if narrow_k > 0:
        tasks["flags"] |= np.where(tasks["k"] < narrow_k, 2, 0).astype(tasks["flags"].dtype)
    mine = shard_tasks(tasks, world, rank)
    my_tasks = tasks[mine]
    my_flops = float((2.0 * my_tasks["m"].astype(np.float64) * my_tasks["n"] * my_tasks["k"]).sum())
    A = apk_b200.fill_normal_bf16((POOL["a_rows"], POOL["a_cols"]), 101)
    B = apk_b200.fill_normal_bf16((POOL["b_rows"], POOL["b_cols"]), 102)
    Au = apk_b200.fill_normal_bf16((256, 256), 31)
    Bu = apk_b200.fill_normal_bf16((256, 256), 32)

    period_us = 1e6 / rate_hz
    with apk_b200.Context(device=local, dtype="bf16", poll="stage", set_mode="host_memcpy", oracle=True,
                          urgent_split_k=1, max_events=16384) as c:
        c.set_task_pool(A, B, POOL["c_rows"], POOL["c_cols"])
        c.set_urgent(Au, Bu)
        nw = c.set_tasks(my_tasks, n_chk)
        c.launch(nw)  # warm-up drain
        c.wait(600)
        c.launch(nw)
        c.wait(600)
        st0 = c.run_stats()
        chk0 = c.read_checksums()
        ex0, _ = c.read_oracle(n_chk)
        # preempted drain: Poisson urgent arrivals over the first 80% of the
        # undisturbed drain's time (the last arrival lands while CTAs drain)
        est_s = st0["launch_ms"] / 1e3
        events = max(1, min(16000, int(est_s * ARRIVAL_SPAN * rate_hz)))
        r = c.run_latency(events=events, period_us=period_us, seed=seed + rank, settle_ms=0.0,
                          bg_tasks=nw, probe_reps=0, poisson=True)
        st1 = c.run_stats()
        chk1 = c.read_checksums()
        ex1, ue = c.read_oracle(n_chk)
        ev = c.read_events()
        n_inj = ev["n_injected"]
        claimed = int(np.count_nonzero(ev["claimer"][:n_inj]))
        outs = [c.read_urgent_output(e) for e in range(n_inj) if ev["claimer"][e]]
        uitems = (256 // c.info["tile_m"]) * (-(-256 // c.info["tile_n"]))
    uchk = [float((o.astype(np.float64) ** 2).sum()) for o in outs]
    own = np.zeros(n_chk, bool)
    for d in my_tasks:
        nt = ((int(d["m"]) + 255) // 256) * (int(d["n"]) // 128)
        own[int(d["chk_base"]):int(d["chk_base"]) + nt] = True
    res = {
        "rank": rank, "tasks": int(len(mine)), "jobs": int(nw), "halves": int(own.sum()), "n_chk": int(n_chk),
        "flops": my_flops, "ms_undisturbed": st0["launch_ms"], "ms_preempted": st1["launch_ms"],
        "exactly_once_local": bool(np.all(ex0[own] == 1) and np.all(ex0[~own] == 0) and np.all(ex1[own] == 1)
                                   and np.all(ex1[~own] == 0)),
        "corrupted": int(np.count_nonzero(chk0[own].view(np.uint64) != chk1[own].view(np.uint64))),
        "arrivals": int(n_inj), "claimed": claimed,
        "urgent_consistent": bool(all(u == uchk[0] for u in uchk)) if uchk else True,
        "urgent_items_exact": bool(all(ue[e] == uitems for e in range(n_inj) if ev["claimer"][e])),
        "checkpoints": int(st1["yields"]),
        "rt_claim_p50_us": r["rt_claim_p50_us"], "rt_claim_p99_us": r["rt_claim_p99_us"],
        "rt_done_p50_us": r["rt_done_p50_us"],
    }
    return res, ex0, ex1


def union_counts(world: int, ex0, ex1):
    """Per-half-tile execution counts summed over ranks (both drains), on
    every rank.  Counts are capped at 15 per rank before the sum so they fit
    a byte at 8 ranks; any count other than 1 fails the verdict either way."""
    import numpy as np
    c = np.minimum(np.stack([ex0, ex1]), 15).astype(np.uint8)
    if world > 1:
        import torch
        import torch.distributed as dist
        t = torch.from_numpy(c)
        dist.all_reduce(t)
        c = t.numpy()
    return c


def summarize(allr, counts, n_tasks: int) -> dict:
    """The configs[4] verdict over all ranks (rank 0)."""
    import numpy as np
    tmax0 = max(x["ms_undisturbed"] for x in allr) / 1e3
    tmax1 = max(x["ms_preempted"] for x in allr) / 1e3
    tot = sum(x["flops"] for x in allr)
    return {
        "n_gpus": len(allr), "tasks": n_tasks, "halves": allr[0]["n_chk"], "pflop": tot / 1e15,
        "tflops_undisturbed": tot / tmax0 / 1e12, "tflops_preempted": tot / tmax1 / 1e12,
        "exactly_once": bool(np.all(counts == 1)) and all(x["exactly_once_local"] for x in allr),
        "corrupted": sum(x["corrupted"] for x in allr),
        "arrivals": sum(x["arrivals"] for x in allr), "urgent_claimed": sum(x["claimed"] for x in allr),
        "urgent_outputs_ok": all(x["urgent_consistent"] and x["urgent_items_exact"] for x in allr),
        "checkpoints": sum(x["checkpoints"] for x in allr),
        "rt_claim_p50_us": statistics.median(x["rt_claim_p50_us"] for x in allr),
        "ms_max": tmax0 * 1e3, "ms_min": min(x["ms_undisturbed"] for x in allr),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tasks", type=int, default=1 << 20)
    ap.add_argument("--seed", type=int, default=21)
    ap.add_argument("--rate-hz", type=float, default=2000.0)
    ap.add_argument("--narrow-k", type=int, default=0,
                    help="tasks with k below this run as 256x128 tiles (APK_TASK_NARROW)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    res, ex0, ex1 = run_rank(local, world, rank, args.tasks, args.seed, args.rate_hz, args.narrow_k)
    counts = union_counts(world, ex0, ex1)
    if world > 1:
        import torch.distributed as dist
        allr = [None] * world
        dist.all_gather_object(allr, res)
    else:
        allr = [res]
    if rank == 0:
        out = summarize(allr, counts, args.tasks)
        out["per_rank"] = [{k: x[k] for k in ("rank", "tasks", "jobs", "ms_undisturbed", "ms_preempted")}
                           for x in allr]
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
