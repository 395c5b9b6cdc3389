"""OBS1 observation dumps and the analyses run on them.

An OBS1 file (the reference's format, src/yield.cu:453-464) is little-endian
int64 throughout: the magic 0x3153424F ("OBS1"), the number of events E and
of CTAs G, then set_ns[E] (device globaltimer of each flag raise, 0 = never
raised) and obs_ns[E][G] (first observation of event e by CTA g, 0 = never).

Analyses, all deterministic (nearest-rank percentiles, a fixed warm-up cut,
a fixed half split), restated for this project's logs:

* `quantiles` -- per event the min / median / p95 / max delay across CTAs,
  then the p50 over events of each and the p99 of the max
  (src/yield.cu:529-560);
* `spread` -- last minus first observation per event and the first
  observer's delay (scripts/reanalyze_spread.py);
* `independent_max_model` -- the held-out independence model: the marginal of per-CTA
  delays is fitted on the first half of the events and the max over N CTAs
  predicted as F^N, against the measured max on the second half
  (scripts/heldout_maxofn.py);
* `floor_check` -- events whose max delay exceeds one timer quantum.

    python -m apk_b200.obs run [--loaded] [--events 1000] [--out vis.obs1]
    python -m apk_b200.obs latency [--events 600] [--out lat.obs1]
    python -m apk_b200.obs analyze FILE [--warmup 100] [--keep-setter]
"""
from __future__ import annotations

import argparse
import math
import json
import struct

import numpy as np

MAGIC = 0x3153424F


def write(path: str, set_ns, obs_ns) -> None:
    set_ns = np.ascontiguousarray(set_ns, "<i8")
    obs_ns = np.ascontiguousarray(obs_ns, "<i8")
    E, G = obs_ns.shape
    assert set_ns.shape == (E,)
    with open(path, "wb") as f:
        f.write(struct.pack("<3q", MAGIC, E, G))
        f.write(set_ns.tobytes())
        f.write(obs_ns.tobytes())


def read(path: str):
    with open(path, "rb") as f:
        magic, E, G = struct.unpack("<3q", f.read(24))
        if magic != MAGIC:
            raise ValueError(f"{path}: not an OBS1 file (magic {magic:#x})")
        set_ns = np.frombuffer(f.read(8 * E), "<i8").copy()
        obs_ns = np.frombuffer(f.read(8 * E * G), "<i8").reshape(E, G).copy()
    return set_ns, obs_ns


def pct(v, q):
    """Nearest rank, v[min(q*n, n-1)] of the sorted values."""
    v = sorted(v)
    return v[min(int(q * len(v)), len(v) - 1)] if v else float("nan")


def delays(set_ns, obs_ns, warmup: int = 100, skip_setter: bool = True):
    """Per-CTA delays (us) of every complete event at or after `warmup`;
    events never raised or not seen by every CTA are counted, not used."""
    lo = 1 if skip_setter else 0
    rows, unset, incomplete = [], 0, 0
    for e in range(len(set_ns)):
        if set_ns[e] == 0:
            unset += 1
            continue
        raw = obs_ns[e, lo:]
        if np.any(raw == 0):
            incomplete += 1
            continue
        if e < warmup:
            continue
        rows.append(((raw - set_ns[e]) / 1e3).tolist())
    return rows, unset, incomplete


def quantiles(rows):
    dmin = [min(r) for r in rows]
    d50 = [pct(r, 0.5) for r in rows]
    d95 = [pct(r, 0.95) for r in rows]
    dmax = [max(r) for r in rows]
    return {"n": len(rows), "dmin_p50_us": pct(dmin, 0.5), "d50_p50_us": pct(d50, 0.5),
            "d95_p50_us": pct(d95, 0.5), "dmax_p50_us": pct(dmax, 0.5), "dmax_p99_us": pct(dmax, 0.99)}


def spread(rows):
    first = [min(r) for r in rows]
    spr = [max(r) - min(r) for r in rows]
    return {"spread_p50_us": pct(spr, 0.5), "spread_p95_us": pct(spr, 0.95), "spread_p99_us": pct(spr, 0.99),
            "first_p50_us": pct(first, 0.5), "first_p99_us": pct(first, 0.99)}


def independent_max_model(rows, qs=(0.5, 0.9, 0.95, 0.99)):
    """Held-out test of whether CTAs observe a raise independently.  The
    per-CTA delays of the first half of the events give an empirical
    marginal F; if the N CTAs of an event observed independently, the
    event's last observation would follow F^N, whose q-quantile is F's
    q^(1/N)-quantile (read off the sorted marginal, no search).  The
    prediction is compared with the maxima measured on the second half."""
    n_cta = len(rows[0])
    n_fit = len(rows) // 2
    pooled = np.sort(np.asarray([d for r in rows[:n_fit] for d in r], dtype=np.float64))
    held_out_max = [max(r) for r in rows[n_fit:]]

    def predicted(q):
        # smallest pooled delay x with F(x) >= q^(1/N), F(x) = rank(x) / size
        rank = int(math.ceil(q ** (1.0 / n_cta) * pooled.size))
        return float(pooled[min(max(rank, 1), pooled.size) - 1])

    cta_medians = [pct([r[b] for r in rows], 0.5) for b in range(n_cta)]
    return {"N": n_cta, "fit_events": n_fit, "test_events": len(held_out_max),
            "quantiles": [{"q": q, "predicted_us": predicted(q), "measured_us": pct(held_out_max, q)}
                          for q in qs],
            "per_cta_median_us": {"min": min(cta_medians), "p50": pct(cta_medians, 0.5), "max": max(cta_medians)}}


def timer_quantum_us(set_ns, obs_ns) -> float:
    """Smallest positive step of the device clock seen in the matrix."""
    vals = np.unique(np.concatenate([set_ns[set_ns > 0], obs_ns[obs_ns > 0]]))
    steps = np.diff(vals)
    steps = steps[steps > 0]
    return float(steps.min()) / 1e3 if steps.size else float("nan")


def floor_check(rows, quantum_us: float):
    mx = [max(r) for r in rows]
    return {"events": len(rows), "absolute_max_us": max(mx) if mx else float("nan"),
            "events_over_one_quantum": sum(1 for m in mx if m > quantum_us * 1.03), "quantum_us": quantum_us}


def analyze(set_ns, obs_ns, warmup: int = 100, skip_setter: bool = True) -> dict:
    rows, unset, incomplete = delays(set_ns, obs_ns, warmup, skip_setter)
    out = {"events": int(len(set_ns)), "ctas": int(obs_ns.shape[1]), "unset": unset, "incomplete": incomplete}
    if rows:
        out.update(quantiles(rows))
        out.update(spread(rows))
        out["independent_max_model"] = independent_max_model(rows) if len(rows) >= 4 else None
        out["floor"] = floor_check(rows, timer_quantum_us(set_ns, obs_ns))
    return out


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run", help="visibility microbenchmark -> OBS1")
    r.add_argument("--events", type=int, default=1000)
    r.add_argument("--loaded", action="store_true")
    r.add_argument("--work-iters", type=int, default=0)
    r.add_argument("--dtype", default="f32", choices=("f32", "bf16"))
    r.add_argument("--out", default="visibility.obs1")
    la = sub.add_parser("latency", help="device-set latency run of the fp32 kernel -> OBS1")
    la.add_argument("--events", type=int, default=600)
    la.add_argument("--out", default="latency.obs1")
    an = sub.add_parser("analyze")
    an.add_argument("file")
    an.add_argument("--warmup", type=int, default=100)
    an.add_argument("--keep-setter", action="store_true")
    args = ap.parse_args()

    if args.cmd == "analyze":
        s, o = read(args.file)
        print(json.dumps(analyze(s, o, args.warmup, not args.keep_setter), indent=1))
        return
    import apk_b200
    if args.cmd == "run":
        with apk_b200.Context(dtype=args.dtype, poll="stage", set_mode="device") as c:
            res, s, o = c.run_visibility(events=args.events, loaded=args.loaded, work_iters=args.work_iters,
                                         raw=True)
        write(args.out, s, o)
        print(json.dumps({"summary": res, "file": args.out}))
    else:
        A, B = apk_b200.fill_uniform(4096, 4096, 4096, 21)
        Au, Bu = apk_b200.fill_uniform(256, 256, 256, 99)
        with apk_b200.Context(poll="stage", set_mode="device", max_events=args.events + 8) as c:
            c.set_background(A, B)
            c.set_urgent(Au, Bu)
            res = c.run_latency(events=args.events, period_us=1000, seed=3, warmup_events=0, settle_ms=2.0,
                                probe_reps=0)
            ev = c.read_events()
        write(args.out, ev["set_ns"][:args.events], ev["obs_ns"][:args.events])
        print(json.dumps({"claim_p50_us": res["claim_p50_us"], "file": args.out}))


if __name__ == "__main__":
    main()
