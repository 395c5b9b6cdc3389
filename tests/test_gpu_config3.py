"""GPU parity tests of the configs[3] scaling-surface geometries, through the
C ABI.

* fp32 at 4 and 8 CTAs per SM runs 64x128 and 32x128 tiles (a CTA of two
  warps or one, the same 8x16 micro-tile and k order as the 128x128 tiles):
  C must be bitwise equal to the default kernel's, within 1e-5*sqrt(K) of the
  float64 oracle (src/persistent.cu:221-227).
* bf16 at 2, 4 and 8 CTAs per SM runs 256x128, 128x128 and 64x128 tiles with
  one TMEM buffer each: per element the same MMA sequence as the one-CTA
  kernel, so C is bitwise equal to it, and within 1e-2 of float64 over the
  rounded inputs (src/tcyield.cu:459-483).
* K-tile 64 and 128 place a stage-level yield site every K-tile / slot-depth
  ring slots: every mid-pipeline claim lands on such a site, and the
  checkpointed-and-resumed drain is bitwise equal to an uninterrupted one,
  with the exactly-once verdict of src/yield.cu:630-663.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def _ctx(**kw):
    import apk_b200
    return apk_b200.Context(**kw)


@pytest.mark.parametrize("cps,k_tile", [(4, 32), (8, 32), (4, 128), (8, 64)])
def test_f32_multi_cta_geometries_bitwise(libapk, cps, k_tile):
    M, N, K = 512, 384, 256
    A, B = oracle.gen_uniform(M, N, K, 3)
    with _ctx(poll="off") as c:
        C0 = c.gemm(A, B)
    with _ctx(poll="stage", ctas_per_sm=cps, k_tile=k_tile, oracle=True) as c:
        info = c.info
        assert info["ctas_per_sm"] == cps and info["grid"] == cps * info["sms"]
        assert (info["tile_m"], info["tile_n"], info["slot_k"]) == ((64 if cps == 4 else 32), 128, 16)
        assert info["threads_per_cta"] == info["tile_m"]
        C = c.gemm(A, B)
    assert np.array_equal(C.view(np.uint32), C0.view(np.uint32))
    mr, bad, nans = oracle.check(C, oracle.gemm_f64(A, B), oracle.fp32_tol(K))
    assert bad == 0 and nans == 0, f"{bad} bad, {nans} NaN, max rel {mr:.3e}"


def _f32_yield_run(cps, k_tile, nev=30, gap_ns=40_000):
    M = N = K = 2048
    A, B = oracle.gen_uniform(M, N, K, 21)
    Au, Bu = oracle.gen_uniform(256, 256, 256, 99)
    split = 256 // k_tile  # an urgent item is one K-tile deep
    with _ctx(poll="off") as c:
        C0 = c.gemm(A, B)
    with _ctx(poll="stage", set_mode="device", oracle=True, ctas_per_sm=cps, k_tile=k_tile,
              urgent_split_k=split) as c:
        info = c.info
        assert info["ctas_per_sm"] == cps and info["k_tile"] == k_tile
        tiles = (M // info["tile_m"]) * (N // info["tile_n"])
        ntasks = 3 * tiles
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_device_events((np.arange(nev, dtype=np.int64) + 1) * gap_ns)
        c.launch(ntasks)
        c.wait(120)
        out = dict(C=c.read_output(), ev=c.read_events(), st=c.run_stats(), info=info, C0=C0)
        out["ex"], out["ue"] = c.read_oracle(ntasks)
        fired = int(np.count_nonzero(out["ev"]["set_ns"][:nev]))
        out["outs"] = [c.read_urgent_output(e) for e in range(fired) if out["ev"]["claimer"][e]]
        out["uitems"] = (256 // info["tile_m"]) * (256 // info["tile_n"]) * split
        out["fired"] = fired
        out["refu"] = oracle.gemm_f64(Au, Bu)
    return out


@pytest.mark.parametrize("cps,k_tile", [(1, 128), (2, 64), (2, 128), (4, 64), (8, 128), (8, 32)])
def test_f32_k_tile_stage_yields_bitwise(libapk, cps, k_tile):
    r = _f32_yield_run(cps, k_tile)
    ev, fired = r["ev"], r["fired"]
    pe = k_tile // r["info"]["slot_k"]
    assert fired >= 15 and r["st"]["yields"] > 0
    sites = [int(ev["claim_site"][e]) for e in range(fired) if ev["claimer"][e]]
    assert any(s > 0 for s in sites), "no mid-pipeline claim"
    assert all(s == -1 or s % pe == 0 for s in sites), f"claims off the K-tile sites (every {pe}): {sites}"
    assert np.array_equal(r["C"].view(np.uint32), r["C0"].view(np.uint32)), "resume not bitwise"
    for Cu in r["outs"]:
        mr, bad, nans = oracle.check(Cu, r["refu"], oracle.fp32_tol(256))
        assert bad == 0 and nans == 0, f"urgent: {bad} bad, max rel {mr:.3e}"
    v = oracle.exactly_once(r["ex"], r["ue"][:fired], ev["claimer"][:fired], ev["set_ns"][:fired], r["uitems"],
                            fired)
    assert v["pass"], v


def _bf16_yield_run(k_tile, nev=30, gap_ns=20_000, **kw):
    import apk_b200
    M = N = K = 4096
    A = apk_b200.fill_normal_bf16((M, K), 21)
    B = apk_b200.fill_normal_bf16((K, N), 22)
    Au = apk_b200.fill_normal_bf16((256, 256), 31)
    Bu = apk_b200.fill_normal_bf16((256, 256), 32)
    with _ctx(dtype="bf16", poll="off", bf16_kernel="single") as c:
        C0 = c.gemm(A, B)
    with _ctx(dtype="bf16", poll="stage", set_mode="device", oracle=True, k_tile=k_tile, urgent_split_k=1,
              max_events=64, **kw) as c:
        info = c.info
        ntasks = 8 * (M // info["tile_m"]) * (N // info["tile_n"])
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_device_events((np.arange(nev, dtype=np.int64) + 1) * gap_ns)
        c.launch(ntasks)
        c.wait(60)
        out = dict(C=c.read_output(), ev=c.read_events(), st=c.run_stats(), info=info, C0=C0)
        out["ex"], out["ue"] = c.read_oracle(ntasks)
        fired = int(np.count_nonzero(out["ev"]["set_ns"][:nev]))
        out["outs"] = [c.read_urgent_output(e) for e in range(fired) if out["ev"]["claimer"][e]]
        out["uitems"] = (256 // info["tile_m"]) * (-(-256 // info["tile_n"]))
        out["fired"] = fired
    out["refu"] = oracle.gemm_f64_bf16_rows(Au, Bu, 0, 256)
    return out


def _check_bf16_yield(r, k_tile):
    ev, fired = r["ev"], r["fired"]
    pe = k_tile // r["info"]["slot_k"]
    assert fired >= 10 and r["st"]["yields"] > 0
    sites = [int(ev["claim_site"][e]) for e in range(fired) if ev["claimer"][e]]
    assert any(s > 0 for s in sites), "no mid-pipeline claim"
    assert all(s == -1 or s % pe == 0 for s in sites), f"claims off the K-tile sites (every {pe}): {sites}"
    assert np.array_equal(r["C"].view(np.uint32), r["C0"].view(np.uint32)), "resume not bitwise"
    for Cu in r["outs"]:
        mr, bad, nans = oracle.check(Cu, r["refu"], oracle.BF16_TOL)
        assert bad == 0 and nans == 0, f"urgent: {bad} bad, max rel {mr:.3e}"
    v = oracle.exactly_once(r["ex"], r["ue"][:fired], ev["claimer"][:fired], ev["set_ns"][:fired], r["uitems"],
                            fired)
    assert v["pass"], v


@pytest.mark.parametrize("bf16_kernel", ["pair", "single"])
def test_bf16_k_tile_128_stage_yields_bitwise(libapk, bf16_kernel):
    r = _bf16_yield_run(128, bf16_kernel=bf16_kernel)
    assert r["info"]["slot_k"] == 64
    _check_bf16_yield(r, 128)


@pytest.mark.parametrize("cps,k_tile", [(2, 64), (2, 32), (4, 64), (8, 128)])
def test_bf16_multi_cta_geometries_bitwise(libapk, cps, k_tile):
    import apk_b200
    M, N, K = 512, 384, 512
    A = apk_b200.fill_normal_bf16((M, K), 1)
    B = apk_b200.fill_normal_bf16((K, N), 2)
    with _ctx(dtype="bf16", poll="off", bf16_kernel="single") as c:
        C0 = c.gemm(A, B)
    with _ctx(dtype="bf16", poll="stage", ctas_per_sm=cps, k_tile=k_tile, oracle=True, urgent_split_k=1) as c:
        info = c.info
        assert info["ctas_per_sm"] == cps and info["grid"] == cps * info["sms"]
        assert (info["tile_m"], info["tile_n"]) == ({2: 256, 4: 128, 8: 64}[cps], 128)
        C = c.gemm(A, B)
    assert np.array_equal(C.view(np.uint32), C0.view(np.uint32))
    ref = oracle.gemm_f64_bf16_rows(A, B, 0, M)
    mr, bad, nans = oracle.check(C, ref, oracle.BF16_TOL)
    assert bad == 0 and nans == 0, f"{bad} bad, {nans} NaN, max rel {mr:.3e}"


@pytest.mark.parametrize("cps,k_tile", [(2, 64), (4, 128), (8, 32)])
def test_bf16_multi_cta_stage_yields_bitwise(libapk, cps, k_tile):
    r = _bf16_yield_run(k_tile, ctas_per_sm=cps)
    assert r["info"]["ctas_per_sm"] == cps
    _check_bf16_yield(r, k_tile)


@pytest.mark.parametrize("dtype,cps", [("f32", 4), ("f32", 8), ("bf16", 4), ("bf16", 8)])
def test_host_set_events_with_flag_copies(libapk, dtype, cps):
    """At 4 and 8 CTAs per SM the yield flag lives in 32 cache-line copies
    (CTA c polls copy c % 32): the host setter writes every copy in one
    copy-engine transfer and the stop writes -1 into all of them.  Host-set
    events on an unbounded launch stopped after the last one: every event
    claimed, none missed by any CTA, and the launch ends on the stop."""
    import apk_b200
    if dtype == "f32":
        A, B = oracle.gen_uniform(2048, 2048, 2048, 21)
        Au, Bu = oracle.gen_uniform(256, 256, 256, 99)
        kw = {"urgent_split_k": 8}
    else:
        A = apk_b200.fill_normal_bf16((4096, 4096), 21)
        B = apk_b200.fill_normal_bf16((4096, 4096), 22)
        Au = apk_b200.fill_normal_bf16((256, 256), 31)
        Bu = apk_b200.fill_normal_bf16((256, 256), 32)
        kw = {"dtype": "bf16", "urgent_split_k": 1}
    with _ctx(poll="stage", set_mode="host_memcpy", ctas_per_sm=cps, max_events=128, **kw) as c:
        assert c.info["ctas_per_sm"] == cps
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        r = c.run_latency(events=60, period_us=500, seed=5, warmup_events=10, probe_reps=0)
        st = c.run_stats()
    assert r["n"] == 50 and r["unclaimed"] == 0 and r["anomalies"] == 0, r
    assert st["device_status"] == 0
