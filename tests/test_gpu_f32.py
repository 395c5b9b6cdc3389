"""GPU parity tests of the fp32 persistent SGEMM path, through the C ABI.

Every check compares against the CPU oracle (float64 restatement of the
reference's host GEMM, src/persistent.cu:221-227) with the north-star
tolerance rel = |got-ref|/max(1,|ref|) <= 1e-5*sqrt(K), or bitwise against an
uninterrupted run of the same kernel (checkpoint/resume), or against the
exactly-once verdict of src/yield.cu:630-663.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

U_M = U_N = U_K = 256  # the urgent GEMM of the configurations


def _ctx(**kw):
    import apk_b200
    return apk_b200.Context(**kw)


def _urgent_ref():
    Au, Bu = oracle.gen_uniform(U_M, U_N, U_K, 99)
    return Au, Bu, oracle.gemm_f64(Au, Bu)


def _check(C, ref, K):
    mr, bad, nans = oracle.check(C, ref, oracle.fp32_tol(K))
    assert nans == 0, f"{nans} NaN (never-written) elements"
    assert bad == 0, f"{bad} elements beyond 1e-5*sqrt(K); max rel {mr:.3e}"
    return mr


def test_info_full_residency(libapk):
    with _ctx() as c:
        info = c.info
    assert info["cc_major"] == 10
    assert info["sms"] >= 100
    assert info["ctas_per_sm"] == info["max_ctas_per_sm"] >= 2
    assert info["grid"] == info["sms"] * info["ctas_per_sm"]


def test_verify_1024_no_yield(libapk):
    """configs[0] shape, plain drain, NaN pre-fill."""
    A, B = oracle.gen_uniform(1024, 1024, 1024, 21)
    with _ctx(poll="off", oracle=True) as c:
        C = c.gemm(A, B)
    ref = oracle.gemm_f64(A, B)
    _check(C, ref, 1024)


@pytest.mark.parametrize("shape", [(384, 640, 96), (1152, 1536, 256), (128, 128, 32)])
def test_streamed_gemm_ragged_shapes(libapk, shape):
    """apk_gemm from host memory: the copy plan interleaves A row panels and
    B column panels, the kernel visits tiles in the order they become
    computable and C blocks come back as they finish.  Shapes with a partial
    row panel, B panels of one 128-column unit (N % 512 != 0) and a single
    tile."""
    M, N, K = shape
    A, B = oracle.gen_uniform(M, N, K, 5)
    with _ctx(poll="stage", oracle=True) as c:
        C = c.gemm(A, B)
    _check(C, oracle.gemm_f64(A, B), K)


def test_streamed_k_slices_under_stage_yields(libapk):
    """apk_gemm from host memory takes K in two chained slices (slice 1
    starts from the accumulators slice 0 handed off).  Device-set yields
    every 20 us checkpoint jobs of both slices mid-pipeline; C must still be
    bitwise equal to a resident drain, every (tile, slice) job run exactly
    once, every urgent output correct."""
    M = N = K = 2048
    A, B = oracle.gen_uniform(M, N, K, 31)
    Au, Bu, refu = _urgent_ref()
    ntiles = (M // 128) * (N // 128)
    with _ctx(poll="off") as c:
        c.set_background(A, B)
        c.launch(ntiles)
        c.wait(60)
        C0 = c.read_output()
    nev = 40
    offs = (np.arange(nev, dtype=np.int64) + 1) * 20_000
    with _ctx(poll="stage", set_mode="device", oracle=True) as c:
        c.set_urgent(Au, Bu)
        c.schedule_device_events(offs)
        C = c.gemm(A, B)
        ev = c.read_events()
        st = c.run_stats()
        ex, ue = c.read_oracle(2 * ntiles)
        outs = [c.read_urgent_output(e) for e in range(nev) if ev["claimer"][e]]
        uitems = (U_M // 128) * (U_N // 128) * c.cfg.urgent_split_k
    fired = int(np.count_nonzero(ev["set_ns"][:nev]))
    assert fired >= 10 and st["yields"] > 0 and st["device_status"] == 0
    assert st["tiles_done"] == ntiles  # tiles, not slices
    assert np.array_equal(C.view(np.uint32), C0.view(np.uint32)), "K-sliced streamed run not bitwise"
    assert np.all(ex == 1), "a (tile, slice) job ran other than once"
    for Cu in outs:
        _check(Cu, refu, U_K)
    v = oracle.exactly_once(ex, ue[:fired], ev["claimer"][:fired], ev["set_ns"][:fired], uitems, fired)
    assert v["pass"], v


def test_fp32_kernels_bitwise_equal(libapk):
    """The warp-specialized and the block-synchronous fp32 kernels run the
    same FMA sequence per element: bitwise-equal C, both within tolerance."""
    A, B = oracle.gen_uniform(1024, 1536, 768, 23)
    out = {}
    for k in ("ws", "sync"):
        with _ctx(poll="stage", f32_kernel=k) as c:
            out[k] = c.gemm(A, B)
            if k == "ws":
                assert c.info["threads_per_cta"] == 384
    assert np.array_equal(out["ws"].view(np.uint32), out["sync"].view(np.uint32))
    _check(out["ws"], oracle.gemm_f64(A, B), 768)


def test_cfg0_yield_at_50_percent_boundary(libapk):
    """1024^3 fp32, one yield at a tile boundary after 50% of the
    64 tiles complete; C within tolerance and bitwise equal to the no-yield
    run; the urgent output within tolerance; the event claimed."""
    A, B = oracle.gen_uniform(1024, 1024, 1024, 21)
    Au, Bu, refu = _urgent_ref()
    with _ctx(poll="off", oracle=True) as c:
        C0 = c.gemm(A, B)
    with _ctx(poll="boundary", set_mode="device", oracle=True) as c:
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_count_events([32])
        c.launch(64)
        c.wait(60)
        C = c.read_output()
        ev = c.read_events()
        ex, ue = c.read_oracle(64)
        Cu = c.read_urgent_output(0)
        uitems = (U_M // 128) * (U_N // 128) * c.cfg.urgent_split_k
    assert ev["set_ns"][0] != 0 and ev["claimer"][0] != 0
    assert ev["claim_site"][0] == -1  # tile boundary
    _check(C, oracle.gemm_f64(A, B), 1024)
    assert np.array_equal(C.view(np.uint32), C0.view(np.uint32))
    _check(Cu, refu, U_K)
    v = oracle.exactly_once(ex, ue[:1], ev["claimer"][:1], ev["set_ns"][:1], uitems, 1)
    assert v["pass"], v


def test_stage_checkpoint_resume_is_bitwise(libapk):
    """Mid-pipeline yields: in-flight TMA stages drained, accumulators spilled
    to the slab and restored; C must be bitwise identical to an uninterrupted
    run and every urgent output correct."""
    M = N = K = 2048
    A, B = oracle.gen_uniform(M, N, K, 21)
    Au, Bu, refu = _urgent_ref()
    with _ctx(poll="off") as c:
        c.set_background(A, B)
        c.launch(c.info["grid"] * 3)  # cycled tiles, same values
        c.wait(60)
        C0 = c.read_output()
    nev = 40
    offs = (np.arange(nev, dtype=np.int64) + 1) * 37_000  # every 37 us
    with _ctx(poll="stage", set_mode="device", oracle=True) as c:
        grid = c.info["grid"]
        ntasks = grid * 3
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_device_events(offs)
        c.launch(ntasks)
        c.wait(120)
        C = c.read_output()
        ev = c.read_events()
        ex, ue = c.read_oracle(ntasks)
        st = c.run_stats()
        outs = [c.read_urgent_output(e) for e in range(nev) if ev["claimer"][e]]
        uitems = (U_M // 128) * (U_N // 128) * c.cfg.urgent_split_k
    fired = int(np.count_nonzero(ev["set_ns"][:nev]))
    assert fired >= nev // 2, "the drain ended before most events fired"
    assert st["yields"] > 0
    mid = [e for e in range(nev) if ev["claimer"][e] and ev["claim_site"][e] >= 0]
    assert mid, "no claim landed mid-pipeline"
    assert any(ev["inflight"][e] > 0 for e in mid), "no buffer-conflicting yield"
    assert np.array_equal(C.view(np.uint32), C0.view(np.uint32)), "resume not bitwise"
    for Cu in outs:
        _check(Cu, refu, U_K)
    v = oracle.exactly_once(ex, ue[:fired], ev["claimer"][:fired], ev["set_ns"][:fired], uitems, fired)
    assert v["pass"], v


def test_back_to_back_yields_bitwise(libapk):
    """Yields 4 us apart: a second yield often lands while the first one's
    urgent items run, before the background tile has resumed.  The tile must
    still resume from its own checkpoint (not from an urgent item's
    accumulators): C bitwise equal to an uninterrupted run."""
    M = N = K = 2048
    A, B = oracle.gen_uniform(M, N, K, 21)
    Au, Bu, refu = _urgent_ref()
    with _ctx(poll="off") as c:
        c.set_background(A, B)
        c.launch(c.info["grid"] * 3)
        c.wait(60)
        C0 = c.read_output()
    nev = 30
    offs = 20_000 + np.arange(nev, dtype=np.int64) * 4_000
    with _ctx(poll="stage", set_mode="device", oracle=True, max_events=64) as c:
        ntasks = c.info["grid"] * 3
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_device_events(offs)
        c.launch(ntasks)
        c.wait(120)
        C = c.read_output()
        ev = c.read_events()
        ex, ue = c.read_oracle(ntasks)
        st = c.run_stats()
        outs = [c.read_urgent_output(e) for e in range(nev) if ev["claimer"][e]]
        uitems = (U_M // 128) * (U_N // 128) * c.cfg.urgent_split_k
    fired = int(np.count_nonzero(ev["set_ns"][:nev]))
    assert fired == nev and st["yields"] > 0
    assert np.array_equal(C.view(np.uint32), C0.view(np.uint32)), "resume not bitwise"
    for Cu in outs:
        _check(Cu, refu, U_K)
    v = oracle.exactly_once(ex, ue[:fired], ev["claimer"][:fired], ev["set_ns"][:fired], uitems, fired)
    assert v["pass"], v


def test_poison_discipline_is_detected(libapk):
    """Positive control (src/midyield.cu:146-147): a corrupted staged urgent
    value must make every claimed event's urgent output fail the check."""
    A, B = oracle.gen_uniform(1024, 1024, 2048, 21)
    Au, Bu, refu = _urgent_ref()
    nev = 8
    with _ctx(poll="stage", discipline="poison", set_mode="device") as c:
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_device_events((np.arange(nev, dtype=np.int64) + 1) * 40_000)
        c.launch(c.info["grid"] * 4)
        c.wait(60)
        ev = c.read_events()
        outs = [c.read_urgent_output(e) for e in range(nev) if ev["claimer"][e]]
    assert outs
    for Cu in outs:
        _, bad, _ = oracle.check(Cu, refu, oracle.fp32_tol(U_K))
        assert bad > 0


def test_host_mapped_injection_and_acks(libapk):
    """The mapped-memory host path (slow by design: every CTA polls across
    PCIe) still claims and completes every event correctly."""
    A, B = oracle.gen_uniform(1024, 1024, 1024, 21)
    Au, Bu, refu = _urgent_ref()
    with _ctx(poll="stage", set_mode="host_mapped", max_events=64) as c:
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.launch(None)
        for _ in range(20):
            e, _t = c.inject()
            assert c.wait_ack(e, 0, 200_000_000) is not None
            assert c.wait_ack(e, 1, 200_000_000) is not None
        c.stop()
        c.wait(30)
        ev = c.read_events()
        outs = [c.read_urgent_output(e) for e in range(20)]
        st = c.run_stats()
    assert ev["n_injected"] == 20
    assert all(ev["claimer"][:20] != 0)
    for Cu in outs:
        _check(Cu, refu, U_K)
    assert st["tiles_done"] > 0 and st["device_status"] == 0


def test_host_memcpy_injection(libapk):
    A, B = oracle.gen_uniform(1024, 1024, 1024, 21)
    Au, Bu, refu = _urgent_ref()
    with _ctx(poll="stage", set_mode="host_memcpy", max_events=16) as c:
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.launch(None)
        for _ in range(5):
            e, _t = c.inject()
            assert c.wait_ack(e, 1, 500_000_000) is not None
        c.stop()
        c.wait(30)
        ev = c.read_events()
        Cu = c.read_urgent_output(4)
    assert all(ev["claimer"][:5] != 0)
    _check(Cu, refu, U_K)


def test_oracle_exactly_once_bounded_run(libapk):
    """A bounded run with many events: every task id exactly once, every
    fired event exactly uitems urgent executions and a claimer."""
    A, B = oracle.gen_uniform(1024, 1024, 512, 5)
    Au, Bu, _ = _urgent_ref()
    nev = 60
    with _ctx(poll="stage", set_mode="device", oracle=True) as c:
        ntasks = 20000
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_device_events((np.arange(nev, dtype=np.int64) + 1) * 25_000)
        c.launch(ntasks)
        c.wait(120)
        ev = c.read_events()
        ex, ue = c.read_oracle(ntasks)
        C = c.read_output()
        uitems = (U_M // 128) * (U_N // 128) * c.cfg.urgent_split_k
    fired = int(np.count_nonzero(ev["set_ns"][:nev]))
    assert fired > 10
    v = oracle.exactly_once(ex, ue[:fired], ev["claimer"][:fired], ev["set_ns"][:fired], uitems, fired)
    assert v["pass"], v
    _check(C, oracle.gemm_f64(A, B), 512)


def test_config1_shape_sampled_rows(libapk):
    """configs[1] background shape 4096^3 (K-tile 32), checked on sampled
    row bands against float64."""
    M = N = K = 4096
    A, B = oracle.gen_uniform(M, N, K, 21)
    with _ctx(poll="stage", oracle=True) as c:
        C = c.gemm(A, B)
    for r0 in (0, 1000, 2048 + 64, 4096 - 16):
        ref = oracle.gemm_f64_rows(A, B, r0, 16)
        _check(C[r0:r0 + 16], ref, K)


def test_k_tile_64_variant(libapk):
    A, B = oracle.gen_uniform(512, 768, 1024, 11)
    with _ctx(poll="stage", k_tile=64, oracle=True) as c:
        C = c.gemm(A, B)
    _check(C, oracle.gemm_f64(A, B), 1024)


def test_bounded_wait_reports_instead_of_hanging(libapk):
    """A spin on a flag nothing sets must give up, report status 3 and leave
    the context usable."""
    A, B = oracle.gen_uniform(256, 256, 256, 1)
    with _ctx(poll="off") as c:
        assert c.selftest_wait_timeout(50_000_000) == 3
        C = c.gemm(A, B)
    _check(C, oracle.gemm_f64(A, B), 256)


def test_latency_mode_smoke(libapk):
    """Latency mode (src/yield.cu:776-958) on a short run: every event
    claimed, none missed by any CTA."""
    A, B = oracle.gen_uniform(4096, 4096, 4096, 21)
    Au, Bu, _ = _urgent_ref()
    with _ctx(poll="stage", set_mode="host_memcpy", max_events=256) as c:
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        r = c.run_latency(events=100, period_us=1000, seed=21, warmup_events=10)
    assert r["n"] == 90 and r["unclaimed"] == 0 and r["anomalies"] == 0
    assert r["rt_claim_p50_us"] < 60
    assert r["bg_tflops"] > 1.0


def test_reserved_capacity_arm(libapk):
    """Reserved-capacity arm (src/urgent_baseline.cu:152-175): with R free
    resident slots the urgent kernel starts at once instead of waiting for
    the drain (R = 0, the no-preemption baseline); holding slots out costs
    background throughput roughly in proportion."""
    A, B = oracle.gen_uniform(4096, 4096, 4096, 21)
    Au, Bu, _ = _urgent_ref()
    with _ctx(poll="off", urgent_split_k=1) as c:
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        grid = c.info["grid"]
        e0, tf0 = c.run_reserved(4096, 0, 8, seed=3)
        e4, tf4 = c.run_reserved(4096, 4, 8, seed=3)
        assert c.info["grid"] == grid  # the reduced grid is restored
        with pytest.raises(Exception):
            c.run_reserved(4096, grid, 2)
    assert np.all(e0 > 0) and np.all(e4 > 0)
    assert np.median(e4) * 5 < np.median(e0), (np.median(e4), np.median(e0))
    assert 0 < tf4 <= tf0 * 1.02 and tf4 > tf0 * 0.9


@pytest.mark.parametrize("loaded", [False, True])
def test_visibility_probe(libapk, loaded):
    """Flag-visibility microbenchmark (src/yield.cu:227-293): every raise
    seen by every CTA, the run ends by itself, the C++ summary matches the
    OBS1 analysis of the same matrix, the loaded variant keeps HBM busy."""
    from apk_b200 import obs
    with _ctx(poll="stage", set_mode="device") as c:
        res, s, o = c.run_visibility(events=200, warmup_events=20, loaded=loaded, raw=True)
        grid = c.info["grid"]
    assert res["device_status"] == 0 and res["unset"] == 0 and res["anomalies"] == 0
    assert res["n"] == 180 and res["cadence_ns"] > 0
    assert o.shape == (200, grid)
    a = obs.analyze(s, o, warmup=20)
    for k in ("dmin_p50_us", "d50_p50_us", "d95_p50_us", "dmax_p50_us", "dmax_p99_us"):
        assert abs(a[k] - res[k]) < 1e-9, k
    assert res["dmax_p99_us"] < 1000.0
    if loaded:
        assert res["hbm_gbs"] > 1000.0


def test_clc_scheduler_drain_exactly_once(libapk):
    """Cluster-launch-control scheduler: one CTA per task, running CTAs take
    the pending ones; every task exactly once, output within tolerance."""
    A, B = oracle.gen_uniform(1024, 1024, 1024, 21)
    ref = oracle.gemm_f64(A, B)
    with _ctx(poll="off", oracle=True, scheduler="clc") as c:
        C = c.gemm(A, B)
        st = c.run_stats()
        c.set_background(A, B)
        c.set_urgent(*oracle.gen_uniform(U_M, U_N, U_K, 99))
        c.launch(3 * 64)
        c.wait(30)
        ex, _ = c.read_oracle(3 * 64)
    _check(C, ref, 1024)
    assert st["tiles_done"] == 64 and st["device_status"] == 0
    assert np.all(ex == 1)


def test_clc_stage_yields_bitwise(libapk):
    """CLC scheduler with per-stage device-set yields: checkpoint/resume is
    bitwise and every task and urgent item runs exactly once."""
    A, B = oracle.gen_uniform(4096, 4096, 4096, 21)
    Au, Bu, refu = _urgent_ref()
    with _ctx(poll="off") as c:
        Cref = c.gemm(A, B)
    nev = 20
    with _ctx(poll="stage", set_mode="device", oracle=True, scheduler="clc") as c:
        ntasks = 2048
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_device_events((np.arange(nev, dtype=np.int64) + 1) * 150_000)
        c.launch(ntasks)
        c.wait(60)
        C = c.read_output()
        ev = c.read_events()
        st = c.run_stats()
        ex, ue = c.read_oracle(ntasks)
        fired = int(np.count_nonzero(ev["set_ns"][:nev]))
        outs = [c.read_urgent_output(e) for e in range(fired) if ev["claimer"][e]]
        uitems = 4 * c.cfg.urgent_split_k
    assert fired >= 10 and st["yields"] > 0 and st["device_status"] == 0
    assert np.array_equal(C.view(np.uint32), Cref.view(np.uint32)), "resume not bitwise"
    for Cu in outs:
        _check(Cu, refu, U_K)
    v = oracle.exactly_once(ex, ue[:fired], ev["claimer"][:fired], ev["set_ns"][:fired], uitems, fired)
    assert v["pass"], v


def test_clc_yields_sms_to_a_higher_priority_kernel(libapk):
    """With the queue scheduler the urgent kernel on the high-priority stream
    waits for the whole drain; under CLC the hardware declines requests while
    it waits, CTAs exit at tile boundaries and it starts within a few tiles."""
    A, B = oracle.gen_uniform(4096, 4096, 4096, 21)
    Au, Bu, _ = _urgent_ref()
    med = {}
    for sched in ("queue", "clc"):
        with _ctx(poll="off", urgent_split_k=1, scheduler=sched) as c:
            c.set_background(A, B)
            c.set_urgent(Au, Bu)
            e2e, tf = c.run_reserved(8192, 0, 8, seed=3)
            med[sched] = float(np.median(e2e))
            assert tf > 10
    assert med["clc"] * 5 < med["queue"], med
