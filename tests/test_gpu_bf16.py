"""GPU parity tests of the bf16 tcgen05 persistent GEMM, through the C ABI.

Reference: float64 over the bf16-rounded inputs (quantise-then-reference,
src/tcyield.cu:459-483), tolerance rel = |got-ref|/max(1,|ref|) <= 1e-2;
resumed tiles bitwise against an uninterrupted run of the same kernel
(BASELINE configs[2]); scheduler invariants as src/yield.cu:630-663.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
TOL = oracle.BF16_TOL


def _ctx(**kw):
    import apk_b200
    kw.setdefault("urgent_split_k", 1)
    return apk_b200.Context(dtype="bf16", **kw)


def _normal(shape, seed):
    import apk_b200
    return apk_b200.fill_normal_bf16(shape, seed)


def _check_rows(C, A, B, rows):
    for r0, n in rows:
        ref = oracle.gemm_f64_bf16_rows(A, B, r0, n)
        mr, bad, nans = oracle.check(C[r0:r0 + n], ref, TOL)
        assert nans == 0 and bad == 0, f"rows {r0}+{n}: {bad} bad, {nans} NaN, max rel {mr:.3e}"


@pytest.mark.parametrize("shape", [(256, 512, 64), (512, 768, 256), (1024, 2048, 512)])
def test_pair_kernel_bitwise_equal_to_single(libapk, shape):
    """The CTA-pair kernel (256x512 tiles over two SMs, cta_group::2 MMAs)
    and the one-CTA kernel issue the same MMA sequence per accumulator: C
    bitwise equal, and within tolerance of float64 over the rounded inputs.
    N = 768 ends each tile row with a 256-wide pair tile (one accumulator)."""
    M, N, K = shape
    A, B = _normal((M, K), 21), _normal((K, N), 22)
    out = {}
    for k in ("pair", "single"):
        with _ctx(poll="stage", oracle=True, bf16_kernel=k) as c:
            out[k] = c.gemm(A, B)
            assert c.info["tile_n"] == (512 if k == "pair" else 256)
    assert np.array_equal(out["pair"].view(np.uint32), out["single"].view(np.uint32))
    _check_rows(out["pair"], A, B, [(0, min(M, 32)), (M - 32, 32)])


@pytest.mark.parametrize("shape", [(256, 128, 64), (256, 256, 320), (512, 384, 1024), (1024, 2048, 512)])
def test_small_shapes_full_check(libapk, shape):
    M, N, K = shape
    A, B = _normal((M, K), 1), _normal((K, N), 2)
    with _ctx(poll="off", oracle=True) as c:
        C = c.gemm(A, B)
    _check_rows(C, A, B, [(0, M)])


def test_uniform_inputs_quantised(libapk):
    """bf16 mode of the scaling-surface cells: uniform[-1,1] from the
    reference generator, rounded to bf16."""
    A16, B16 = oracle.gen_uniform_bf16(512, 512, 512, 21)
    with _ctx(poll="stage", oracle=True) as c:
        C = c.gemm(A16, B16)
    _check_rows(C, A16, B16, [(0, 512)])


def test_config2_shape_sampled_rows(libapk):
    """8192^3, N(0,1) rounded to bf16; sampled row bands against
    float64 (each band spans every K)."""
    M = N = K = 8192
    A, B = _normal((M, K), 21), _normal((K, N), 22)
    with _ctx(poll="stage", oracle=True) as c:
        C = c.gemm(A, B)
    _check_rows(C, A, B, [(0, 8), (255, 2), (4096 + 128, 8), (M - 8, 8)])


def _yield_run(poll, nev=30, gap_ns=20_000, discipline="drain", n=4096, drains=0):
    M = N = K = n
    A, B = _normal((M, K), 21), _normal((K, N), 22)
    Au, Bu = _normal((256, 256), 31), _normal((256, 256), 32)
    with _ctx(poll="off") as c:
        Cref = c.gemm(A, B)
    with _ctx(poll=poll, set_mode="device", oracle=True, discipline=discipline, max_events=max(64, nev + 8)) as c:
        # task t computes tile t mod tiles: 1024 tasks, or whole drains of C
        ntasks = drains * (M // c.info["tile_m"]) * (N // c.info["tile_n"]) if drains else 1024
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_device_events((np.arange(nev, dtype=np.int64) + 1) * gap_ns)
        c.launch(ntasks)
        c.wait(60)
        C = c.read_output()
        ev = c.read_events()
        st = c.run_stats()
        ex, ue = c.read_oracle(ntasks)
        fired = int(np.count_nonzero(ev["set_ns"][:nev]))
        outs = [c.read_urgent_output(e) for e in range(fired) if ev["claimer"][e]]
        info = c.info
        uitems = (256 // info["tile_m"]) * (-(-256 // info["tile_n"])) * c.cfg.urgent_split_k
    refu = oracle.gemm_f64_bf16_rows(Au, Bu, 0, 256)
    return dict(C=C, Cref=Cref, ev=ev, st=st, ex=ex, ue=ue, fired=fired, outs=outs, refu=refu, uitems=uitems,
                tile_n=info["tile_n"])


def test_stage_checkpoint_resume_is_bitwise(libapk):
    """configs[2] property: yields at random pipeline stages, including
    buffer-conflicting ones; accumulators spilled from TMEM and restored;
    output bitwise equal to the uninterrupted run."""
    r = _yield_run("stage")
    ev = r["ev"]
    assert r["fired"] >= 10
    assert r["st"]["yields"] > 0
    sites = [ev["claim_site"][e] for e in range(r["fired"]) if ev["claimer"][e]]
    assert any(s > 0 for s in sites), "no mid-pipeline claim"
    assert any(ev["inflight"][e] > 0 for e in range(r["fired"])), "no buffer-conflicting yield"
    assert np.array_equal(r["C"].view(np.uint32), r["Cref"].view(np.uint32)), "resume not bitwise"
    # every checkpoint spills one wide 256x256 fp32 accumulator per CTA
    # (two CTAs for a 256x512 pair tile) and the drain restores each of them
    st = r["st"]
    ctas = r["tile_n"] // 256
    assert st["ckpt_spill_bytes"] == st["yields"] * 256 * 256 * 4 * ctas
    assert st["ckpt_restore_bytes"] == st["ckpt_spill_bytes"]
    assert st["ckpt_spill_ns"] > 0 and st["ckpt_restore_ns"] > 0
    for Cu in r["outs"]:
        mr, bad, nans = oracle.check(Cu, r["refu"], TOL)
        assert bad == 0 and nans == 0
    f = r["fired"]
    v = oracle.exactly_once(r["ex"], r["ue"][:f], ev["claimer"][:f], ev["set_ns"][:f], r["uitems"], f)
    assert v["pass"], v


def test_config2_full_shape_stage_yields_bitwise(libapk):
    """configs[2] at its own size, 8192^3: yields at random pipeline stages
    (40 device-set events 15 us apart, inside two ~0.7 ms drains), including
    buffer-conflicting ones; the resumed output is bitwise equal to the
    uninterrupted run, every tile and urgent item ran exactly once and every
    urgent output matches float64."""
    r = _yield_run("stage", nev=40, gap_ns=15_000, n=8192, drains=2)
    ev = r["ev"]
    assert r["fired"] >= 20 and r["st"]["yields"] > 0
    claimed = [e for e in range(r["fired"]) if ev["claimer"][e]]
    assert any(ev["claim_site"][e] > 0 for e in claimed), "no mid-pipeline claim"
    assert any(ev["inflight"][e] > 0 for e in claimed), "no buffer-conflicting yield"
    assert np.array_equal(r["C"].view(np.uint32), r["Cref"].view(np.uint32)), "resume not bitwise"
    for Cu in r["outs"]:
        mr, bad, nans = oracle.check(Cu, r["refu"], TOL)
        assert bad == 0 and nans == 0, f"urgent: {bad} bad, max rel {mr:.3e}"
    f = r["fired"]
    v = oracle.exactly_once(r["ex"], r["ue"][:f], ev["claimer"][:f], ev["set_ns"][:f], r["uitems"], f)
    assert v["pass"], v


def test_boundary_yield_is_bitwise(libapk):
    r = _yield_run("boundary")
    assert np.array_equal(r["C"].view(np.uint32), r["Cref"].view(np.uint32))
    assert all(r["ev"]["claim_site"][e] == -1 for e in range(r["fired"]) if r["ev"]["claimer"][e])
    for Cu in r["outs"]:
        assert oracle.check(Cu, r["refu"], TOL)[1] == 0


def test_poison_discipline_is_detected(libapk):
    r = _yield_run("stage", nev=8, discipline="poison")
    assert r["outs"]
    for Cu in r["outs"]:
        assert oracle.check(Cu, r["refu"], TOL)[1] > 0
    # the background output is still exact: poison only touches urgent stages
    assert np.array_equal(r["C"].view(np.uint32), r["Cref"].view(np.uint32))


def test_host_memcpy_injection(libapk):
    M = N = K = 2048
    A, B = _normal((M, K), 3), _normal((K, N), 4)
    Au, Bu = _normal((256, 256), 5), _normal((256, 256), 6)
    refu = oracle.gemm_f64_bf16_rows(Au, Bu, 0, 256)
    with _ctx(poll="stage", set_mode="host_memcpy", max_events=32) as c:
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.launch(None)
        for _ in range(10):
            e, _t = c.inject()
            assert c.wait_ack(e, 1, 500_000_000) is not None
        c.stop()
        c.wait(30)
        ev = c.read_events()
        outs = [c.read_urgent_output(e) for e in range(10)]
    assert all(ev["claimer"][:10] != 0)
    for Cu in outs:
        assert oracle.check(Cu, refu, TOL)[1] == 0


def test_split_k_urgent_items(libapk):
    """Urgent GEMM split into K slices accumulated with atomics."""
    M = N = K = 2048
    A, B = _normal((M, K), 7), _normal((K, N), 8)
    Au, Bu = _normal((256, 256), 9), _normal((256, 256), 10)
    refu = oracle.gemm_f64_bf16_rows(Au, Bu, 0, 256)
    with _ctx(poll="stage", set_mode="device", urgent_split_k=4, oracle=True) as c:
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_device_events(np.array([10_000, 30_000, 50_000], np.int64))
        c.launch(512)
        c.wait(60)
        ev = c.read_events()
        outs = [c.read_urgent_output(e) for e in range(3) if ev["claimer"][e]]
        _, ue = c.read_oracle(512)
        items = (256 // c.info["tile_m"]) * (-(-256 // c.info["tile_n"])) * 4
    assert outs
    for Cu in outs:
        assert oracle.check(Cu, refu, TOL)[1] == 0
    assert all(ue[e] == items for e in range(3) if ev["claimer"][e])


def test_narrow_edge_tiles_yield_bitwise(libapk):
    """Widths that are odd multiples of 128 end each tile row with a 256x128
    tile (one TMEM accumulator) after 256x256 ones (two): stage yields
    checkpoint and resume both kinds bitwise; a 384-wide urgent GEMM runs one
    item of each kind."""
    M, N, K = 2048, 1152, 8192
    A, B = _normal((M, K), 41), _normal((K, N), 42)
    Au, Bu = _normal((256, 256), 43), _normal((256, 384), 44)
    with _ctx(poll="off") as c:
        Cref = c.gemm(A, B)
    _check_rows(Cref, A, B, [(0, 4), (M - 4, 4)])
    nev = 16
    with _ctx(poll="stage", set_mode="device", oracle=True) as c:
        ntasks = 3 * c.info["grid"]
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_device_events((np.arange(nev, dtype=np.int64) + 1) * 8_000)
        c.launch(ntasks)
        c.wait(60)
        C = c.read_output()
        ev = c.read_events()
        st = c.run_stats()
        ex, ue = c.read_oracle(ntasks)
        fired = int(np.count_nonzero(ev["set_ns"][:nev]))
        outs = [c.read_urgent_output(e) for e in range(fired) if ev["claimer"][e]]
    assert fired >= 8 and st["yields"] > 0
    assert any(ev["claim_site"][e] > 0 for e in range(fired) if ev["claimer"][e]), "no mid-pipeline claim"
    assert np.array_equal(C.view(np.uint32), Cref.view(np.uint32)), "resume not bitwise"
    refu = oracle.gemm_f64_bf16_rows(Au, Bu, 0, 256)
    assert outs
    for Cu in outs:
        mr, bad, nans = oracle.check(Cu, refu, TOL)
        assert bad == 0 and nans == 0, f"urgent: {bad} bad, max rel {mr:.3e}"
    v = oracle.exactly_once(ex, ue[:fired], ev["claimer"][:fired], ev["set_ns"][:fired], 2, fired)
    assert v["pass"], v


@pytest.mark.parametrize("shape", [(256, 128, 32), (512, 384, 1056), (1024, 2048, 512)])
def test_k_tile_32_full_check(libapk, shape):
    """K-tile 32: [128][32] A boxes in the 64-byte-swizzled K-major layout,
    a 7-slot ring."""
    M, N, K = shape
    A, B = _normal((M, K), 11), _normal((K, N), 12)
    with _ctx(poll="off", oracle=True, k_tile=32) as c:
        assert c.info["k_tile"] == 32 and c.info["stages"] == 7
        C = c.gemm(A, B)
    _check_rows(C, A, B, [(0, M)])


def test_k_tile_32_stage_yield_bitwise(libapk):
    M = N = K = 4096
    A, B = _normal((M, K), 13), _normal((K, N), 14)
    Au, Bu = _normal((256, 256), 15), _normal((256, 256), 16)
    with _ctx(poll="off", k_tile=32) as c:
        Cref = c.gemm(A, B)
    _check_rows(Cref, A, B, [(0, 4), (M - 4, 4)])
    nev = 20
    with _ctx(poll="stage", set_mode="device", oracle=True, k_tile=32) as c:
        ntasks = 1024
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_device_events((np.arange(nev, dtype=np.int64) + 1) * 15_000)
        c.launch(ntasks)
        c.wait(60)
        C = c.read_output()
        ev = c.read_events()
        st = c.run_stats()
        ex, ue = c.read_oracle(ntasks)
        fired = int(np.count_nonzero(ev["set_ns"][:nev]))
        outs = [c.read_urgent_output(e) for e in range(fired) if ev["claimer"][e]]
    assert fired >= 10 and st["yields"] > 0
    assert np.array_equal(C.view(np.uint32), Cref.view(np.uint32)), "resume not bitwise"
    refu = oracle.gemm_f64_bf16_rows(Au, Bu, 0, 256)
    for Cu in outs:
        mr, bad, nans = oracle.check(Cu, refu, TOL)
        assert bad == 0 and nans == 0
    v = oracle.exactly_once(ex, ue[:fired], ev["claimer"][:fired], ev["set_ns"][:fired], 1, fired)
    assert v["pass"], v


@pytest.mark.parametrize("kernel", ["narrow", "narrow_spill"])
def test_narrow_jobs_park_or_spill_bitwise(libapk, kernel):
    """256x128 background and urgent jobs, each in one of the two TMEM
    buffers.  NARROW parks a yielding background job's accumulator in its
    buffer while the urgent items run in the other (no spill or restore
    bytes); NARROW_SPILL checkpoints it to the slab.  Either way the resumed
    MMAs continue the same sequence: C bitwise equal to the one-CTA
    kernel's uninterrupted drain, every urgent output within 1e-2 of
    float64, exactly once."""
    M = N = K = 4096
    A, B = _normal((M, K), 21), _normal((K, N), 22)
    Au, Bu = _normal((256, 256), 31), _normal((256, 256), 32)
    refu = oracle.gemm_f64_bf16_rows(Au, Bu, 0, 256)
    with _ctx(poll="off", bf16_kernel="single") as c:
        C0 = c.gemm(A, B)
    nev = 30
    with _ctx(poll="stage", set_mode="device", oracle=True, bf16_kernel=kernel, max_events=64) as c:
        info = c.info
        assert (info["tile_m"], info["tile_n"]) == (256, 128)
        ntasks = 8 * (M // 256) * (N // 128)
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_device_events((np.arange(nev, dtype=np.int64) + 1) * 20_000)
        c.launch(ntasks)
        c.wait(60)
        C = c.read_output()
        ev = c.read_events()
        st = c.run_stats()
        ex, ue = c.read_oracle(ntasks)
        fired = int(np.count_nonzero(ev["set_ns"][:nev]))
        outs = [c.read_urgent_output(e) for e in range(fired) if ev["claimer"][e]]
    assert fired >= 10 and st["yields"] > 0
    if kernel == "narrow":
        assert st["parks"] == st["yields"] and st["ckpt_spill_bytes"] == 0 and st["ckpt_restore_bytes"] == 0
    else:
        assert st["parks"] == 0 and st["ckpt_spill_bytes"] == st["yields"] * 256 * 128 * 4
    assert np.array_equal(C.view(np.uint32), C0.view(np.uint32)), "resume not bitwise"
    for Cu in outs:
        mr, bad, nans = oracle.check(Cu, refu, TOL)
        assert bad == 0 and nans == 0, f"urgent: {bad} bad, max rel {mr:.3e}"
    v = oracle.exactly_once(ex, ue[:fired], ev["claimer"][:fired], ev["set_ns"][:fired], 2, fired)
    assert v["pass"], v


@pytest.mark.parametrize("kern", ["single", "pair"])
def test_clc_scheduler_drain_exactly_once_bitwise(libapk, kern):
    """bf16 under cluster launch control: one CTA (or one CTA pair) per
    task, running CTAs take the pending ones -- on pairs the leader cancels
    a pending cluster and relays its tile to the peer through the stage
    tags; every task exactly once and C bitwise equal to the
    queue-scheduled one-CTA kernel's."""
    M, N, K = 2048, 2048, 1024
    A, B = _normal((M, K), 51), _normal((K, N), 52)
    with _ctx(poll="off", bf16_kernel="single") as c:
        C0 = c.gemm(A, B)
    with _ctx(poll="off", oracle=True, scheduler="clc", bf16_kernel=kern) as c:
        info = c.info
        assert info["tile_n"] == (512 if kern == "pair" else 256)
        tiles = (M // info["tile_m"]) * (N // info["tile_n"])
        ntasks = 3 * tiles
        C = c.gemm(A, B)
        st = c.run_stats()
        c.set_background(A, B)
        c.launch(ntasks)
        c.wait(30)
        ex, _ = c.read_oracle(ntasks)
        st2 = c.run_stats()
    assert np.array_equal(C.view(np.uint32), C0.view(np.uint32))
    assert st["tiles_done"] == tiles and st["device_status"] == 0
    assert st2["tiles_done"] == ntasks and st2["device_status"] == 0
    assert np.all(ex == 1)


@pytest.mark.parametrize("kern", ["single", "pair"])
def test_clc_stage_yields_bitwise(libapk, kern):
    """bf16 CLC with per-stage device-set yields (on pairs: only the leader
    polls, the peer follows its tags): checkpoints resume bitwise; every
    task and urgent item exactly once."""
    M = N = K = 4096
    A, B = _normal((M, K), 21), _normal((K, N), 22)
    Au, Bu = _normal((256, 256), 31), _normal((256, 256), 32)
    refu = oracle.gemm_f64_bf16_rows(Au, Bu, 0, 256)
    with _ctx(poll="off", bf16_kernel="single") as c:
        C0 = c.gemm(A, B)
    nev = 30
    with _ctx(poll="stage", set_mode="device", oracle=True, scheduler="clc", max_events=64, bf16_kernel=kern) as c:
        info = c.info
        assert info["tile_n"] == (512 if kern == "pair" else 256)
        ntasks = 8 * (M // info["tile_m"]) * (N // info["tile_n"])
        c.set_background(A, B)
        c.set_urgent(Au, Bu)
        c.schedule_device_events((np.arange(nev, dtype=np.int64) + 1) * 20_000)
        c.launch(ntasks)
        c.wait(60)
        C = c.read_output()
        ev = c.read_events()
        st = c.run_stats()
        ex, ue = c.read_oracle(ntasks)
        fired = int(np.count_nonzero(ev["set_ns"][:nev]))
        outs = [c.read_urgent_output(e) for e in range(fired) if ev["claimer"][e]]
    assert fired >= 10 and st["yields"] > 0 and st["device_status"] == 0
    assert any(ev["claim_site"][e] > 0 for e in range(fired) if ev["claimer"][e]), "no mid-pipeline claim"
    assert np.array_equal(C.view(np.uint32), C0.view(np.uint32)), "resume not bitwise"
    for Cu in outs:
        mr, bad, nans = oracle.check(Cu, refu, TOL)
        assert bad == 0 and nans == 0
    v = oracle.exactly_once(ex, ue[:fired], ev["claimer"][:fired], ev["set_ns"][:fired], 1, fired)
    assert v["pass"], v
