"""configs[4] on one GPU: the heterogeneous bf16 task queue.

Every global tile of every task runs exactly once; the per-tile checksums
sum(c^2) (fixed summation order) are bitwise identical whether the task list
runs whole, as two shards (each keeping the global checksum index), or with
urgent GEMMs preempting mid-pipeline; sampled tasks' outputs match float64
(quantise-then-reference, src/tcyield.cu:459-483) within 1e-2.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

N_TASKS = 3000
SEED = 21


def _pools():
    import apk_b200
    from apk_b200.runtime import POOL
    A = apk_b200.fill_normal_bf16((POOL["a_rows"], POOL["a_cols"]), 101)
    B = apk_b200.fill_normal_bf16((POOL["b_rows"], POOL["b_cols"]), 102)
    return A, B, POOL


def _ctx(**kw):
    import apk_b200
    kw.setdefault("urgent_split_k", 1)
    return apk_b200.Context(dtype="bf16", **kw)


def _run(ctx, A, B, pool, tasks, n_chk):
    ctx.set_task_pool(A, B, pool["c_rows"], pool["c_cols"])
    nw = ctx.set_tasks(tasks, n_chk)
    ctx.launch(nw)
    ctx.wait(120)
    return nw


@pytest.fixture(scope="module")
def whole_run(libapk):
    from apk_b200.runtime import gen_tasks
    A, B, pool = _pools()
    tasks, n_chk = gen_tasks(N_TASKS, SEED)
    with _ctx(poll="off", oracle=True) as c:
        _run(c, A, B, pool, tasks, n_chk)
        chk = c.read_checksums()
        ex, _ = c.read_oracle(n_chk)
        st = c.run_stats()
        samples = {}
        for t in range(8):
            d = tasks[t]
            samples[t] = c.read_pool_window(int(d["c_row0"]), int(d["c_col0"]), int(d["m"]), int(d["n"]))
    return dict(A=A, B=B, pool=pool, tasks=tasks, n_chk=n_chk, chk=chk, ex=ex, st=st, samples=samples)


def test_every_tile_exactly_once(whole_run):
    ex = whole_run["ex"]
    assert len(ex) == whole_run["n_chk"]
    assert int(np.count_nonzero(ex != 1)) == 0
    assert whole_run["st"]["tiles_done"] == whole_run["n_chk"]
    assert np.all(whole_run["chk"] > 0)


def test_sampled_tasks_match_float64(whole_run):
    A, B, tasks = whole_run["A"], whole_run["B"], whole_run["tasks"]
    for t, C in whole_run["samples"].items():
        d = tasks[t]
        m, n, k = int(d["m"]), int(d["n"]), int(d["k"])
        Aw = np.ascontiguousarray(A[d["a_row0"]:d["a_row0"] + m, d["a_k0"]:d["a_k0"] + k])
        Bw = np.ascontiguousarray(B[d["b_k0"]:d["b_k0"] + k, d["b_col0"]:d["b_col0"] + n])
        for r0 in (0, m - 8):
            ref = oracle.gemm_f64_bf16_rows(Aw, Bw, r0, 8)
            mr, bad, nans = oracle.check(C[r0:r0 + 8], ref, oracle.BF16_TOL)
            assert bad == 0 and nans == 0, f"task {t} rows {r0}: {bad} bad, max rel {mr:.3e}"
        # the checksum of tile (0,0) against float64 when the task fits one tile
        if m <= 256 and n <= 128:
            ref = oracle.gemm_f64_bf16_rows(Aw, Bw, 0, m)
            want = float((ref ** 2).sum())
            assert abs(whole_run["chk"][d["chk_base"]] - want) <= 1e-3 * want


def test_two_shards_reproduce_checksums_bitwise(whole_run):
    from apk_b200.runtime import shard_tasks
    tasks, n_chk = whole_run["tasks"], whole_run["n_chk"]
    merged = np.zeros(n_chk, np.float64)
    counts = np.zeros(n_chk, np.int64)
    with _ctx(poll="off", oracle=True) as c:
        for rank in range(2):
            idx = shard_tasks(tasks, 2, rank)
            _run(c, whole_run["A"], whole_run["B"], whole_run["pool"], tasks[idx], n_chk)
            chk = c.read_checksums()
            ex, _ = c.read_oracle(n_chk)
            merged[chk != 0] = chk[chk != 0]
            counts += ex
    assert np.all(counts == 1), "a tile ran twice or never across the shards"
    assert np.array_equal(merged.view(np.uint64), whole_run["chk"].view(np.uint64))


@pytest.mark.parametrize("kern", ["auto", "pair"])
def test_urgent_preemption_keeps_checksums_bitwise(whole_run, kern):
    """Device-set yields every 50 us while the task list drains, on the
    one-CTA kernel and on CTA pairs (6-slot task ring): every half-tile
    exactly once, checksums bitwise equal to the undisturbed run, every
    claimed event's urgent output complete and correct."""
    tasks, n_chk = whole_run["tasks"], whole_run["n_chk"]
    import apk_b200
    Au = apk_b200.fill_normal_bf16((256, 256), 31)
    Bu = apk_b200.fill_normal_bf16((256, 256), 32)
    refu = oracle.gemm_f64_bf16_rows(Au, Bu, 0, 256)
    nev = 40
    with _ctx(poll="stage", set_mode="device", oracle=True, max_events=64, bf16_kernel=kern) as c:
        c.set_urgent(Au, Bu)
        c.schedule_device_events((np.arange(nev, dtype=np.int64) + 1) * 50_000)
        _run(c, whole_run["A"], whole_run["B"], whole_run["pool"], tasks, n_chk)
        chk = c.read_checksums()
        ex, ue = c.read_oracle(n_chk)
        ev = c.read_events()
        st = c.run_stats()
        fired = int(np.count_nonzero(ev["set_ns"][:nev]))
        outs = [c.read_urgent_output(e) for e in range(fired) if ev["claimer"][e]]
        items = (256 // c.info["tile_m"]) * (-(-256 // c.info["tile_n"]))
    assert fired >= 10 and st["yields"] > 0
    assert np.all(ex == 1)
    assert np.array_equal(chk.view(np.uint64), whole_run["chk"].view(np.uint64)), "preemption changed a tile"
    for Cu in outs:
        assert oracle.check(Cu, refu, oracle.BF16_TOL)[1] == 0
    assert all(ue[e] == items for e in range(fired) if ev["claimer"][e])


def test_config4_poisson_host_stream_2e16_tasks(libapk):
    """configs[4] on 2^16 tasks with its own arrival process: urgent 256^3
    GEMMs injected by the host as a 2 kHz Poisson stream while the shard
    drains.  Every half-tile runs exactly once in both drains, no half-tile's
    checksum changes under preemption, every arrival is claimed and its
    urgent output is complete (src/yield.cu:576-667 verdict)."""
    from apk_b200 import config4
    res, ex0, ex1 = config4.run_rank(0, 1, 0, n_tasks=1 << 16, seed=SEED, rate_hz=2000.0)
    out = config4.summarize([res], config4.union_counts(1, ex0, ex1), 1 << 16)
    assert out["exactly_once"], res
    assert out["corrupted"] == 0
    assert out["arrivals"] >= 20 and out["urgent_claimed"] == out["arrivals"], res
    assert out["urgent_outputs_ok"] and out["checkpoints"] > 0


def test_clc_scheduler_task_queue_bitwise(whole_run):
    """The task list under cluster launch control (one CTA per work entry):
    every half-tile exactly once, checksums bitwise equal to the queue run."""
    tasks, n_chk = whole_run["tasks"], whole_run["n_chk"]
    with _ctx(poll="off", oracle=True, scheduler="clc") as c:
        _run(c, whole_run["A"], whole_run["B"], whole_run["pool"], tasks, n_chk)
        chk = c.read_checksums()
        ex, _ = c.read_oracle(n_chk)
        st = c.run_stats()
    assert st["device_status"] == 0
    assert np.all(ex == 1)
    assert np.array_equal(chk.view(np.uint64), whole_run["chk"].view(np.uint64))


def test_pair_and_single_kernels_checksums_bitwise(whole_run):
    """The task list on CTA pairs (256x256 jobs, 128-row tiles as N = 128
    pair MMAs, 128-wide edges computed by the pair and stored by the leader
    only) and on the one-CTA kernel: every half-tile exactly once on both,
    checksums bitwise equal (same MMA sequence per element, same summation
    order)."""
    tasks, n_chk = whole_run["tasks"], whole_run["n_chk"]
    out = {}
    for kern in ("pair", "single"):
        with _ctx(poll="off", oracle=True, bf16_kernel=kern) as c:
            _run(c, whole_run["A"], whole_run["B"], whole_run["pool"], tasks, n_chk)
            out[kern] = c.read_checksums()
            ex, _ = c.read_oracle(n_chk)
            st = c.run_stats()
        assert np.all(ex == 1), kern
        assert st["tiles_done"] == n_chk and st["device_status"] == 0, kern
    assert np.array_equal(out["pair"].view(np.uint64), out["single"].view(np.uint64))


@pytest.mark.parametrize("kern", ["pair", "single"])
def test_task_list_exit_is_prompt(libapk, kern):
    """A 2^16-task list drains in ~0.1 s on either kernel.  At exit a
    producer waits out only the loads of its last ring slots: waiting from a
    lagging consumed count reused a slot's barrier parity and held the pair
    kernel at exit for the whole bounded-wait limit (2 s, no device status)
    -- so the launch time must stay far below that limit."""
    from apk_b200.runtime import gen_tasks
    A, B, pool = _pools()
    tasks, n_chk = gen_tasks(1 << 16, SEED)
    import apk_b200
    with _ctx(poll="stage", bf16_kernel=kern) as c:
        c.set_urgent(apk_b200.fill_normal_bf16((256, 256), 31), apk_b200.fill_normal_bf16((256, 256), 32))
        _run(c, A, B, pool, tasks, n_chk)
        st = c.run_stats()
    assert st["device_status"] == 0 and st["tiles_done"] == n_chk
    assert st["launch_ms"] < 1000.0, st["launch_ms"]
