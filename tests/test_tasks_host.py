"""configs[4] host logic without a GPU: the seeded task generator, the static
LPT shard, and the shard union over two gloo ranks (the N>1 path's host
side; the data path has no collective)."""
import os
import socket

import numpy as np
import pytest


def test_generator_is_deterministic_and_in_bounds(libapk):
    from apk_b200.runtime import POOL, gen_tasks
    t1, n1 = gen_tasks(5000, 21)
    t2, n2 = gen_tasks(5000, 21)
    t3, _ = gen_tasks(5000, 22)
    assert n1 == n2 and np.array_equal(t1, t2) and not np.array_equal(t1, t3)
    m, n, k = t1["m"], t1["n"], t1["k"]
    assert np.all((m % 128 == 0) & (m >= 128) & (m <= 2048))
    assert np.all((n % 128 == 0) & (n >= 128) & (n <= 2048))
    assert np.all((k % 64 == 0) & (k >= 256) & (k <= 4096))
    tiles_m = (m + 255) // 256
    assert np.all(t1["a_row0"] + tiles_m * 256 <= POOL["a_rows"])
    assert np.all(t1["a_k0"] + k <= POOL["a_cols"]) and np.all(t1["a_k0"] % 64 == 0)
    assert np.all(t1["b_k0"] + k <= POOL["b_rows"]) and np.all(t1["b_col0"] + n <= POOL["b_cols"])
    assert np.all(t1["c_row0"] + m <= POOL["c_rows"]) and np.all(t1["c_col0"] + n <= POOL["c_cols"])
    # chk_base is the running tile count
    tiles = tiles_m * (n // 128)
    assert np.array_equal(t1["chk_base"], np.concatenate([[0], np.cumsum(tiles)[:-1]]))
    assert n1 == int(tiles.sum())
    # sampled tasks own disjoint output windows above every other task's rows
    free = POOL["c_rows"] - 2048 * 2
    assert np.all(t1["c_row0"][8:] + m[8:] <= free)
    slots = {(int(r), int(c)) for r, c in zip(t1["c_row0"][:8], t1["c_col0"][:8])}
    assert len(slots) == 8


def test_log_uniform_shape_distribution(libapk):
    from apk_b200.runtime import gen_tasks
    t, _ = gen_tasks(200000, 5)
    # log-uniform on [128, 2048]: about half the mass below sqrt(128*2048) = 512
    frac = float(np.mean(t["m"] <= 512))
    assert 0.45 < frac < 0.6
    fl = 2.0 * t["m"].astype(np.float64) * t["n"] * t["k"]
    assert 1.1e9 < fl.mean() < 1.5e9  # ~1.3 GFLOP per task


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_lpt_shards_are_disjoint_complete_and_balanced(libapk, world):
    from apk_b200.runtime import gen_tasks, shard_tasks
    t, _ = gen_tasks(20000, 9)
    parts = [shard_tasks(t, world, r) for r in range(world)]
    u = np.concatenate(parts)
    assert len(u) == len(t) and len(np.unique(u)) == len(t)
    assert all(np.all(np.diff(p) > 0) for p in parts)
    fl = 2.0 * t["m"].astype(np.float64) * t["n"] * t["k"]
    loads = [fl[p].sum() for p in parts]
    assert max(loads) / min(loads) < 1.01


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    import torch.distributed as dist

    from apk_b200.runtime import gen_tasks, shard_tasks
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    t, n_chk = gen_tasks(4000, 33)  # every rank derives the same list from the seed
    mine = shard_tasks(t, world, rank)
    tiles = np.zeros(n_chk, np.int32)
    for i in mine:  # the global half-tiles this rank's oracle counters would show
        d = t[i]
        nt = ((int(d["m"]) + 255) // 256) * (int(d["n"]) // 128)
        tiles[int(d["chk_base"]):int(d["chk_base"]) + nt] += 1
    # the bench's host-side union of both drains' counters (uint8 sum over gloo)
    from apk_b200 import config4
    counts = config4.union_counts(world, tiles, tiles.copy())
    # a planted duplicate (rank 0 counts its first half-tile twice) must fail
    planted = tiles.copy()
    if rank == 0:
        planted[int(t[mine[0]]["chk_base"])] += 1
    dup = config4.union_counts(world, planted, tiles.copy())
    q.put((rank, int((counts == 1).all() and not (dup == 1).all()), len(mine)))
    dist.destroy_process_group()


def test_two_gloo_ranks_cover_every_tile_once(libapk):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res)
    assert sum(n for _, _, n in res) == 4000
