"""The runtime's error contract on a B200 (the apk_status codes of
include/apk.h): bad shapes, configurations the kernels do not serve,
launches that could not end, an empty task list and a launch longer than
the task list come back as status codes --
APK_EINVAL for arguments, APK_EUNSUPPORTED for variants that are not built,
APK_ESTATE for calls out of order -- and the context stays usable after
each (the reference's CUDA_CHECK -> exit(1) becomes a returned status)."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def _status(excinfo):
    return excinfo.value.status


def test_invalid_configurations_fail_at_create(libapk):
    import apk_b200
    from apk_b200 import _lib as L
    cases = [
        (dict(k_tile=48), L.APK_EINVAL),                        # K-tile 32/64/128 only
        (dict(poll="off", discipline="poison"), L.APK_EINVAL),  # poison needs polling
        (dict(scheduler="clc", discipline="poison", poll="stage"), L.APK_EUNSUPPORTED),
        (dict(dtype="bf16", scheduler="clc", ctas_per_sm=4), L.APK_EUNSUPPORTED),
        (dict(dtype="bf16", bf16_kernel="pair", k_tile=32), L.APK_EUNSUPPORTED),
        (dict(f32_kernel="ws", scheduler="clc"), L.APK_EUNSUPPORTED),   # ws drains the queue only
        (dict(f32_kernel="ws", ctas_per_sm=1), L.APK_EUNSUPPORTED),    # ws runs two workers per SM
        (dict(grid=10_000), L.APK_EINVAL),                      # beyond residency (src/yield.cu:815-822)
    ]
    for kw, want in cases:
        with pytest.raises(apk_b200.ApkError) as e:
            apk_b200.Context(**kw)
        assert _status(e) == want, (kw, e.value)
    # a valid context still comes up afterwards
    with apk_b200.Context() as c:
        assert c.info["grid"] > 0


def test_invalid_shapes_and_launches_are_rejected(libapk):
    import apk_b200
    from apk_b200 import _lib as L
    with apk_b200.Context(poll="stage") as c:
        A, B = oracle.gen_uniform(256, 256, 256, 1)
        with pytest.raises(apk_b200.ApkError) as e:       # no background set yet
            c.launch(4)
        assert _status(e) == L.APK_ESTATE
        bad = np.zeros((200, 256), np.float32)             # M not a multiple of 128
        with pytest.raises(apk_b200.ApkError) as e:
            c.set_background(bad, B)
        assert _status(e) == L.APK_EINVAL
        with pytest.raises(apk_b200.ApkError) as e:
            c.gemm(np.zeros((256, 200), np.float32), np.zeros((200, 256), np.float32))  # K not of the K-tile
        assert _status(e) == L.APK_EINVAL
        c.set_background(A, B)
        with pytest.raises(apk_b200.ApkError) as e:       # nothing to drain
            c.launch(0)
        assert _status(e) == L.APK_EINVAL
        with pytest.raises(apk_b200.ApkError) as e:       # polling launch without urgent operands
            c.launch(4)
        assert _status(e) == L.APK_ESTATE
        c.set_urgent(*oracle.gen_uniform(256, 256, 256, 2))
        c.launch(4)
        c.wait(30)
        C = c.read_output()
    mr, bad_n, nans = oracle.check(C, oracle.gemm_f64(A, B), oracle.fp32_tol(256))
    assert bad_n == 0 and nans == 0


def test_bf16_and_task_errors(libapk):
    import apk_b200
    from apk_b200 import _lib as L
    from apk_b200.runtime import POOL, gen_tasks
    with apk_b200.Context(dtype="bf16", poll="off") as c:
        A = apk_b200.fill_normal_bf16((128, 256), 1)       # bf16 M must be a multiple of 256
        B = apk_b200.fill_normal_bf16((256, 256), 2)
        with pytest.raises(apk_b200.ApkError) as e:
            c.set_background(A, B)
        assert _status(e) == L.APK_EINVAL
        Ap = apk_b200.fill_normal_bf16((POOL["a_rows"], POOL["a_cols"]), 3)
        Bp = apk_b200.fill_normal_bf16((POOL["b_rows"], POOL["b_cols"]), 4)
        c.set_task_pool(Ap, Bp, POOL["c_rows"], POOL["c_cols"])
        tasks, n_chk = gen_tasks(64, 5)
        with pytest.raises(apk_b200.ApkError) as e:       # an empty task list
            c.set_tasks(tasks[:0], n_chk)
        assert _status(e) == L.APK_EINVAL
        nw = c.set_tasks(tasks, n_chk)
        with pytest.raises(apk_b200.ApkError) as e:       # task mode needs a bounded launch
            c.launch(None)
        assert _status(e) == L.APK_EINVAL
        with pytest.raises(apk_b200.ApkError) as e:       # more than the work list holds
            c.launch(nw + 1)
        assert _status(e) == L.APK_EINVAL
        c.launch(nw)
        c.wait(30)
        assert c.run_stats()["tiles_done"] == n_chk
    with apk_b200.Context() as c:
        with pytest.raises(apk_b200.ApkError) as e:       # task pools are bf16 only
            c.set_task_pool(np.zeros((256, 256), np.float32), np.zeros((256, 256), np.float32), 256, 256)
        assert _status(e) == L.APK_EUNSUPPORTED
        with pytest.raises(apk_b200.ApkError) as e:       # no task pool: no task list either
            c.set_tasks(gen_tasks(4, 5)[0], 4)
        assert _status(e) == L.APK_ESTATE
