"""Python mirror of the runtime's C ABI (include/apk.h).

This is the host-side convenience layer over libapk.so; every call goes
straight to the native runtime.  The modes mirror the reference binaries'
``--mode`` switches (verify / latency / overhead / oracle / baseline), see
``src/yield.cu:327-960`` and ``src/urgent_baseline.cu:144-380`` in
AyaanFaisal21/APK.
"""
from __future__ import annotations

import ctypes
import weakref

import numpy as np

from . import _lib as L

_POLL = {"off": L.APK_POLL_OFF, "boundary": L.APK_POLL_BOUNDARY, "stage": L.APK_POLL_STAGE}
_DISC = {"drain": L.APK_DISC_DRAIN, "poison": L.APK_DISC_POISON}
_SET = {"device": L.APK_SET_DEVICE, "host_mapped": L.APK_SET_HOST_MAPPED,
        "host_memcpy": L.APK_SET_HOST_MEMCPY}
_DTYPE = {"f32": L.APK_F32, "bf16": L.APK_BF16}
_SCHED = {"queue": L.APK_SCHED_QUEUE, "clc": L.APK_SCHED_CLC}
_F32K = {"auto": 0, "ws": 1, "sync": 2}
_BF16K = {"auto": 0, "pair": 1, "single": 2, "narrow": 3, "narrow_spill": 4}


class ApkError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{L.STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def _ptr(a: np.ndarray):
    if not a.flags["C_CONTIGUOUS"]:
        raise ValueError("array must be C-contiguous")
    return ctypes.c_void_p(a.ctypes.data)


def fill_uniform(M: int, N: int, K: int, seed: int = 21):
    """A (MxK) then B (KxN) from srand(seed)/rand(), src/persistent.cu:132-135."""
    A = np.empty((M, K), np.float32)
    B = np.empty((K, N), np.float32)
    L.load().apk_fill_uniform(seed, _ptr(A), A.size, _ptr(B), B.size)
    return A, B


def fill_normal_bf16(shape, seed: int) -> np.ndarray:
    out = np.empty(shape, np.uint16)
    L.load().apk_fill_normal_bf16(seed, _ptr(out), out.size)
    return out


def round_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    L.load().apk_round_bf16(_ptr(x), _ptr(out), x.size)
    return out


# numpy mirror of apk_task (include/apk.h): 10 int32 + int64 = 48 bytes
TASK_DTYPE = np.dtype([("m", "<i4"), ("n", "<i4"), ("k", "<i4"), ("a_row0", "<i4"), ("a_k0", "<i4"),
                       ("b_k0", "<i4"), ("b_col0", "<i4"), ("c_row0", "<i4"), ("c_col0", "<i4"),
                       ("flags", "<i4"), ("chk_base", "<i8")], align=True)
assert TASK_DTYPE.itemsize == 48

# configs[4] pools: windows of these operand pools (A, B bf16; C fp32)
POOL = dict(a_rows=4096 + 256, a_cols=4096, b_rows=4096, b_cols=4096, c_rows=4096 + 4096, c_cols=8192)


def gen_tasks(n: int, seed: int = 21, mn_lo: int = 128, mn_hi: int = 2048, k_lo: int = 256, k_hi: int = 4096,
              n_samples: int = 8, pool: dict | None = None):
    """configs[4] task list (log-uniform m, n in [mn_lo, mn_hi] to x128, k in
    [k_lo, k_hi] to x64) as windows of the pools; returns (tasks, n_chk)."""
    pool = pool or POOL
    out = np.zeros(n, TASK_DTYPE)
    n_chk = L.load().apk_gen_tasks(seed, n, mn_lo, mn_hi, k_lo, k_hi, pool["a_rows"], pool["a_cols"],
                                   pool["b_rows"], pool["b_cols"], pool["c_rows"], pool["c_cols"], n_samples,
                                   _ptr(out))
    return out, int(n_chk)


def shard_tasks(tasks: np.ndarray, world: int, rank: int) -> np.ndarray:
    """Static LPT shard: this rank's task indices (ascending)."""
    idx = np.zeros(len(tasks), np.int32)
    m = L.load().apk_shard_tasks(_ptr(tasks), len(tasks), world, rank, _ptr(idx))
    return idx[:m].copy()


def pinned_empty(shape, dtype) -> np.ndarray:
    """Page-locked host array (freed when the array is garbage collected)."""
    dtype = np.dtype(dtype)
    n = int(np.prod(shape)) * dtype.itemsize
    lib = L.load()
    p = lib.apk_host_alloc(max(n, 1))
    if not p:
        raise MemoryError(f"apk_host_alloc({n}) failed")
    buf = (ctypes.c_byte * n).from_address(p)
    arr = np.frombuffer(buf, dtype=dtype).reshape(shape)
    weakref.finalize(buf, lib.apk_host_free, p)
    return arr


class Context:
    """One preemptible persistent-GEMM runtime on one device."""

    def __init__(self, device: int = 0, dtype: str = "f32", ctas_per_sm: int = 0, grid: int = 0,
                 k_tile: int = 0, poll: str = "stage", discipline: str = "drain",
                 set_mode: str = "host_memcpy", max_events: int = 4096, oracle: bool = False,
                 urgent_split_k: int = 8, wait_limit_ns: int = 2_000_000_000, scheduler: str = "queue",
                 f32_kernel: str = "auto", bf16_kernel: str = "auto"):
        self._lib = L.load()
        cfg = L.Config()
        self._lib.apk_config_default(ctypes.byref(cfg))
        cfg.device, cfg.dtype, cfg.ctas_per_sm, cfg.grid = device, _DTYPE[dtype], ctas_per_sm, grid
        cfg.k_tile, cfg.poll, cfg.discipline = k_tile, _POLL[poll], _DISC[discipline]
        cfg.set_mode, cfg.max_events, cfg.oracle = _SET[set_mode], max_events, int(oracle)
        cfg.urgent_split_k, cfg.wait_limit_ns = urgent_split_k, int(wait_limit_ns)
        cfg.scheduler = _SCHED[scheduler]
        cfg.f32_kernel = _F32K[f32_kernel]
        cfg.bf16_kernel = _BF16K[bf16_kernel]
        self.cfg = cfg
        self.dtype = dtype
        h = ctypes.c_void_p()
        st = self._lib.apk_create(ctypes.byref(cfg), ctypes.byref(h))
        self._h = h
        if st != L.APK_OK:
            msg = self._lib.apk_last_error(h).decode() if h.value else "apk_create failed"
            self._lib.apk_destroy(h)
            self._h = ctypes.c_void_p()
            raise ApkError(st, msg)
        self.M = self.N = self.K = 0
        self.Mu = self.Nu = self.Ku = 0
        self._keep = []

    # ------------------------------------------------------------------ util
    def _check(self, st: int):
        if st != L.APK_OK:
            raise ApkError(st, self._lib.apk_last_error(self._h).decode())

    def close(self):
        if self._h and self._h.value:
            self._lib.apk_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def info(self) -> dict:
        i = L.DeviceInfo()
        self._check(self._lib.apk_get_info(self._h, ctypes.byref(i)))
        d = {f: getattr(i, f) for f, _ in L.DeviceInfo._fields_}
        d["name"] = i.name.decode()
        return d

    # ------------------------------------------------------------- operands
    def set_background(self, A: np.ndarray, B: np.ndarray):
        M, K = A.shape
        K2, N = B.shape
        assert K == K2
        self._check(self._lib.apk_set_background(self._h, _ptr(A), _ptr(B), None, M, N, K, L.APK_MEM_HOST))
        self.M, self.N, self.K = M, N, K

    def set_background_device(self, A_ptr: int, B_ptr: int, C_ptr: int, M: int, N: int, K: int):
        self._check(self._lib.apk_set_background(self._h, ctypes.c_void_p(A_ptr), ctypes.c_void_p(B_ptr),
                                                 ctypes.c_void_p(C_ptr), M, N, K, L.APK_MEM_DEVICE))
        self.M, self.N, self.K = M, N, K

    def set_urgent(self, A: np.ndarray, B: np.ndarray):
        M, K = A.shape
        K2, N = B.shape
        assert K == K2
        self._check(self._lib.apk_set_urgent(self._h, _ptr(A), _ptr(B), M, N, K, L.APK_MEM_HOST))
        self.Mu, self.Nu, self.Ku = M, N, K

    # ------------------------------------------------------ task queue (cfg 4)
    def set_task_pool(self, A_pool: np.ndarray, B_pool: np.ndarray, c_rows: int, c_cols: int):
        self._check(self._lib.apk_set_task_pool(self._h, _ptr(A_pool), A_pool.shape[0], A_pool.shape[1],
                                                _ptr(B_pool), B_pool.shape[0], B_pool.shape[1], c_rows, c_cols,
                                                L.APK_MEM_HOST))
        self.c_pool = (c_rows, c_cols)

    def set_tasks(self, tasks: np.ndarray, n_chk: int) -> int:
        tasks = np.ascontiguousarray(tasks, TASK_DTYPE)
        nw = ctypes.c_ulonglong()
        self._check(self._lib.apk_set_tasks(self._h, _ptr(tasks), len(tasks), n_chk, ctypes.byref(nw)))
        self.n_chk = n_chk
        return nw.value

    def read_checksums(self) -> np.ndarray:
        out = np.zeros(self.n_chk, np.float64)
        self._check(self._lib.apk_read_checksums(self._h, _ptr(out), self.n_chk))
        return out

    def read_pool_window(self, row0: int, col0: int, rows: int, cols: int) -> np.ndarray:
        out = np.empty((rows, cols), np.float32)
        self._check(self._lib.apk_read_pool_window(self._h, row0, col0, rows, cols, _ptr(out)))
        return out

    # ---------------------------------------------------------------- launch
    def schedule_device_events(self, offsets_ns):
        arr = np.ascontiguousarray(offsets_ns, np.int64)
        self._check(self._lib.apk_schedule_device_events(self._h, _ptr(arr), arr.size))

    def schedule_count_events(self, counts):
        arr = np.ascontiguousarray(counts, np.uint64)
        self._check(self._lib.apk_schedule_count_events(self._h, _ptr(arr), arr.size))

    def selftest_wait_timeout(self, limit_ns: int = 50_000_000) -> int:
        st = ctypes.c_int()
        self._check(self._lib.apk_selftest_wait_timeout(self._h, int(limit_ns), ctypes.byref(st)))
        return st.value

    def launch(self, num_tasks: int | None = None):
        n = L.APK_TASKS_UNBOUNDED if num_tasks is None else int(num_tasks)
        self._check(self._lib.apk_launch(self._h, n))

    def inject(self):
        ev = ctypes.c_int()
        t = ctypes.c_longlong()
        self._check(self._lib.apk_inject_urgent(self._h, ctypes.byref(ev), ctypes.byref(t)))
        return ev.value, t.value

    def wait_ack(self, event: int, which: int = 0, timeout_ns: int = 100_000_000):
        t = ctypes.c_longlong()
        st = self._lib.apk_wait_ack(self._h, event, which, int(timeout_ns), ctypes.byref(t))
        if st == L.APK_ETIMEDOUT:
            return None
        self._check(st)
        return t.value

    def stop(self):
        self._check(self._lib.apk_stop(self._h))

    def wait(self, timeout_s: float = 60.0):
        self._check(self._lib.apk_wait(self._h, int(timeout_s * 1e9)))

    # -------------------------------------------------------------- readback
    def read_output(self) -> np.ndarray:
        C = np.empty((self.M, self.N), np.float32)
        self._check(self._lib.apk_read_output(self._h, _ptr(C)))
        return C

    def read_urgent_output(self, event: int) -> np.ndarray:
        C = np.empty((self.Mu, self.Nu), np.float32)
        self._check(self._lib.apk_read_urgent_output(self._h, event, _ptr(C)))
        return C

    def read_events(self) -> dict:
        E = self.cfg.max_events
        G = self.info["grid"]
        out = {k: np.zeros(E, np.int64) for k in ("set_ns", "host_set_ns", "host_ack_ns", "host_done_ns",
                                                  "claim_ns", "done_ns")}
        for k in ("claimer", "claim_site", "inflight"):
            out[k] = np.zeros(E, np.int32)
        out["obs_ns"] = np.zeros((E, G), np.int64)
        log = L.EventLog()
        for k in out:
            setattr(log, k, out[k].ctypes.data)
        self._check(self._lib.apk_read_events(self._h, ctypes.byref(log)))
        out["n_injected"] = log.n_injected
        out["n_fired"] = log.n_fired
        out["grid"] = log.grid
        return out

    def read_oracle(self, num_tasks: int | None):
        ex = np.zeros(num_tasks, np.int32) if num_tasks else None
        ue = np.zeros(self.cfg.max_events, np.int32)
        self._check(self._lib.apk_read_oracle(self._h, _ptr(ex) if ex is not None else None, _ptr(ue)))
        return ex, ue

    def run_stats(self) -> dict:
        s = L.RunStats()
        self._check(self._lib.apk_read_run_stats(self._h, ctypes.byref(s)))
        return {f: getattr(s, f) for f, _ in L.RunStats._fields_}

    # ------------------------------------------------------------ one-shots
    def gemm(self, A: np.ndarray, B: np.ndarray, C: np.ndarray | None = None) -> np.ndarray:
        M, K = A.shape
        K2, N = B.shape
        assert K == K2
        if C is None:
            C = np.empty((M, N), np.float32)
        self._check(self._lib.apk_gemm(self._h, _ptr(A), _ptr(B), _ptr(C), M, N, K, L.APK_MEM_HOST))
        self.M, self.N, self.K = M, N, K
        return C

    def probe_copy(self, A: np.ndarray, B: np.ndarray, C: np.ndarray, reps: int = 5) -> dict:
        """Copy ceiling of gemm() from these host buffers (no kernel): ms of
        A+B in, C out, and both at once (medians over reps)."""
        out = np.zeros(3, np.float64)
        self._check(self._lib.apk_probe_copy(self._h, _ptr(A), _ptr(B), _ptr(C), reps, _ptr(out)))
        return {"h2d_ms": float(out[0]), "d2h_ms": float(out[1]), "both_ms": float(out[2])}

    def gemm_device(self, A_ptr: int, B_ptr: int, C_ptr: int, M: int, N: int, K: int):
        self._check(self._lib.apk_gemm(self._h, ctypes.c_void_p(A_ptr), ctypes.c_void_p(B_ptr),
                                       ctypes.c_void_p(C_ptr), M, N, K, L.APK_MEM_DEVICE))
        self.M, self.N, self.K = M, N, K

    # ---------------------------------------------------------------- modes
    def run_latency(self, events: int, period_us: float = 1000.0, seed: int = 21, warmup_events: int = 0,
                    settle_ms: float = 20.0, bg_tasks: int = 0, probe_reps: int = 64,
                    poisson: bool = False) -> dict:
        """bg_tasks = 0: unbounded launch stopped after the last event;
        bg_tasks > 0: a bounded launch that ends by itself.  probe_reps:
        host-set visibility calibration reps (0 = host round trips only).
        poisson: exponential gaps with mean period_us instead of one arrival
        per period."""
        lc = L.LatencyConfig(events, int(period_us * 1000), seed, warmup_events, int(settle_ms * 1e6),
                             int(bg_tasks), int(probe_reps), int(poisson))
        r = L.LatencyResult()
        self._check(self._lib.apk_run_latency(self._h, ctypes.byref(lc), ctypes.byref(r)))
        return {f: getattr(r, f) for f, _ in L.LatencyResult._fields_}

    def probe_visibility(self, reps: int = 64) -> np.ndarray:
        out = np.zeros(reps, np.int64)
        self._check(self._lib.apk_probe_visibility(self._h, reps, _ptr(out)))
        return out

    def run_visibility(self, events: int = 1000, gap_us=(150.0, 400.0), seed: int = 21, warmup_events: int = 100,
                       work_iters: int = 0, loaded: bool = False, traffic_bytes: int = 0, raw: bool = False):
        """Flag-visibility microbenchmark (no tile work).  Returns the summary
        dict; with raw=True also (set_ns, obs_ns[events][grid]) for OBS1."""
        vc = L.VisibilityConfig(events, int(gap_us[0] * 1000), int(gap_us[1] * 1000), seed, warmup_events,
                                work_iters, int(loaded), int(traffic_bytes))
        r = L.VisibilityResult()
        grid = self.info["grid"]
        set_ns = np.zeros(events, np.int64)
        obs_ns = np.zeros((events, grid), np.int64)
        self._check(self._lib.apk_run_visibility(self._h, ctypes.byref(vc), ctypes.byref(r), _ptr(set_ns),
                                                 _ptr(obs_ns)))
        res = {f: getattr(r, f) for f, _ in L.VisibilityResult._fields_}
        return (res, set_ns, obs_ns) if raw else res

    def run_overhead(self, num_tasks: int, reps: int = 5):
        a = ctypes.c_double()
        b = ctypes.c_double()
        self._check(self._lib.apk_run_overhead(self._h, num_tasks, reps, ctypes.byref(a), ctypes.byref(b)))
        return a.value, b.value

    def run_baseline(self, num_tasks: int, trials: int, seed: int = 21) -> np.ndarray:
        out = np.zeros(trials, np.float64)
        self._check(self._lib.apk_run_baseline(self._h, num_tasks, trials, seed, _ptr(out)))
        return out

    def run_reserved(self, num_tasks: int, reserve: int, trials: int, seed: int = 21):
        """Reserved-capacity arm: (e2e_us per trial, background TFLOP/s with
        `reserve` resident slots held out)."""
        out = np.zeros(trials, np.float64)
        tf = ctypes.c_double()
        self._check(self._lib.apk_run_reserved(self._h, num_tasks, reserve, trials, seed, _ptr(out),
                                               ctypes.byref(tf)))
        return out, tf.value
