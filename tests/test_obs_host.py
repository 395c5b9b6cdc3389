"""OBS1 dump format and analyses (host only)."""
import json
import struct

import numpy as np
import pytest

from apk_b200 import obs


def _matrix(E=40, G=9, seed=0):
    rng = np.random.default_rng(seed)
    set_ns = (np.arange(E, dtype=np.int64) + 1) * 1_000_000
    obs_ns = set_ns[:, None] + rng.integers(1, 40, size=(E, G)) * 256
    obs_ns[:, 0] = set_ns  # the setter sees its own raise at once
    return set_ns, obs_ns


def test_round_trip_and_layout(tmp_path):
    s, o = _matrix()
    p = tmp_path / "x.obs1"
    obs.write(str(p), s, o)
    raw = p.read_bytes()
    assert struct.unpack("<3q", raw[:24]) == (0x3153424F, 40, 9)
    assert len(raw) == 24 + 8 * 40 + 8 * 40 * 9
    s2, o2 = obs.read(str(p))
    assert np.array_equal(s, s2) and np.array_equal(o, o2)


def test_bad_magic(tmp_path):
    p = tmp_path / "bad.obs1"
    p.write_bytes(struct.pack("<3q", 7, 0, 0))
    with pytest.raises(ValueError):
        obs.read(str(p))


def test_delays_cut_setter_unset_and_incomplete():
    s, o = _matrix(E=10, G=4)
    s[3] = 0
    o[5, 2] = 0
    rows, unset, incomplete = obs.delays(s, o, warmup=2)
    assert unset == 1 and incomplete == 1
    assert len(rows) == 10 - 2 - 2  # warm-up cut applies to complete events only
    assert all(len(r) == 3 for r in rows)  # CTA 0 (the setter) left out
    rows_all, _, _ = obs.delays(s, o, warmup=0, skip_setter=False)
    assert min(min(r) for r in rows_all) == 0.0


def test_quantiles_known_answer():
    rows = [[float(d) for d in range(1, 101)] for _ in range(7)]
    q = obs.quantiles(rows)
    assert (q["dmin_p50_us"], q["d50_p50_us"], q["d95_p50_us"], q["dmax_p50_us"]) == (1.0, 51.0, 96.0, 100.0)
    sp = obs.spread(rows)
    assert sp["spread_p50_us"] == 99.0 and sp["first_p50_us"] == 1.0


def test_independent_max_model_predicts_iid_maxima():
    rng = np.random.default_rng(21)
    rows = rng.exponential(2.0, size=(4000, 16)).tolist()
    m = obs.independent_max_model(rows)
    for q in m["quantiles"][:3]:
        assert abs(q["predicted_us"] - q["measured_us"]) / q["measured_us"] < 0.08, q


def test_quantum_floor_and_determinism():
    s, o = _matrix(E=200)
    assert abs(obs.timer_quantum_us(s, o) - 0.256) < 1e-12
    a = json.dumps(obs.analyze(s, o, warmup=10))
    b = json.dumps(obs.analyze(s, o, warmup=10))
    assert a == b
    fl = obs.analyze(s, o, warmup=10)["floor"]
    assert fl["events"] == 190 and fl["events_over_one_quantum"] == 190
