"""Host logic of the configs[3] surface runner: which cells cannot run and
why (no GPU needed)."""
from apk_b200.config3 import CTAS, KTILES, SHAPES, _infeasible_reason


def test_surface_has_24_cells_per_dtype():
    assert len(CTAS) * len(KTILES) * len(SHAPES) == 24


def test_k_tile_128_is_reported_infeasible():
    for dtype in ("f32", "bf16"):
        r = _infeasible_reason(dtype, 1, 128, None)
        assert r is not None and "K-tile 128" in r


def test_cta_count_above_residency_is_reported():
    info = {"ctas_per_sm": 2, "max_ctas_per_sm": 2}
    assert _infeasible_reason("f32", 2, 32, info) is None
    info4 = {"ctas_per_sm": 2, "max_ctas_per_sm": 2}
    r = _infeasible_reason("f32", 4, 32, info4)
    assert r is not None and "at most 2" in r
    r = _infeasible_reason("bf16", 2, 64, {"ctas_per_sm": 1, "max_ctas_per_sm": 1})
    assert r is not None and "TMEM" in r
