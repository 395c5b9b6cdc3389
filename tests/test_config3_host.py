"""Host logic of the configs[3] surface runner (no GPU needed): the 24 cells
per dtype, every cell with a geometry, and the occupancy report for a cell
whose CTAs would not all fit."""
from apk_b200.config3 import CTAS, KTILES, SHAPES, _infeasible_reason, geometry


def test_surface_has_24_cells_per_dtype():
    assert len(CTAS) * len(KTILES) * len(SHAPES) == 24
    assert KTILES == (32, 64, 128)


def test_every_cell_has_a_geometry():
    for dtype in ("f32", "bf16"):
        for cps in CTAS:
            assert geometry(dtype, cps)
            for kt in KTILES:
                assert _infeasible_reason(dtype, cps, kt, None) is None


def test_cta_count_above_residency_is_reported():
    info = {"ctas_per_sm": 2, "max_ctas_per_sm": 2}
    assert _infeasible_reason("f32", 2, 32, info) is None
    r = _infeasible_reason("f32", 4, 32, {"ctas_per_sm": 3, "max_ctas_per_sm": 3})
    assert r is not None and "at most 3" in r
