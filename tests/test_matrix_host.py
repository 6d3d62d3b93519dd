"""Host-side checks of the per-frame cross-attention harness (bench_matrix.py)."""

from __future__ import annotations

import pytest


def test_config5_cells_and_flops():
    import bench_matrix as matrix
    cells = matrix.cell_order()
    assert len(cells) == 5 * 4 * 2
    assert {c.policy for c in cells} == {"none", "uniform", "recency", "motion", "reuse_weighted"}
    # None leads every (regime, budget) group: the other policies are checked against it
    for i in range(0, len(cells), 5):
        assert cells[i].policy == "none"
        assert len({(c.regime, c.budget_frac) for c in cells[i:i + 5]}) == 1
    # 16 frames x 1560 tokens x 12 heads: 2.0335e12 FLOP per cell
    assert matrix.cross_flops(16, 1560, 12) == pytest.approx(2.0335e12, rel=1e-4)
    # config 2: 8 frames
    assert matrix.cross_flops(8, 1560, 12) == pytest.approx(5.383e11, rel=1e-3)


def test_config5_regimes_shapes():
    from kvp.traces import motion_config5
    s = motion_config5("static", frames=16)
    h = motion_config5("high", frames=16)
    assert s.shape == h.shape == (16, 98)
    assert s.max() < 0.05 and h.max() < 1.0 and h.max() > 0.5


def test_config3_flops():
    import bench_matrix as matrix
    # 50 frames, window of 5 frames: 240 frame-units per (layer, head); 1.0765e14 FLOP
    assert matrix.window_flops(50, 1560, 12, 30, 5) == pytest.approx(1.0765e14, rel=1e-4)
    assert matrix.window_flops(3, 1560, 12, 1, 5) == pytest.approx(matrix.cross_flops(3, 1560, 12))


@pytest.mark.parametrize("order", ["ascending", "descending", "permuted"])
def test_slot_order_maps(order):
    """--matrix 10 maps: whole 16-row tiles, every slot used once; ascending
    and descending runs inside each tile as named."""
    import torch
    from bench_matrix import slot_order_map
    m, rows, slots = slot_order_map(32760, 16, 640, order, seed=1, device="cpu")
    assert rows.numel() == 10240 and int((m >= 0).sum()) == 10240
    assert sorted(slots.tolist()) == list(range(10240))
    assert bool((rows % 32 < 16).all())                     # every other tile
    per_tile = m[rows].view(-1, 16)
    d = per_tile[:, 1:] - per_tile[:, :-1]
    if order == "ascending":
        assert bool((d == 1).all())
    elif order == "descending":
        assert bool((d == -1).all())
    else:
        assert not bool((d == 1).all()) and not bool((d == -1).all())
    with pytest.raises(ValueError):
        slot_order_map(64, 16, 1, "sideways", seed=0, device="cpu")
