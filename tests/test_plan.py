"""CPU tests of dispatch and the reference's tile tables (no GPU).

Port of the reference's tests/test_plan.py: same assertions, same private
names (_geom_ok, _pick_bk, _pick_tiles, conv3d_plan).
"""
import os

os.environ.setdefault("RDNA4_CONV3D_BACKEND", "hybrid")

from rdna4_conv3d.conv3d_wmma import _geom_ok, _pick_bk, _pick_tiles, _split_k, conv3d_plan


def test_geom_ok_k1_k3_only():
    assert _geom_ok(3, 1, 1, 1)
    assert _geom_ok(1, 1, 1, 1)
    assert _geom_ok((3, 3, 3), (1, 1, 1), (1, 1, 1), 1)
    assert not _geom_ok(5, 1, 1, 1)
    assert not _geom_ok(3, 2, 1, 1)
    assert not _geom_ok(3, 1, 2, 1)
    assert not _geom_ok(3, 1, 1, 2)
    assert not _geom_ok((3, 3, 1), 1, 1, 1)


def test_pick_bk_fit_not_straddle():
    assert _pick_bk(24) == 16
    assert _pick_bk(48) == 16
    assert _pick_bk(32) == 32
    assert _pick_bk(96) == 32
    assert _pick_bk(192) == 32


def test_wgrad_tiles_split_on_cout():
    bm, bn, bk, warps, stages = _pick_tiles(24, 24 * 27, 64 * 128 * 128, "wgrad")
    assert bk == 32 and warps == 8 and stages == 2
    _, _, bk2, warps2, _ = _pick_tiles(48, 48 * 27, 32 * 64 * 64, "wgrad")
    assert bk2 == 64 and warps2 == 4
    _, _, _, warps1, _ = _pick_tiles(1, 24 * 1, 64 * 128 * 128, "wgrad")
    assert warps1 == 4


def test_fwd_tile_table():
    # BLOCK_N follows N (and M for the 33..64 band); BLOCK_M follows M.
    assert _pick_tiles(100000, 16, 24)[:2] == (128, 16)
    assert _pick_tiles(100000, 24, 24)[:2] == (128, 32)
    assert _pick_tiles(100000, 48, 48)[:2] == (128, 64)
    assert _pick_tiles(1000, 48, 48)[:2] == (64, 32)
    assert _pick_tiles(1000, 64, 48)[:2] == (64, 64)
    assert _pick_tiles(10, 192, 192)[:2] == (32, 64)
    assert _pick_tiles(100000, 192, 192, "dgrad")[3] == 8


def test_split_k_bounds():
    assert _split_k(24, 648, 64 * 128 * 128, 32, 64, 32) == 32
    assert _split_k(24, 648, 100, 32, 64, 32) == 1
    assert 1 <= _split_k(192, 5184, 10 ** 6, 64, 64, 64) <= 32


def test_plan_values_are_wmma_or_miopen():
    plan = conv3d_plan(24, 24, 3)
    assert set(plan) == {"fwd", "dw", "dx"}
    assert plan["fwd"] in ("wmma", "miopen")
    slow = conv3d_plan(24, 24, 3, stride=2)
    assert slow == {"fwd": "miopen", "dw": "miopen", "dx": "miopen"}
