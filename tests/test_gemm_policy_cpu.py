"""Host-side choices of the own GEMM (no GPU needed): tile width, raster group, K split and the size gate,
for a B200's 74 CTA pairs."""

import pytest

from rl_project_b200.ops import gemm


@pytest.fixture(autouse=True)
def b200_pairs(monkeypatch):
    monkeypatch.setitem(gemm._CLUSTERS, 0, 74)
    monkeypatch.setattr(gemm, "_NSUB", 0)
    monkeypatch.setattr(gemm, "_GROUP_M", 0)
    monkeypatch.setattr(gemm, "_SPLITK", "auto")
    monkeypatch.setattr(gemm, "_MIN_TILES", -1)


def test_weight_gradients_take_wide_tiles_and_split_k_where_waves_are_short():
    # dense-1B weight gradients: (out features, in features, tokens)
    assert gemm.nsub_for(3072, 2048, 0, 0, a_mn=1) == 2
    assert gemm.k_splits(3072, 2048, 32768, 2, 0) == 3      # 48 tiles -> 144 units, 1.95 waves
    assert gemm.k_splits(2048, 8192, 32768, 2, 0) == 4      # 128 tiles -> 512 units
    assert gemm.k_splits(128256, 2048, 32768, 2, 0) == 1    # 2004 tiles: 27 waves already
    assert gemm.k_splits(4096, 4096, 256, 2, 0) == 1        # K too short to divide


def test_split_k_override_and_off(monkeypatch):
    monkeypatch.setattr(gemm, "_SPLITK", "off")
    assert gemm.k_splits(3072, 2048, 32768, 2, 0) == 1
    monkeypatch.setattr(gemm, "_SPLITK", "5")
    assert gemm.k_splits(3072, 2048, 32768, 2, 0) == 5
    assert gemm.k_splits(3072, 2048, 128, 2, 0) == 2        # never more ranges than 64-deep K slices


def test_raster_group_for_wide_outputs_only():
    assert gemm.group_for(16384, 0) == 32 and gemm.group_for(128256, 0) == 32 and gemm.group_for(8192, 0) == 32
    assert gemm.group_for(2048, 0) == 8 and gemm.group_for(16384, 1) == 8


def test_forward_tile_width_follows_wave_fill():
    assert gemm.nsub_for(32768, 16384, 0, 0) == 2
    assert gemm.nsub_for(32768, 256, 0, 0) == 1             # too narrow for 512 columns
    assert gemm.nsub_for(32768, 2048, 1, 0) == 1            # fp32 output: 256-wide tiles


def test_small_products_go_to_cublas():
    assert gemm.fills_gpu(32768, 2048, 512, 0)               # 128 x 4 tiles
    assert not gemm.fills_gpu(64, 2048, 512, 0)              # a decode step: 4 tiles for 74 pairs
    assert not gemm.fills_gpu(1024, 3072, 512, 0)
    gemm._MIN_TILES = 0
    assert gemm.fills_gpu(64, 2048, 512, 0)
