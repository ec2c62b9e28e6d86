"""Tile-width and split-K choices of the GEMM wrapper (host arithmetic, CPU)."""

from packbalance_b200.ops.gemm import pick_bn, pick_tiling

SMS = 148  # B200


def test_narrow_outputs_take_192_wide_tiles() -> None:
    # N = 768: 192 tiles of 128 x 256 are 1.3 waves on 148 SMs, 256 tiles of 128 x 192
    # are 1.73 waves
    assert pick_bn(8192, 768, SMS) == 192
    # wide outputs keep 256-wide tiles
    assert pick_bn(8192, 4096, SMS) == 256
    assert pick_bn(8192, 32000, SMS) == 256
    # without 192 in the allowed set (MN-major B), 256 stays
    assert pick_bn(8192, 768, SMS, (256, 128, 64)) == 256


def test_wgrad_split_k_fills_the_gpu() -> None:
    for m, n, k in ((768, 768, 8192), (768, 2048, 8192), (4096, 768, 8192), (1280, 768, 8192)):
        bn, splits = pick_tiling(m, n, k, SMS)
        assert bn in (256, 128, 64)
        tiles = -(-m // 128) * -(-n // bn) * splits
        assert tiles >= SMS * 0.8, (m, n, k, bn, splits)  # most SMs get a work unit
        assert -(-k // 64) // splits >= 4  # at least 4 k-blocks per split
