"""tileLimit on CUDA: an integer limit bounds the output extent of one
convolution launch (the reference bounds the OpenGL tile a convolution pass
renders into, drivers/matrixman/config.py:305-314 and
backends/opengl/convolution.py:1299); ``auto`` means no bound.  These CPU
tests cover the region decomposition and the mapping from the setting; the
GPU tests check that tiled convolutions equal untiled ones bit for bit."""

import pytest

from matrixman_b200 import ops


def test_regions_cover_output_once_in_row_major_order():
    for oh, ow, cap in [(320, 320, 256), (37, 45, 16), (5, 5, 1), (20, 20, 7), (8, 3, 8)]:
        regions = ops.conv_regions(oh, ow, cap)
        covered = [[0] * ow for _ in range(oh)]
        for r0, c0, rows, cols in regions:
            assert 0 < rows <= cap and 0 < cols <= cap
            for i in range(r0, r0 + rows):
                for j in range(c0, c0 + cols):
                    covered[i][j] += 1
        assert all(v == 1 for row in covered for v in row)
        assert regions == sorted(regions)


def test_one_region_when_uncapped_or_fitting():
    assert ops.conv_regions(640, 480, None) == [(0, 0, 640, 480)]
    assert ops.conv_regions(256, 256, 256) == [(0, 0, 256, 256)]
    assert len(ops.conv_regions(320, 320, 256)) == 4
    with pytest.raises(ValueError):
        ops.conv_regions(4, 4, 0)


def test_cap_follows_the_setting_and_its_override():
    """The default (256, as the reference reports it) and ``auto`` keep one
    launch per convolution, like the reference's CUDA backend; a value the user
    sets caps each launch."""
    from matrixman_b200.config import Configuration, config
    value = config.tileLimit
    explicit = config.source("tileLimit") != "default" and value != "auto"
    assert ops.conv_tile_cap() == (int(value) if explicit else None)
    assert ops.conv_tile_cap(None) is None
    assert ops.conv_tile_cap(12) == 12
    cfg = Configuration()
    assert cfg.tile_limit == 256 and cfg.source("tile_limit") == "default"
