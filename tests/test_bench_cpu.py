"""Host-side helpers of bench.py (no GPU): the e2e leg's query chunking."""
import os
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


@pytest.mark.parametrize("blocks", [[(0, 131072)], [(0, 8192), (122880, 131072)], [(0, 5000)],
                                    [(0, 1000)], [(4096, 4096 + 70000)]])
def test_e2e_chunks_partition_each_block(blocks):
    import bench
    chunks = bench.e2e_chunks(blocks)
    # ascending, contiguous, covering every block exactly once
    covered = []
    for (bs, be) in blocks:
        mine = [c for c in chunks if bs <= c[0] < be]
        assert mine[0][0] == bs and mine[-1][1] == be
        for (a0, a1), (b0, b1) in zip(mine, mine[1:]):
            assert a1 == b0
        covered += mine
    assert covered == chunks
    assert all(c1 > c0 and c1 - c0 <= 16384 for c0, c1 in chunks)


def test_e2e_chunks_shape_at_128k():
    import bench
    chunks = bench.e2e_chunks([(0, 131072)])
    sizes = [c1 - c0 for c0, c1 in chunks]
    assert sizes[:4] == [2048, 4096, 8192, 16384]
    assert sizes[-1] == 4096
