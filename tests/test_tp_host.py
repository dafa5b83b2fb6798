"""The row split of the N-sharded MUL_MAT (ggml_b200.tp.shard_rows), on the CPU: every rank's
block is whole 16-row groups, the blocks tile [0, N) in rank order without overlap, and they differ
in size by at most one group except where the weight runs out."""
import pytest

from ggml_b200.tp import shard_rows


@pytest.mark.parametrize("N", [16, 64, 496, 4096, 14336, 1008])
@pytest.mark.parametrize("G", [1, 2, 3, 4, 8])
def test_shard_rows_tile_the_weight(N, G):
    blocks = [shard_rows(N, G, r) for r in range(G)]
    assert blocks[0][0] == 0 and blocks[-1][1] == N
    for (lo, hi), (lo2, _) in zip(blocks, blocks[1:]):
        assert hi == lo2
    for lo, hi in blocks:
        assert lo % 16 == 0 and hi % 16 == 0 and 0 <= lo <= hi <= N
    full = [hi - lo for lo, hi in blocks if hi > lo]
    assert max(full) - min(full[:-1] or full) <= 16


def test_shard_rows_needs_16_row_groups():
    with pytest.raises(ValueError):
        shard_rows(100, 2, 0)
