"""The block split of the host-operand streaming path (titan_rs_b200.streaming.split_rows),
on the CPU: blocks cover every row once, in order, never more blocks than asked, and
256-row multiples (CTA-pair tiles) whenever the rows allow it."""
import pytest

from titan_rs_b200.streaming import split_rows


@pytest.mark.parametrize("rows,blocks", [(8192, 4), (2048, 4), (1000, 3), (1000, 4), (1, 4), (7, 3), (300, 1),
                                         (4096, 3), (255, 2), (1024, 4), (1025, 4)])
def test_split_rows_covers_every_row_in_order(rows, blocks):
    parts = split_rows(rows, blocks)
    assert 1 <= len(parts) <= blocks
    assert parts[0][0] == 0
    for (r0, n), (r1, _) in zip(parts, parts[1:]):
        assert r1 == r0 + n and n > 0
    assert parts[-1][0] + parts[-1][1] == rows
    if rows >= 256 * blocks:
        assert all(n % 256 == 0 for _, n in parts[:-1])


def test_split_rows_of_c3_is_four_2048_row_blocks():
    assert split_rows(8192, 4) == [(0, 2048), (2048, 2048), (4096, 2048), (6144, 2048)]


def test_split_rows_rejects_empty_inputs():
    with pytest.raises(ValueError):
        split_rows(0, 4)
    with pytest.raises(ValueError):
        split_rows(8, 0)
