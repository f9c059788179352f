"""Host-side planning of the host-resident pipeline (llmx_b200.streaming):
which (batch, row) pieces are uploaded, computed and downloaded, in order."""
import pytest

from llmx_b200.streaming import plan_pieces


@pytest.mark.parametrize("ranges,S,tail", [
    ([(0, 1), (1, 2), (2, 8)], 2048, 2), ([(0, 8)], 2048, 4), ([(0, 3)], 1000, 3), ([(0, 2), (2, 4)], 512, 2),
    ([(0, 1)], 300, 4), ([(0, 4)], 2048, 1), ([(0, 2), (2, 3)], 4096, 8)])
def test_pieces_cover_every_row_once_in_order(ranges, S, tail):
    pieces = plan_pieces(ranges, S, tail)
    covered = [(b, r) for b0, b1, r0, r1 in pieces for b in range(b0, b1) for r in range(r0, r1)]
    assert sorted(covered) == [(b, r) for b in range(ranges[-1][1]) for r in range(S)]
    assert len(covered) == len(set(covered))
    # only the last batch element is cut, at multiples of 128 rows
    for b0, b1, r0, r1 in pieces:
        if (r0, r1) != (0, S):
            assert (b0, b1) == (ranges[-1][1] - 1, ranges[-1][1])
            assert r0 % 128 == 0 and (r1 % 128 == 0 or r1 == S)
    last = [p for p in pieces if p[0] <= ranges[-1][1] - 1 < p[1]]  # pieces holding the last element
    n_cut = len(last)
    if tail > 1 and S >= 2 * tail * 128:
        assert n_cut == tail
    else:
        assert n_cut == 1 and last[0][2:] == (0, S)


def test_pieces_without_a_cut_are_the_chunks():
    ranges = [(0, 3), (3, 5), (5, 8)]
    assert plan_pieces(ranges, 2048, 1) == [(a, b, 0, 2048) for a, b in ranges]
