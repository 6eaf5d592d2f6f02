"""The index arithmetic the tile kernel and the stack runner rely on, restated
on the CPU over many (row blocks, K blocks, grid) combinations:

* aligned splits (gemm_tm.cuh, launch_tm / tm_choose_grid): with G = NB * S
  CTAs over U = NB * KB tiles, CTA i's range [i*U/G, (i+1)*U/G) stays inside
  row block i // S, and the S CTAs of a row block cover it exactly -- for any
  1 <= S <= KB, powers of two or not (floor(KB/S) or ceil(KB/S) K blocks each);
* the split-K hand-off (gemm_tm.cuh epilogue, stack.cuh epilogue): the owners
  of a row block's first and last tile, i_lo = ((first+1)*G - 1) // U and
  i_hi = ((last+1)*G - 1) // U, bracket exactly the CTAs holding a partial of
  it; every contributor after i_lo starts inside the row block (slot 0), and
  i_lo's slot is 0 only if its range starts at the row block's first tile;
* the stack runner's spread of a linear over Gl = min(G, U) CTAs
  (stack.cuh, st_range): every CTA below Gl holds at least one tile.
"""
import itertools

import pytest


def ranges(U, G):
    return [((i * U) // G, ((i + 1) * U) // G) for i in range(G)]


@pytest.mark.parametrize("NB", [1, 4, 8, 16, 32, 48, 192])
def test_aligned_splits_cover_their_row_block(NB):
    for KB in (1, 8, 20, 32, 76, 81, 96):
        for S in range(1, min(KB, 16) + 1):
            G, U = NB * S, NB * KB
            for i, (a, b) in enumerate(ranges(U, G)):
                nb = i // S
                assert nb * KB <= a < b <= (nb + 1) * KB
            for nb in range(NB):
                assert ranges(U, G)[nb * S][0] == nb * KB
                assert ranges(U, G)[nb * S + S - 1][1] == (nb + 1) * KB


def contributors(NB, KB, G):
    """row block -> [(CTA, slot)] for the CTAs that leave a partial of it
    (slot 0: the CTA's first segment, 1: its last), from the ranges alone."""
    U = NB * KB
    out = {}
    for i, (u0, u1) in enumerate(ranges(U, G)):
        u = u0
        while u < u1:
            nb = u // KB
            end = min(u1, (nb + 1) * KB)
            whole = u % KB == 0 and end == (nb + 1) * KB
            if not whole:
                out.setdefault(nb, []).append((i, 0 if u == u0 else 1))
            u = end
    return out


@pytest.mark.parametrize("NB, KB", list(itertools.product([1, 2, 3, 6, 32, 48, 192, 1187], [1, 2, 4, 32, 96])))
def test_split_k_owners_and_slots(NB, KB):
    U = NB * KB
    for G in (7, 64, 148, 192, 296):
        Gl = min(G, U)                      # the stack runner's spread; the tile kernel has G <= U
        for a, b in ranges(U, Gl):
            assert b > a                    # every working CTA holds a tile
        parts = contributors(NB, KB, Gl)
        for nb in range(NB):
            first, last = nb * KB, nb * KB + KB - 1
            i_lo = ((first + 1) * Gl - 1) // U
            i_hi = ((last + 1) * Gl - 1) // U
            if i_lo == i_hi:
                assert nb not in parts      # one CTA holds the whole row block: stored directly
                continue
            got = sorted(parts[nb])
            assert [i for i, _ in got] == list(range(i_lo, i_hi + 1))
            si_lo = 0 if (i_lo * U) // Gl == first else 1
            for i, slot in got:
                assert slot == (si_lo if i == i_lo else 0)
