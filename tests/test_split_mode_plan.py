"""Split-mode work division of the assignment kernel, restated in Python (no GPU).

With an uneven last wave, the (tile, chunk) units are cut into one contiguous range per
CTA (assign_tc.cu: SegIter). A tile cut by a range boundary is shared: each CTA that
touches it writes its per-row best to partial slot 2*cta + (first segment ? 0 : 1), and
splitk_fixup_kernel (one CTA per range boundary) merges them. This checks, for many
shapes, that every unit is processed exactly once, that every shared tile is merged by
exactly one boundary, and that the fixup reads exactly the slots the CTAs wrote."""

from __future__ import annotations

import itertools

import pytest


def segments(unit, units, total_tiles, nchunks):
    """SegIter(split=true).next() for CTA `unit`: [(tile, ch0, ch1), ...]."""
    U = total_tiles * nchunks
    u, u_end = unit * U // units, (unit + 1) * U // units
    out = []
    while u < u_end:
        tile = u // nchunks
        ch0 = u - tile * nchunks
        left = u_end - u
        ch1 = ch0 + left if left < nchunks - ch0 else nchunks
        out.append((tile, ch0, ch1))
        u += ch1 - ch0
    return out


def split_u0(c, U, G):
    return c * U // G


def split_cta_of(u, U, G):
    c = u * G // U
    while c + 1 < G and split_u0(c + 1, U, G) <= u:
        c += 1
    while c > 0 and split_u0(c, U, G) > u:
        c -= 1
    return c


def fixup_reads(G, total_tiles, nchunks):
    """{tile: [slots read]} of splitk_fixup_kernel (blocks c = 1 .. G-1)."""
    U = total_tiles * nchunks
    out = {}
    for c in range(1, G):
        u0 = split_u0(c, U, G)
        if u0 % nchunks == 0:
            continue
        t = u0 // nchunks
        t_begin = t * nchunks
        if split_u0(c - 1, U, G) > t_begin:
            continue
        c_first, c_last = split_cta_of(t_begin, U, G), split_cta_of(t_begin + nchunks - 1, U, G)
        assert t not in out, "a shared tile merged twice"
        out[t] = [2 * cc + (0 if split_u0(cc, U, G) >= t_begin else 1)
                  for cc in range(c_first, c_last + 1)]
    return out


SHAPES = [(G, T, C) for G, T, C in itertools.product([148, 96, 7], [150, 256, 300, 1000, 2049],
                                                      [2, 8, 32, 33])
          if T % G != 0 and T * C >= G]


@pytest.mark.parametrize("G,total_tiles,nchunks", SHAPES)
def test_split_mode_covers_and_merges(G, total_tiles, nchunks):
    written = {}  # tile -> slots written as partials
    covered = [0] * (total_tiles * nchunks)
    for cta in range(G):
        segs = segments(cta, G, total_tiles, nchunks)
        assert segs, "every CTA gets at least one unit when U >= G"
        for k, (tile, ch0, ch1) in enumerate(segs):
            for ch in range(ch0, ch1):
                covered[tile * nchunks + ch] += 1
            if ch0 != 0 or ch1 != nchunks:  # shared tile: partial slot
                written.setdefault(tile, []).append(2 * cta + (0 if k == 0 else 1))
    assert all(v == 1 for v in covered)
    reads = fixup_reads(G, total_tiles, nchunks)
    assert set(reads) == set(written)
    for t in written:
        assert sorted(reads[t]) == sorted(written[t]), t
        assert len(set(written[t])) == len(written[t])
