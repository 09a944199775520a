"""The assignment kernel's mbarrier protocol, simulated on the CPU (no GPU).

Each role of a CTA (TMA producer warp, MMA lane, each epilogue warp) runs as a
coroutine that performs the same barrier operations, in the same order and with the same
phase parities, as assign_tc.cu: waits on c_full/c_empty (centroid stages), x_full/x_empty
(row-tile buffers), acc_full/acc_empty (TMEM slots), merge_full/merge_empty (per-row best
exchange between the two column slices, crossed and deferred to the next tile). Copies
and MMAs complete at once. A scheduler runs whatever can run; the test fails if a state
is reached where no role can make progress before all have finished (a deadlock in the
kernel would be a wait that expires). Checked for every configuration the dispatch uses
(stages, slots, one or two row-tile buffers, sub-tile owners or column slices) and for
whole-tile and split-mode work lists."""

from __future__ import annotations

import itertools

import pytest

from test_split_mode_plan import segments


class Bar:
    def __init__(self, count):
        self.count, self.pending, self.phase = count, count, 0

    def arrive(self):
        self.pending -= 1
        assert self.pending >= 0
        if self.pending == 0:
            self.pending = self.count
            self.phase += 1

    def done(self, parity):
        # try_wait.parity(P): the phase of parity P has completed
        return (self.phase & 1) != parity


def wait(bar, parity):
    while not bar.done(parity):
        yield


def producer(B, segs, MT, ST, XS, nchunks):
    c_it = x_it = 0
    for tile, ch0, ch1 in segs:
        for ch in range(ch0, ch1):
            st, ph = c_it % ST, (c_it // ST) & 1
            yield from wait(B["c_empty"][st], ph ^ 1)
            B["c_full"][st].arrive()
            c_it += 1
            if ch == ch0:
                xb, xph = x_it % XS, (x_it // XS) & 1
                for s in range(MT):
                    xi = xb * MT + s
                    yield from wait(B["x_empty"][xi], xph ^ 1)
                    B["x_full"][xi].arrive()
        x_it += 1


def mma(B, segs, MT, ST, XS, slots):
    c_it = x_it = item = 0
    for tile, ch0, ch1 in segs:
        for ch in range(ch0, ch1):
            st, ph = c_it % ST, (c_it // ST) & 1
            yield from wait(B["c_full"][st], ph)
            for s in range(MT):
                xi = (x_it % XS) * MT + s
                if ch == ch0:
                    yield from wait(B["x_full"][xi], (x_it // XS) & 1)
                slot = item % slots
                yield from wait(B["acc_empty"][slot], ((item // slots) & 1) ^ 1)
                B["acc_full"][slot].arrive()  # tcgen05.commit
                if ch == ch1 - 1:
                    B["x_empty"][xi].arrive()
                item += 1
            B["c_empty"][st].arrive()
            c_it += 1
        x_it += 1


def owner_warp(B, segs, MT, slots, part):
    item = 0
    for tile, ch0, ch1 in segs:
        for ch in range(ch0, ch1):
            for s in range(MT):
                if s == part:
                    slot = item % slots
                    yield from wait(B["acc_full"][slot], (item // slots) & 1)
                    B["acc_empty"][slot].arrive()
                item += 1


def slice_warp(B, segs, MT, slots, part):
    peer = part ^ 1
    owns = part < MT
    sends = MT > 1 or part == 1
    item = tcount = 0
    pending = False

    def finish():
        nonlocal pending
        yield from wait(B["merge_full"][peer], (tcount & 1) ^ 1)
        B["merge_empty"][peer].arrive()
        pending = False

    for tile, ch0, ch1 in segs:
        for ch in range(ch0, ch1):
            for s in range(MT):
                slot = item % slots
                yield from wait(B["acc_full"][slot], (item // slots) & 1)
                B["acc_empty"][slot].arrive()
                item += 1
                if pending:
                    yield from finish()
        if sends:
            yield from wait(B["merge_empty"][part], (tcount & 1) ^ 1)
            B["merge_full"][part].arrive()
        if owns:
            pending = True
        tcount += 1
    if pending:
        yield from finish()


def producer_xs(B, segs, ST, XS, PB, norm_first=True):
    """Streamed x (split fp32 rows wider than 512 elements, MT = 1): per tile the norm
    slice into the row-tile buffer, then per chunk PB stages of one column block each."""
    c_it = x_it = 0
    for tile, ch0, ch1 in segs:
        for ch in range(ch0, ch1):
            if ch == ch0 and norm_first:
                xi, xph = x_it % XS, (x_it // XS) & 1
                yield from wait(B["x_empty"][xi], xph ^ 1)
                B["x_full"][xi].arrive()
            for j in range(PB):
                st, ph = c_it % ST, (c_it // ST) & 1
                yield from wait(B["c_empty"][st], ph ^ 1)
                B["c_full"][st].arrive()
                c_it += 1
            if ch == ch0 and not norm_first:
                xi, xph = x_it % XS, (x_it // XS) & 1
                yield from wait(B["x_empty"][xi], xph ^ 1)
                B["x_full"][xi].arrive()
        x_it += 1


def mma_xs(B, segs, ST, XS, slots, PB):
    c_it = x_it = item = 0
    for tile, ch0, ch1 in segs:
        for ch in range(ch0, ch1):
            xi = x_it % XS
            if ch == ch0:
                yield from wait(B["x_full"][xi], (x_it // XS) & 1)
            slot = item % slots
            yield from wait(B["acc_empty"][slot], ((item // slots) & 1) ^ 1)
            for j in range(PB):
                st, ph = c_it % ST, (c_it // ST) & 1
                yield from wait(B["c_full"][st], ph)
                B["c_empty"][st].arrive()
                c_it += 1
            B["acc_full"][slot].arrive()
            if ch == ch1 - 1:
                B["x_empty"][xi].arrive()
            item += 1
        x_it += 1


def run_cta(segs, MT, ST, NC, XS, own, nchunks, acc_empty_count=None, PB=0, norm_first=True):
    slots = 512 // NC
    if acc_empty_count is None:
        acc_empty_count = 4 if own else 8
    B = {
        "c_full": [Bar(1) for _ in range(ST)], "c_empty": [Bar(1) for _ in range(ST)],
        "x_full": [Bar(1) for _ in range(XS * MT)], "x_empty": [Bar(1) for _ in range(XS * MT)],
        "acc_full": [Bar(1) for _ in range(slots)],
        "acc_empty": [Bar(acc_empty_count) for _ in range(slots)],
        "merge_full": [Bar(4) for _ in range(2)], "merge_empty": [Bar(4) for _ in range(2)],
    }
    if PB:
        roles = [producer_xs(B, segs, ST, XS, PB, norm_first), mma_xs(B, segs, ST, XS, slots, PB)]
    else:
        roles = [producer(B, segs, MT, ST, XS, nchunks), mma(B, segs, MT, ST, XS, slots)]
    for w in range(8):  # epilogue warps 2..9: half = (w >> 2)
        part = w >> 2
        roles.append(owner_warp(B, segs, MT, slots, part) if own
                     else slice_warp(B, segs, MT, slots, part))
    live = list(roles)

    def state():
        return [(b.phase, b.pending) for v in B.values() for b in v]

    while live:
        # one sweep: every live role runs until it blocks (yields) or finishes
        before, finished = state(), False
        for r in list(live):
            try:
                next(r)
            except StopIteration:
                live.remove(r)
                finished = True
        if not finished and state() == before:
            raise AssertionError("deadlock: no role can make progress")


# (DB, MT, NC, ST) of the single-CTA dispatch, with kXS and ownership as the kernel derives
CONFIGS = [
    # D <= 64: two x buffers, sub-tile owners
    dict(MT=2, NC=256, ST=3, XS=2, own=True),
    # D <= 128: column slices with the crossed, deferred merge
    dict(MT=2, NC=256, ST=2, XS=1, own=False),
    # D <= 192: 128-centroid chunks, owners, four slots
    dict(MT=2, NC=128, ST=2, XS=1, own=True),
    # D <= 256 (MT = 1): column slices, slice 1 sends, slice 0 finishes
    dict(MT=1, NC=128, ST=2, XS=1, own=False),
    # split fp32, 192 < D <= 384: x streamed, four to six column blocks per item
    dict(MT=1, NC=128, ST=3, XS=2, own=False, PB=4),
    dict(MT=1, NC=128, ST=3, XS=2, own=False, PB=5),
    dict(MT=1, NC=128, ST=3, XS=2, own=False, PB=6),
    # fp16/bf16, 384 < D <= 512: x streamed with 256-centroid chunks, 7 or 8 blocks per item
    dict(MT=1, NC=256, ST=3, XS=2, own=False, PB=7),
    dict(MT=1, NC=256, ST=3, XS=2, own=False, PB=8),
]


@pytest.mark.parametrize("cfg", CONFIGS, ids=lambda c: "-".join(f"{k}{v}" for k, v in c.items()))
@pytest.mark.parametrize("total_tiles,nchunks,units", [(7, 1, 3), (9, 4, 4), (20, 3, 6),
                                                       (5, 8, 3), (13, 2, 13), (300, 2, 148)])
def test_no_deadlock(cfg, total_tiles, nchunks, units):
    # whole-tile mode (tile, tile + units, ...) and split mode (contiguous unit ranges)
    for unit in range(min(units, 6)):
        whole = [(t, 0, nchunks) for t in range(unit, total_tiles, units)]
        run_cta(whole, nchunks=nchunks, **cfg)
        if total_tiles * nchunks >= units:
            run_cta(segments(unit, units, total_tiles, nchunks), nchunks=nchunks, **cfg)


def test_streamed_x_needs_the_norm_slice_first():
    # the tile's norm slice requested after the chunk's stages: with more column blocks
    # than stages the producer waits for a stage the MMA cannot free (it waits for the
    # norm slice first), which the kernel avoids by loading the norm slice first
    with pytest.raises(AssertionError, match="deadlock"):
        run_cta([(0, 0, 2), (1, 0, 2)], MT=1, ST=3, NC=128, XS=2, own=False, nchunks=2, PB=6,
                norm_first=False)


def test_simulator_detects_a_broken_protocol():
    # one arrival too many expected on the slot barriers: the MMA must stall for good
    with pytest.raises(AssertionError, match="deadlock"):
        run_cta([(0, 0, 4), (1, 0, 4)], MT=2, ST=2, NC=256, XS=1, own=False, nchunks=4,
                acc_empty_count=9)


def run_pair(segs, MT, ST, NC, XS, own, nchunks):
    """CTA pair (cta_group::2): both CTAs load their halves into the leader's full
    barriers (modelled as one arrival each), the leader's MMA lane commits to both CTAs'
    empty/full barriers (multicast), and both CTAs' epilogue warps release the leader's
    slot barriers."""
    slots = 512 // NC
    per = 4 if own else 8

    def cta_bars():
        return {
            "c_full": [Bar(2) for _ in range(ST)], "c_empty": [Bar(1) for _ in range(ST)],
            "x_full": [Bar(2) for _ in range(XS * MT)],
            "x_empty": [Bar(1) for _ in range(XS * MT)],
            "acc_full": [Bar(1) for _ in range(slots)],
            "acc_empty": [Bar(2 * per) for _ in range(slots)],
            "merge_full": [Bar(4) for _ in range(2)], "merge_empty": [Bar(4) for _ in range(2)],
        }

    lead, follow = cta_bars(), cta_bars()

    class Multicast:
        """Commit targets: the same barrier in both CTAs."""

        def __init__(self, a, b):
            self.a, self.b = a, b

        def arrive(self):
            self.a.arrive()
            self.b.arrive()

    mma_view = dict(lead)
    for k in ("c_empty", "x_empty", "acc_full"):
        mma_view[k] = [Multicast(a, b) for a, b in zip(lead[k], follow[k])]

    def producer_of(own_bars):
        view = dict(own_bars)
        view["c_full"], view["x_full"] = lead["c_full"], lead["x_full"]
        return producer(view, segs, MT, ST, XS, nchunks)

    def epi_of(own_bars, part):
        view = dict(own_bars)
        view["acc_empty"] = lead["acc_empty"]
        return (owner_warp(view, segs, MT, slots, part) if own
                else slice_warp(view, segs, MT, slots, part))

    roles = [producer_of(lead), producer_of(follow), mma(mma_view, segs, MT, ST, XS, slots)]
    for bars in (lead, follow):
        for w in range(8):
            roles.append(epi_of(bars, w >> 2))
    live = list(roles)

    def state():
        return [(b.phase, b.pending) for B in (lead, follow) for v in B.values() for b in v]

    while live:
        before, finished = state(), False
        for r in list(live):
            try:
                next(r)
            except StopIteration:
                live.remove(r)
                finished = True
        if not finished and state() == before:
            raise AssertionError("deadlock: no role can make progress")


PAIR_CONFIGS = [
    dict(MT=1, NC=64, ST=2, XS=1, own=False),    # 384 < D <= 512 (pairs opted in)
    dict(MT=1, NC=128, ST=2, XS=1, own=False),   # 256 < D <= 384
    dict(MT=2, NC=256, ST=8, XS=1, own=True),    # D <= 64 (pairs opted in)
    dict(MT=2, NC=256, ST=4, XS=1, own=False),   # D <= 128 (pairs opted in)
    dict(MT=1, NC=256, ST=2, XS=1, own=False),   # D <= 256 (pairs opted in)
]


@pytest.mark.parametrize("cfg", PAIR_CONFIGS, ids=lambda c: "-".join(f"{k}{v}" for k, v in c.items()))
@pytest.mark.parametrize("total_tiles,nchunks,units", [(7, 1, 3), (9, 4, 4), (20, 3, 6), (5, 8, 3)])
def test_pairs_no_deadlock(cfg, total_tiles, nchunks, units):
    for unit in range(min(units, 4)):  # pairs run whole tiles only (no split mode)
        run_pair([(t, 0, nchunks) for t in range(unit, total_tiles, units)], nchunks=nchunks,
                 **cfg)
