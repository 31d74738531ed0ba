"""The cut schedule's last round, on CPU: slice arithmetic and the merge protocol.

In the cut schedule (csrc/attn_shared.cuh: slice_lo, slice_of, SegIter,
segment_epilogue) the key tiles of the last round's units are dealt as equal slices to the
CTAs.  A CTA writes an fp32 partial for each cut unit its slice touches -- slot 0 for the
unit its slice starts in, slot 1 for the unit it ends in -- and the warpgroup that completes a
unit tile's arrival counter merges every slice of it.  These tests mirror that code by hand
(a change to one must be made in the other) and check:
  * over many shapes, that the slices cover every tile exactly once, that a CTA writes at
    most one partial per slot, that slice_of agrees with the slices, and that the merging
    side finds each contributor's partial in the slot that contributor wrote;
  * over random interleavings of the contributors, that the counter protocol -- a read of
    the counter before storing (a warpgroup that finds every other slice counted is last and
    skips its own partial), else store, then atomic add -- elects exactly one merger, that
    the merger sees every other contributor's partial, and that it leaves the counter at zero
    for the next call."""
import random

import pytest


def slice_lo(c, tiles, ctas):
    return c * tiles // ctas


def slice_of(t, tiles, ctas):
    return ((t + 1) * ctas + tiles - 1) // tiles - 1


def tail_segments(c, tiles, ctas, n):
    """SegIter's walk of CTA c through the last round: (unit, k0, k1, full, slot)."""
    lo, hi = slice_lo(c, tiles, ctas), slice_lo(c + 1, tiles, ctas)
    t, out = lo, []
    while t < hi:
        ut = t // n
        ubeg = ut * n
        uend = ubeg + n
        k0, k1 = t - ubeg, min(uend, hi) - ubeg
        out.append((ut, k0, k1, k0 == 0 and k1 == n, 0 if t == lo else 1))
        t = min(uend, hi)
    return out


def part_slot(c, ut, tiles, ctas, n):
    """The merging side's choice of CTA c's partial slot for unit ut (part_of)."""
    t0, lo_c = ut * n, slice_lo(c, tiles, ctas)
    return 0 if max(t0, lo_c) == lo_c else 1


SHAPES = [(tail, n, sm, min_slice) for tail in (1, 2, 5, 24, 28, 48, 68, 108, 136, 147)
          for n in (1, 3, 4, 8, 16, 20, 32, 48, 64, 128) for sm in (148, 132)
          for min_slice in (4, 8)]


@pytest.mark.parametrize("tail,n,sm,min_slice", SHAPES)
def test_slices_cover_the_last_round_and_partials_match(tail, n, sm, min_slice):
    tiles = tail * n
    ctas = max(1, min(sm, tiles // min_slice))  # the planner's rule
    covered = [0] * tiles
    written = {}  # (unit) -> {cta: slot}
    for c in range(ctas):
        segs = tail_segments(c, tiles, ctas, n)
        assert segs, "every CTA of the last round gets a slice"
        slots = [s for (_, _, _, full, s) in segs if not full]
        assert slots.count(0) <= 1 and slots.count(1) <= 1
        for ut, k0, k1, full, slot in segs:
            for k in range(k0, k1):
                covered[ut * n + k] += 1
            if not full:
                written.setdefault(ut, {})[c] = slot
    assert covered == [1] * tiles
    for t in range(tiles):
        c = slice_of(t, tiles, ctas)
        assert slice_lo(c, tiles, ctas) <= t < slice_lo(c + 1, tiles, ctas)
    for ut, by_cta in written.items():
        c0, c1 = slice_of(ut * n, tiles, ctas), slice_of(ut * n + n - 1, tiles, ctas)
        assert sorted(by_cta) == list(range(c0, c1 + 1))  # contributors: exactly c0..c1
        for c, slot in by_cta.items():
            assert part_slot(c, ut, tiles, ctas, n) == slot


def merge_round(k, rnd):
    """k contributors of one unit tile, interleaved at random; returns (mergers, counter)."""
    cnt = [0]
    stored = [False] * k
    mergers = []

    def contributor(me):
        last = cnt[0] == k - 1          # read before storing
        yield
        if not last:
            stored[me] = True           # partial store (then a fence)
            yield
            prev = cnt[0]               # atomic add
            cnt[0] += 1
            last = prev == k - 1
            yield
        if last:
            others = [o for o in range(k) if o != me]
            assert all(stored[o] for o in others), "merge before every partial landed"
            mergers.append(me)
            yield
            cnt[0] = 0                  # leave the counter zero for the next call

    gens = [contributor(c) for c in range(k)]
    live = list(range(k))
    while live:
        c = rnd.choice(live)
        try:
            next(gens[c])
        except StopIteration:
            live.remove(c)
    return mergers, cnt[0]


@pytest.mark.parametrize("k", [2, 3, 4, 6, 33])
def test_counter_protocol_elects_one_merger(k):
    rnd = random.Random(k)
    for _ in range(400):
        mergers, final = merge_round(k, rnd)
        assert len(mergers) == 1 and final == 0
