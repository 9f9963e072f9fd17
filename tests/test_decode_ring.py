"""The decode kernel's split-partial ring, as a protocol (CPU).

Split partials of paged_decode_kernel live in a ring of slots
(csrc/paged_decode.cu): the schedule orders rows longest first and gives each
(row, split) of a splitting row the next ring "pair" in that order; work
items are claimed in order by resident CTAs; an item may write its partial
to slot pair % ring only once the slot's sequence word equals its pair, and
the row's last merge (all head blocks of all its splits done) advances the
row's slots by one ring length. This event simulation runs that protocol
with random item durations and asserts what the kernel relies on: every
item completes (no wait cycle) and no slot is written while an earlier row
still owns it -- including rings as small as two rows of splits, where
almost every write waits."""

from __future__ import annotations

import heapq
import random

import pytest

MAX_SPLITS = 128


def ring_slots(rows, splits, ring_min=4096):
    """The library's ring size for a launch (csrc/paged_decode.cu ring_slots)."""
    return min(rows * splits, max(2 * splits, ring_min))


def simulate(split_counts, blocks_per_row, workers, seed, ring):
    rnd = random.Random(seed)
    order = sorted(range(len(split_counts)), key=lambda r: -split_counts[r])
    items, part_base, pairs = [], {}, 0
    for r in order:
        count = split_counts[r]
        if count > 1:
            part_base[r] = pairs
            pairs += count
        for split in range(count):
            for hb in range(blocks_per_row):
                items.append((r, split, hb))
    slot_seq = list(range(ring))
    owner = [None] * ring
    finished, row_merges, waiting = {}, {}, {}
    events, claimed, done, waits = [], 0, 0, 0

    def claim(worker, now):
        nonlocal claimed
        if claimed < len(items):
            heapq.heappush(events, (now + rnd.expovariate(1.0), worker, items[claimed]))
            claimed += 1

    for w in range(workers):
        claim(w, 0.0)
    while events:
        now, worker, (r, split, hb) = heapq.heappop(events)
        count = split_counts[r]
        if count > 1:
            pair = part_base[r] + split
            slot = pair % ring
            if slot_seq[slot] != pair:  # the slot's previous row has not merged
                waits += 1
                waiting.setdefault(slot, []).append((worker, (r, split, hb)))
                continue
            assert owner[slot] in (None, (r, split)), "slot written while another row owns it"
            owner[slot] = (r, split)
            key = (r, hb)
            finished[key] = finished.get(key, 0) + 1
            if finished[key] == count:  # the last split of (row, head block) merges
                row_merges[r] = row_merges.get(r, 0) + 1
                if row_merges[r] == blocks_per_row:  # the row's last merge hands slots on
                    for sp in range(count):
                        s = (part_base[r] + sp) % ring
                        slot_seq[s] += ring
                        owner[s] = None
                        for resumed in waiting.pop(s, []):
                            heapq.heappush(events, (now, *resumed))
        done += 1
        claim(worker, now)
    assert done == len(items), "a wait never ended"
    return waits, pairs


@pytest.mark.parametrize("seed", range(12))
def test_library_sized_rings(seed):
    rnd = random.Random(seed)
    rows = rnd.choice([1, 3, 64, 256, 1024])
    counts = [min(MAX_SPLITS, max(1, int(rnd.paretovariate(1.2)))) for _ in range(rows)]
    _, pairs = simulate(counts, rnd.choice([1, 4, 16]), rnd.choice([592, 148, 37]), seed,
                        ring_slots(rows, MAX_SPLITS))
    assert pairs >= 0


@pytest.mark.parametrize("blocks_per_row,workers", [(4, 592), (16, 592), (1, 37)])
def test_smallest_ring_two_rows_of_splits(blocks_per_row, workers):
    counts = [MAX_SPLITS] * 40 + [1] * 100 + [5] * 50
    waits, pairs = simulate(counts, blocks_per_row, workers, 1, 2 * MAX_SPLITS)
    assert pairs > 2 * MAX_SPLITS and waits > 0  # the ring wrapped many times


def test_ring_sizes():
    assert ring_slots(256, 128) == 4096  # the reference's graph width: 4096 not 32768 slots
    assert ring_slots(4, 128) == 512     # small launches: one slot per possible pair
    assert ring_slots(256, 32) == 4096
