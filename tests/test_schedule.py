"""The tensor-core pass's stream-K schedule, restated on the CPU, and the invariants its in-pass merge relies on.

The pass (omniasr-trt_b200/csrc/attention_tc.cu: total_cost, TileIter, the write-out warp) gives every (group, head)
unit a cost of ``unit_cost + 8 * tiles``, lays the units out group-major, head-minor, and gives CTA b the cost range
[b * per, (b + 1) * per), per = max(ceil(total / grid), 8). A unit's segments are numbered by CTA, from the CTA of its
first tile to the CTA of its last; the last of them to count on the unit's counter merges them all, so

* every segment number of a unit must be written by exactly one CTA (else the count never completes, or a partial
  is written twice), and
* a unit has at most ``ceil(keys / 128)`` segments, within the ``ceil(keys / 128) + 1`` partial slots of its row.

These tests enumerate the schedule for random shapes and check both (CPU only; the GPU tests check the outputs).
"""

import math
import random

import pytest

BN, TILE_COST = 128, 8


def schedule(lengths, heads, nq, causal, cap, unit_cost, grid):
    """{(group, head): {cta: tiles}} for the pass's static stream-K split."""
    def need(g):
        n = lengths[g] + (nq - 1 if causal else 0)
        return min(max(n, 0), cap)

    tiles = [(need(g) + BN - 1) // BN for g in range(len(lengths))]
    ucost = [unit_cost + TILE_COST * t if t else 0 for t in tiles]
    total = sum(c * heads for c in ucost)
    per = max(-(-total // grid), TILE_COST)
    owners = {}
    pre = 0
    for g, t in enumerate(tiles):
        for h in range(heads):
            pos0 = pre + h * ucost[g] + unit_cost
            unit = owners.setdefault((g, h), {})
            for i in range(t):
                cta = (pos0 + TILE_COST * i) // per
                assert cta < grid, "a tile past the last CTA"
                unit[cta] = unit.get(cta, 0) + 1
        pre += ucost[g] * heads
    return owners, per


@pytest.mark.parametrize("seed", range(6))
def test_every_segment_of_a_unit_has_exactly_one_writer(seed):
    rng = random.Random(seed)
    for _ in range(300):
        groups = rng.choice([1, 2, 3, 8, 40, 64, 300])
        heads = rng.choice([1, 2, 8, 32])
        nq = rng.choice([1, 2, 3, 5, 8, 9, 16])
        causal = nq > 1 and rng.random() < 0.7
        keys = rng.choice([128, 256, 1024, 2048, 4096, 8192])
        cap = keys
        lengths = [rng.randint(0, keys - (nq - 1 if causal else 0)) for _ in range(groups)]
        unit_cost = 0 if nq <= 1 else rng.choice([8, 10])
        grid = rng.choice([148, 132, 16, 1])
        owners, per = schedule(lengths, heads, nq, causal, cap, unit_cost, grid)
        slots = math.ceil(keys / BN) + 1
        for (g, h), ctas in owners.items():
            if not ctas:
                continue  # a unit without keys: its rows get zeros from the pass, no segment
            first, last = min(ctas), max(ctas)
            # Segment s of the unit is CTA first + s: each CTA in between holds at least one of its tiles (the
            # ranges are at least one tile's cost long), so every segment number is written, and by one CTA only.
            assert sorted(ctas) == list(range(first, last + 1)), (g, h, sorted(ctas), per)
            nseg = last - first + 1
            assert nseg <= slots - 1, (nseg, slots)


def test_units_cut_between_ctas_occur_and_whole_units_too():
    """The config-2 shape cuts some units between CTAs and finishes others inside one: both merge paths run."""
    lengths = [1852, 1843, 1573, 1983, 1713, 778, 207, 1805]
    owners, _ = schedule([n + 1 for n in lengths], 32, 5, True, 4096, 10, 148)
    nsegs = [len(c) for c in owners.values() if c]
    assert max(nsegs) >= 2 and min(nsegs) == 1
