"""Properties of the grouped-query balanced schedule spec (oracle.gqa_schedule):
every block of every entry is decoded exactly once, the shares are equal to a
unit, and the merge records name exactly the slots the pieces use."""

import numpy as np
import pytest

import oracle


def _check(lens, hkv, parts, block_n=128):
    pieces, merge = oracle.gqa_schedule(lens, hkv, parts, block_n=block_n)
    E = len(lens) * hkv
    covered = {e: [] for e in range(E)}
    slots = {}
    for p, plist in enumerate(pieces):
        for e, t0, t1, final, slot in plist:
            covered[e].append((t0, t1, p, final, slot))
            if not final:
                assert slot not in slots, (slot, e)
                slots[slot] = e
    for e in range(E):
        n = max(int(lens[e // hkv]), 0)
        segs = sorted(covered[e])
        assert segs, e
        if n == 0:
            assert len(segs) == 1 and segs[0][0] == segs[0][1] == 0 and segs[0][3]
        else:
            assert segs[0][0] == 0 and segs[-1][1] == n
            for a, b in zip(segs, segs[1:]):
                assert a[1] == b[0] and a[0] < a[1]
        head, first, count = merge[e]
        if len(segs) == 1:
            assert head == -1 and segs[0][3]
        else:
            assert head == segs[0][4] and [s[4] for s in segs[1:]] == list(range(first, first + count))
    return pieces


@pytest.mark.parametrize("block_n", [128, 64, 192, 32])  # head 256 / small-head / paired head-256 tiles
def test_schedule_covers_every_block_once(block_n):
    rs = np.random.RandomState(3)
    for trial in range(60):
        B = int(rs.randint(1, 40))
        hkv = int(rs.choice([1, 2, 8]))
        lens = rs.randint(0 if trial % 5 == 0 else 1, 3000, size=B)
        pieces = _check(lens, hkv, int(rs.randint(1, 160)), block_n)
        # pieces start and end on block boundaries (or the sequence end)
        for pl in pieces:
            for e, t0, t1, _, _ in pl:
                assert t0 % block_n == 0
                assert t1 % block_n == 0 or t1 == lens[e // hkv]


def test_schedule_shares_are_balanced():
    lens = [4096] * 32
    pieces = _check(lens, 8, 148)
    units = [sum((t1 - t0 + 127) // 128 + (1 if t0 == 0 else 0) for _, t0, t1, _, _ in pl)
             for pl in pieces]
    # every CTA gets T / P units (+-1 for the cut; +1 for a header unit)
    assert max(units) - min(units) <= 2
    assert max(len(pl) for pl in pieces) <= 3


def test_tiny_workloads_use_fewer_parts():
    pieces, merge = oracle.gqa_schedule([5], 1, 148)
    # two units (the entry's leading unit and its one block) over two CTAs:
    # the block, and so the whole piece, sits in CTA 1
    assert [len(pl) for pl in pieces[:3]] == [0, 1, 0] and merge[0][0] == -1
