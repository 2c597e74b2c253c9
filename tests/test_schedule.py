"""The kernel's work plan (schedule.cuh), enumerated through the library on the CPU.

``avo_b200_schedule_units`` runs the same host/device code every role of the kernel
walks, so these checks cover what the GPU will do:

* every KV tile of every (pair, query block) item is computed exactly once;
* a split item is one first piece (tiles from 0) plus continuation pieces on the next
  CTAs, and the first piece names exactly the CTAs holding them;
* per CTA and segment at most one continuation piece (its first unit) and one first
  piece (its last unit), so a merging CTA only waits for work its neighbours did at the
  start of their runs, and slots alternate between segments;
* the runs are balanced; causal launches with many items use per-CTA lists over groups of
  heads (balanced like longest-first waves, with few pairs in flight);
* the flag protocol on the slots (writer waits for 0, sets 1; merger waits for 1,
  resets to 0) ends under random CTA speeds and never hands a merger another item's
  piece.
"""

from __future__ import annotations

import random
from collections import defaultdict

import pytest

WHOLE, FIRST, CONT = 0, 1, 2
SHAPES = [
    # (num_bh, seq, causal)
    (64, 4096, False),      # bench workload, one GPU: whole items in waves
    (8, 8192, False),       # target point, one of 8 GPUs: split tail
    (16, 8192, False),      # target point, one of 4 GPUs
    (2, 16384, False),      # B1 H16 S16384 over 8 GPUs
    (8, 4096, False),       # bench workload over 8 GPUs
    (32, 8192, True),       # B2 H16 S8192 causal: whole items, longest first
    (16, 32768, True),      # B1 H16 S32768 causal
    (3, 1000, True),        # ragged causal, few items
    (40, 1000, True),       # ragged causal with a clipped last block
    (300, 384, True),
    (4, 512, False),
    (1, 128, True),
]


def item_tiles(q0, seq, causal):
    n_kv = (seq + 127) // 128
    if not causal:
        return n_kv
    last = min(q0 + 256, seq) - 1
    return min(n_kv, last // 128 + 1)


@pytest.mark.parametrize("num_bh,seq,causal", SHAPES)
@pytest.mark.parametrize("split", [False, True])
def test_plan_covers_every_tile_once(b200, num_bh, seq, causal, split):
    mode, grid, _, _, units = b200.schedule_units(num_bh, seq, seq, causal, split=split, max_units=4096)
    if not split:
        assert mode == 0
    covered = defaultdict(list)
    for cta, seq_units in enumerate(units):
        for bh, q0, t0, t1, kind, seg, lo, hi in seq_units:
            assert 0 <= t0 <= t1 <= item_tiles(q0, seq, causal)
            covered[(bh, q0)].append((t0, t1, kind, cta, seg, lo, hi))
    nq = (seq + 255) // 256
    assert set(covered) == {(bh, qb * 256) for bh in range(num_bh) for qb in range(nq)}
    for (bh, q0), pieces in covered.items():
        n = item_tiles(q0, seq, causal)
        pieces.sort()
        assert pieces[0][0] == 0 and pieces[-1][1] == n
        for a, b in zip(pieces, pieces[1:]):
            assert a[1] == b[0]  # contiguous, no overlap
        if len(pieces) == 1:
            assert pieces[0][2] == WHOLE
            continue
        first = pieces[0]
        assert first[2] == FIRST and all(p[2] == CONT for p in pieces[1:])
        assert [p[3] for p in pieces[1:]] == list(range(first[5], first[6] + 1))
        assert first[5] == first[3] + 1
        assert all(p[4] == first[4] for p in pieces)


@pytest.mark.parametrize("num_bh,seq,causal", SHAPES)
def test_split_pieces_sit_at_the_ends_of_runs(b200, num_bh, seq, causal):
    _, _, _, _, units = b200.schedule_units(num_bh, seq, seq, causal, split=True, max_units=4096)
    for seq_units in units:
        by_seg = defaultdict(list)
        for u in seq_units:
            if u[5] >= 0:
                by_seg[u[5]].append(u[4])
        for kinds in by_seg.values():
            assert kinds.count(CONT) <= 1 and kinds.count(FIRST) <= 1
            if CONT in kinds:
                assert kinds[0] == CONT
            if FIRST in kinds:
                assert kinds[-1] == FIRST


@pytest.mark.parametrize("num_bh,seq,causal,bound", [
    (8, 8192, False, 1.01), (16, 8192, False, 1.02), (2, 16384, False, 1.01), (8, 4096, False, 1.05)])
def test_split_plans_balance_the_ctas(b200, num_bh, seq, causal, bound):
    mode, grid, _, _, units = b200.schedule_units(num_bh, seq, seq, causal, split=True, max_units=4096)
    assert mode == 1 and 140 <= grid <= 148
    tiles = [sum(u[3] - u[2] for u in us) for us in units]
    total = sum(tiles)
    assert max(tiles) <= bound * total / 148 + 2, (max(tiles), total / 148)


@pytest.mark.parametrize("num_bh,seq,group,pairs_bound", [(32, 8192, 8, 16), (16, 32768, 2, 8), (16, 16384, 4, 8)])
def test_causal_table_plan_is_balanced_and_l2_local(b200, num_bh, seq, group, pairs_bound):
    # causal, many items, with a workspace: whole items in host-built per-CTA lists over
    # groups of pairs (mode 2), as balanced as longest-first waves, with far fewer pairs in
    # flight; without a workspace the launch keeps the waves (mode 0)
    assert b200.schedule_units(num_bh, seq, seq, True, split=False)[0] == 0
    mode, grid, g, _, units = b200.schedule_units(num_bh, seq, seq, True, split=True, max_units=4096)
    assert mode == 2 and grid == 148 and g == group
    tiles = [sum(u[3] - u[2] for u in us) for us in units]
    assert max(tiles) <= 1.02 * sum(tiles) / grid
    depth = max(len(us) for us in units)
    in_flight = max(len({us[k][0] for us in units if len(us) > k}) for k in range(depth))
    assert in_flight <= pairs_bound < num_bh
    # every CTA's list runs through the groups in order
    for us in units:
        groups = [u[0] // g for u in us]
        assert groups == sorted(groups)


def test_causal_few_items_keep_the_wave_order(b200):
    # fewer than two items per SM: longest query blocks first over all heads, in waves
    mode, grid, _, _, units = b200.schedule_units(3, 1000, 1000, True)
    assert mode == 0
    assert [u[:2] for u in units[0]] == [[0, 768]]


def simulate_flags(units, seed):
    """Random-speed run of the slot protocol; returns the merges in order."""
    rnd = random.Random(seed)
    grid = len(units)
    flag = defaultdict(int)
    content = {}
    pos = [0] * grid
    merged = []
    steps = 0
    while any(pos[c] < len(units[c]) for c in range(grid)):
        steps += 1
        assert steps < 10**6, "no progress: the slot protocol deadlocked"
        c = rnd.randrange(grid)
        if pos[c] >= len(units[c]):
            continue
        bh, q0, t0, t1, kind, seg, lo, hi = units[c][pos[c]]
        key = (bh, q0)
        if kind == CONT:
            slot = (c, seg & 1)
            if flag[slot] != 0:
                continue  # slot still holds an unmerged piece
            content[slot] = (key, t0, t1)
            flag[slot] = 1
        elif kind == FIRST:
            slots = [(cc, seg & 1) for cc in range(lo, hi + 1)]
            if any(flag[s] != 1 for s in slots):
                continue
            got = [content[s] for s in slots]
            assert all(g[0] == key for g in got), (key, got)
            assert got[0][1] == t1 and all(a[2] == b[1] for a, b in zip(got, got[1:]))
            for s in slots:
                flag[s] = 0
            merged.append(key)
        pos[c] += 1
    assert all(v == 0 for v in flag.values())
    return merged


@pytest.mark.parametrize("num_bh,seq,causal", [(8, 8192, False), (2, 16384, False), (8, 4096, False),
                                               (16, 8192, False), (1, 1000, False)])
def test_slot_protocol_ends_and_matches_pieces(b200, num_bh, seq, causal):
    _, _, _, _, units = b200.schedule_units(num_bh, seq, seq, causal, split=True, max_units=4096)
    firsts = sum(1 for us in units for u in us if u[4] == FIRST)
    for seed in range(3):
        assert len(simulate_flags(units, seed)) == firsts
