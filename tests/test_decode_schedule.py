"""CPU model of the paged decode kernel's work split and merge protocol.

The kernel (helm_b200/csrc/paged_attention.cu) cuts the flattened tiles of all
(sequence, KV-head) pairs into equal worker ranges, flushes per-worker partial
states, pre-merges the states of warps that end in the same pair inside a CTA,
and lets the last CTA touching a split pair merge the CTA partials.  This test
replays that index arithmetic in Python for many shapes and checks that every
non-empty pair is finalised exactly once from sources covering each of its
tiles exactly once, that partial slots never collide within a call, and that
every counter target equals the number of CTAs that bump it.
"""
import random


def simulate(tiles_per_seq, hkv, grid, ncw):
    B = len(tiles_per_seq)
    cum = [0]
    for t in tiles_per_seq:
        cum.append(cum[-1] + t)
    total = cum[-1] * hkv
    if total == 0:
        return
    workers = grid * ncw
    W = -(-total // workers)

    def pair_of(x):
        b = max(i for i in range(B) if cum[i] * hkv <= x)
        tb = cum[b + 1] - cum[b]
        return b * hkv + (x - cum[b] * hkv) // tb

    def span(p):
        b, h = divmod(p, hkv)
        tb = cum[b + 1] - cum[b]
        st = cum[b] * hkv + h * tb
        en = st + tb
        vf, vl = st // W, (en - 1) // W
        return tb, st, en, vf, vl, min((vl + 1) * W, total) > en

    finals = {}
    warp_slots, cta_slots = {}, {}
    counters = {}
    # --- per-worker processing: mid-range flushes ---
    end_state = {}
    for v in range(workers):
        lo, hi = v * W, min((v + 1) * W, total)
        if lo >= hi:
            continue
        pairs = []
        for x in range(lo, hi):
            p = pair_of(x)
            if not pairs or pairs[-1][0] != p:
                pairs.append([p, set()])
            pairs[-1][1].add(x)
        for i, (p, tiles) in enumerate(pairs):
            tb, st, en, vf, vl, cont = span(p)
            last = i == len(pairs) - 1
            if vf == vl:
                assert p not in finals
                finals[p] = set(tiles)
            elif not last:
                key = v + p
                assert key not in warp_slots, "warp slot collision"
                warp_slots[key] = (p, tiles)
                assert v == vl and cont
            else:
                end_state[v] = (p, tiles)
    # --- per CTA: pre-merge end states, then counters ---
    for c in range(grid):
        v0 = c * ncw
        groups = {}
        for w in range(ncw):
            if v0 + w in end_state:
                p, tiles = end_state[v0 + w]
                groups.setdefault(p, set()).update(tiles)
        for p, tiles in groups.items():
            tb, st, en, vf, vl, cont = span(p)
            cf, cl = vf // ncw, vl // ncw
            if cf == cl:
                src = set(tiles)
                if cont:
                    wp, wt = warp_slots[vl + p]
                    assert wp == p
                    src |= wt
                assert p not in finals
                finals[p] = src
            else:
                key = c + p
                assert key not in cta_slots, "CTA slot collision"
                cta_slots[key] = (p, tiles)
        lo, hi = v0 * W, min((v0 + ncw) * W, total)
        if lo >= hi:
            continue
        for p in range(pair_of(lo), pair_of(hi - 1) + 1):
            tb, st, en, vf, vl, cont = span(p)
            if tb == 0 or vf == vl or vf // ncw == vl // ncw:
                continue
            counters[p] = counters.get(p, 0) + 1
            if counters[p] == vl // ncw - vf // ncw + 1:
                vl_end = vl - 1 if cont else vl
                src = set()
                for cc in range(vf // ncw, vl_end // ncw + 1):
                    cp, ct = cta_slots[cc + p]
                    assert cp == p
                    assert not (src & ct)
                    src |= ct
                if cont:
                    wp, wt = warp_slots[vl + p]
                    assert not (src & wt)
                    src |= wt
                assert p not in finals
                finals[p] = src
    for p in range(B * hkv):
        tb, st, en, *_ = span(p)
        if tb == 0:
            assert p not in finals
        else:
            assert finals.get(p) == set(range(st, en)), f"pair {p} not covered exactly"


def test_config2_shape():
    simulate([2048] * 4, hkv=8, grid=148, ncw=8)


def test_small_and_ragged_shapes():
    simulate([1, 0, 3, 128], hkv=8, grid=148, ncw=8)
    simulate([36], hkv=8, grid=148, ncw=8)
    simulate([0, 0, 5], hkv=2, grid=3, ncw=4)
    simulate([7] * 16, hkv=5, grid=37, ncw=8)


def test_random_shapes():
    rng = random.Random(0)
    for _ in range(300):
        B = rng.randint(1, 12)
        tiles = [rng.choice([0, 1, 2, 5, 16, 63, 64, 200, 1000]) for _ in range(B)]
        simulate(tiles, hkv=rng.choice([1, 2, 5, 8]), grid=rng.choice([1, 2, 7, 37, 148]),
                 ncw=rng.choice([4, 8]))
