"""CPU checks of the GEMM's stream-K work schedule (gemm.cuh ``Schedule`` and
rpfq_b200.cu ``sk_tail``, restated here line for line): over many tile /
unit / k-block counts every (tile, k-block) is computed exactly once, a tile
is cut at most once into a head (k-blocks from 0) and a tail (the rest); a
unit's head is its first item of all (before its data-parallel tiles) and its
tail its last, and the tail's head is the previous unit's. The kernel loads a tail's head while the item
before the tail runs, or right after flagging its own head when that is the
item before — so a unit's head never waits, and no wait chains through
units."""

import pytest


def sk_tail(tiles: int, units: int) -> int:
    if units <= 0 or tiles <= units or tiles % units == 0:
        return 0
    if (tiles % units) / units > 0.85:
        return 0
    return tiles - (tiles // units - 1) * units


def schedule(unit: int, units: int, num_tiles: int, num_k: int, sk_tiles: int):
    dp_tiles = num_tiles - sk_tiles
    total = sk_tiles * num_k
    lo, hi = unit * total // units, (unit + 1) * total // units
    whole, whole_end = -(-lo // num_k) * num_k, hi // num_k * num_k

    def seg(a, b, mode):
        j = a // num_k
        return (dp_tiles + j, a - j * num_k, b - j * num_k, mode)

    items = []
    if lo < hi and whole_end < hi:
        items.append(seg(whole_end, hi, "head"))
    items += [(t, 0, num_k, "whole") for t in range(unit, dp_tiles, units)]
    if lo >= hi:
        return items
    for a in range(whole, whole_end, num_k):
        items.append(seg(a, a + num_k, "whole"))
    if lo % num_k:
        items.append(seg(lo, (lo // num_k + 1) * num_k, "tail"))
    return items


CASES = [(t, u, k) for u in (74, 148, 3, 7) for t in range(1, 5 * u + 3, max(1, u // 9)) for k in (1, 3, 12, 48)]


@pytest.mark.parametrize("tiles,units,num_k", CASES)
def test_schedule_invariants(tiles, units, num_k):
    sk = sk_tail(tiles, units)
    assert sk == 0 or units <= sk < 2 * units  # a share is at least one tile long
    grid = units if sk else min(tiles, units)
    seen = {}
    per_unit = [schedule(u, grid, tiles, num_k, sk) for u in range(grid)]
    for u, items in enumerate(per_unit):
        modes = [m for _, _, _, m in items]
        assert modes.count("head") <= 1 and modes.count("tail") <= 1
        for i, (t, lo, hi, mode) in enumerate(items):
            assert 0 <= t < tiles and 0 <= lo < hi <= num_k
            for kb in range(lo, hi):
                assert (t, kb) not in seen, "k-block computed twice"
                seen[(t, kb)] = u
            n_dp = len(range(u, tiles - sk, grid))
            if mode == "tail":
                assert i == len(items) - 1 and i >= 1, "a tail is the unit's last item, after another"
                assert hi == num_k
                prev = per_unit[u - 1]
                heads = [x for x in prev if x[3] == "head"]
                assert heads == [(t, 0, lo, "head")], "the previous unit holds the head"
            if mode == "head":
                assert i == 0, "a head is the unit's first item"
                assert per_unit[u + 1][-1] == (t, hi, num_k, "tail")
    assert len(seen) == tiles * num_k


def sk_chosen(tiles: int, units: int, num_k: int) -> bool:
    """plan_gemm's cost rule: the tail only when the idle part of the last wave
    is at least 24 k-blocks long."""
    if sk_tail(tiles, units) == 0:
        return False
    return (-(-tiles // units) - tiles / units) * num_k >= 24.0


def test_cost_rule_examples():
    # ViT-B at 32 images per GPU: only fc2 (K = 3072) takes the tail
    assert sk_chosen(75, 74, 48) and not sk_chosen(75, 74, 12)
    assert not sk_chosen(225, 74, 12) and not sk_chosen(300, 74, 12)
    # ViT-L at 256 images per GPU: fc2 (788 tiles, 10.65 waves, K = 4096) keeps whole tiles
    assert not sk_chosen(788, 74, 64)


def test_tail_examples():
    # ViT-B at 32 images per GPU (m = 6304) on 74 CTA pairs
    assert sk_tail(75, 74) == 75            # proj / fc2: one tile more than a wave
    assert sk_tail(225, 74) == 77           # qkv
    assert sk_tail(300, 74) == 78           # fc1
    # ViT-B at 256 images (m = 50432): every last wave is over 85 % full
    assert sk_tail(591, 74) == 0 and sk_tail(1773, 74) == 0 and sk_tail(2364, 74) == 0
    assert sk_tail(1413, 74) == 81
    assert sk_tail(148, 74) == 0 and sk_tail(50, 74) == 0
