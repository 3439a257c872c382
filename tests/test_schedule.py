"""Host-side check of the split-K tcgen05 kernel's work split
(rustyllm_b200/csrc/rq_mm_skinny.cu, `Segs`, `cta_of` and the piece slots),
restated here: CTA b of G owns units [U b / G, U (b+1) / G) of the (128-row
tile, super-block) order; a tile's pieces belong to CTAs cta_of(first unit)
.. cta_of(last unit); a piece is stored at workspace slot tile + cta, and the
host sizes the workspace for tiles + G slots.  Every unit must belong to
exactly one CTA, cta_of must invert the ranges, and no two pieces may share
a slot."""
import itertools


def ranges(units, grid):
    return [(units * b // grid, units * (b + 1) // grid) for b in range(grid)]


def cta_of(units, grid, x):
    # ((x + 1) G + U - 1) / U - 1, integer division as in the kernel
    return ((x + 1) * grid + units - 1) // units - 1


def segments(units, grid, nblk, b):
    u, u1 = ranges(units, grid)[b]
    out = []
    while u < u1:
        t, sb0 = divmod(u, nblk)
        e = min(u1, (t + 1) * nblk)
        out.append((t, sb0, sb0 + (e - u)))
        u = e
    return out


def test_split_covers_every_unit_once_and_slots_are_unique():
    for tiles, nblk, grid in itertools.product([1, 2, 8, 64, 80, 224, 448],
                                               [1, 4, 32, 56, 112], [1, 7, 148]):
        units = tiles * nblk
        grid = min(grid, units)
        owner = {}
        pieces = {}
        for b in range(grid):
            for t, sb0, sb1 in segments(units, grid, nblk, b):
                assert 0 <= sb0 < sb1 <= nblk
                for sb in range(sb0, sb1):
                    x = t * nblk + sb
                    assert x not in owner
                    owner[x] = b
                    assert cta_of(units, grid, x) == b
                pieces.setdefault(t, []).append(b)
        assert len(owner) == units
        slots = set()
        for t, bs in pieces.items():
            first, last = cta_of(units, grid, t * nblk), cta_of(units, grid, t * nblk + nblk - 1)
            assert bs == list(range(first, last + 1))      # pieces in CTA order, none missing
            for b in bs:
                slot = t + b
                assert slot not in slots and slot < tiles + grid
                slots.add(slot)
