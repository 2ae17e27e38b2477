"""The work split of the small-batch Q4_K GEMV (xwfes_b200/csrc/gemv_imma.cu),
restated on the host: CTA i of a k-group owns units [bnd(i), bnd(i+1)) with
bnd(i) = i * U // G; unit_owner(q) finds that CTA; a row block's parts lie
with the consecutive CTAs owner(first unit) .. owner(last unit); and the
fix-up slot index rb + owner is unique, so no two partials share a slot."""
import itertools

import pytest


def bnd(i, U, G):
    return i * U // G


def owner(q, U, G):
    return ((q + 1) * G + U - 1) // U - 1


@pytest.mark.parametrize("R,nsbg,G", [(8, 16, 128), (112, 16, 148), (32, 56, 148), (1, 1, 1),
                                      (3, 7, 5), (224, 16, 148), (64, 14, 37), (2, 3, 6)])
def test_unit_ranges_and_owners(R, nsbg, G):
    U = R * nsbg
    G = min(G, U)
    ranges = [(bnd(i, U, G), bnd(i + 1, U, G)) for i in range(G)]
    assert ranges[0][0] == 0 and ranges[-1][1] == U
    assert all(a < b for a, b in ranges)  # no CTA without a unit when G <= U
    assert all(ranges[i][1] == ranges[i + 1][0] for i in range(G - 1))
    for q in range(U):
        i = owner(q, U, G)
        assert ranges[i][0] <= q < ranges[i][1]
    slots = set()
    for rb in range(R):
        first, last = rb * nsbg, rb * nsbg + nsbg - 1
        owners = list(range(owner(first, U, G), owner(last, U, G) + 1))
        # every CTA in between holds at least one part of the row block
        for i in owners:
            a, b = ranges[i]
            assert max(a, first) < min(b, last + 1)
        for i in owners:
            assert rb + i < R + G
            assert (rb + i) not in slots
            slots.add(rb + i)


def test_slot_index_bound_exhaustive():
    for R, nsbg, G in itertools.product(range(1, 9), range(1, 6), range(1, 12)):
        test_unit_ranges_and_owners(R, nsbg, G)
