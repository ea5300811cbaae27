"""Exhaustive interleaving check of the column-strip GEMV's shared-memory ring (``csrc/gemv_strip.cu``).

One producer fills ring slot ``li % R`` with stage ``li`` (after waiting for the slot's previous
fill to be consumed); C consumer warps each own the slots ``j`` with ``j % C == warp`` and consume
every fill of those slots in order (the kernel's slot walk). Barriers are modelled as the hardware
sees them: an mbarrier only knows the parity of its current phase, and ``try_wait.parity(P)``
succeeds as soon as that parity differs from P -- so a waiter that is two phases early passes.

The check explores every interleaving (memoised) and asserts that each consumer reads exactly the
stage it expects (never an older or newer fill), the producer never overwrites an unconsumed
fill, every stage is consumed once, and no state is stuck. The same harness run on the earlier
assignment (warp w takes stages w, w + C, ... regardless of slot) finds the phase aliasing that
faulted on the GPU when there were more consumer warps than ring slots (C = 4, R = 3).
"""

from __future__ import annotations

import pytest


def _consumer_walk(warp, C, R, nloc):
    """The stages warp ``warp`` consumes, in order, following the kernel's slot walk."""
    out = []
    li, rnd = (warp if warp < R else nloc), 0
    while li < nloc:
        out.append(li)
        li += C
        if li - rnd >= R:
            rnd += R
            li = rnd + warp
    return out


def _old_assignment(warp, C, R, nloc):
    return list(range(warp, nloc, C))


def _explore(R, C, nloc, assign):
    plans = [tuple(assign(w, C, R, nloc)) for w in range(C)]
    flat = sorted(s for p in plans for s in p)
    assert flat == list(range(nloc)), f"stages not partitioned: {plans}"
    # state: producer index, consumer positions, completed phases of each slot's full and empty
    # barriers, and the stage each slot holds
    init = (0, tuple(0 for _ in range(C)), (0,) * R, (0,) * R, (None,) * R)
    seen = {init}
    stack = [init]
    while stack:
        st = stack.pop()
        prod, pos, full, empty, content = st
        succ = []
        # producer
        if prod < nloc:
            slot, fill = prod % R, prod // R
            ok = True
            if fill > 0:  # wait on empty[slot] for the consumption of fill - 1
                ok = (empty[slot] & 1) != ((fill - 1) & 1)
            if ok:
                assert empty[slot] >= fill, f"producer overwrote stage {content[slot]} unconsumed (stage {prod})"
                f2, c2 = list(full), list(content)
                f2[slot] += 1
                c2[slot] = prod
                succ.append((prod + 1, pos, tuple(f2), empty, tuple(c2)))
        # consumers
        for w in range(C):
            if pos[w] == len(plans[w]):
                continue
            li = plans[w][pos[w]]
            slot, fill = li % R, li // R
            if (full[slot] & 1) != (fill & 1):  # try_wait.parity(fill & 1) passes
                assert content[slot] == li, (
                    f"warp {w} waited for stage {li} in slot {slot} and read {content[slot]}")
                e2, p2 = list(empty), list(pos)
                e2[slot] += 1
                p2[w] += 1
                succ.append((prod, tuple(p2), full, tuple(e2), content))
        if not succ:
            assert prod == nloc and all(pos[w] == len(plans[w]) for w in range(C)), f"stuck: {st}"
        for s in succ:
            if s not in seen:
                seen.add(s)
                stack.append(s)
    return len(seen)


CASES = [(3, 4, 7), (4, 4, 9), (2, 8, 5), (5, 2, 11), (3, 3, 8), (1, 4, 3), (6, 4, 13), (4, 16, 10),
         (3, 2, 7), (16, 16, 18)]


@pytest.mark.parametrize("R,C,nloc", CASES)
def test_slot_walk_never_aliases(R, C, nloc):
    assert _explore(R, C, nloc, _consumer_walk) > 1


@pytest.mark.parametrize("R,C,nloc", [(3, 4, 7), (2, 3, 6), (3, 5, 9)])
def test_old_assignment_aliases(R, C, nloc):
    # More warps than slots: warp R's first stage is the second fill of slot 0, and its parity
    # wait passes before the first fill has even landed.
    with pytest.raises(AssertionError, match="read|overwrote"):
        _explore(R, C, nloc, _old_assignment)


@pytest.mark.parametrize("R,C", [(4, 4), (5, 3), (8, 4), (16, 8)])
def test_old_assignment_was_safe_with_no_more_warps_than_slots(R, C):
    assert _explore(R, C, 2 * R + 1, _old_assignment) > 1
