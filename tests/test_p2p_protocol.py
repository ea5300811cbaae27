"""Exhaustive interleaving check of the one-shot all-reduce protocol (``csrc/p2p_allreduce.cu``).

The kernel's steps per call, per rank, are modelled as atomic actions over shared state:

  bump    epoch = ++counter[rank]
  stage   slot[rank][epoch & 1] = (rank, epoch)          (the local partial)
  pub q   flags[q][rank] = epoch                         (for every peer q; release)
  wait    block until flags[rank][q] >= epoch for every peer q   (acquire)
  read r  observe slot[r][epoch & 1]                      (for every rank r, in rank order)

A rank's calls run one after another (stream order: each call's reads finish before the next
call's stage). Every interleaving of the ranks' actions is explored with memoisation; the check is
that every read of call ``e`` sees exactly ``(r, e)`` -- never the previous or the next call's
partial -- and that no reachable state is stuck while some rank still has calls to make. A second
model lets any wait give up (the kernel's time limit) with a sticky abort, and checks that a rank
never publishes or stages after aborting and that no completed read is wrong.
"""

from __future__ import annotations

import pytest


def _actions(rank, world):
    acts = [("bump",), ("stage",)]
    acts += [("pub", q) for q in range(world) if q != rank]
    acts += [("wait",)]
    acts += [("read", r) for r in range(world)]
    return acts


def _explore(world, calls, allow_timeout=False, nslots=2):
    """Return (states visited, terminal states). Raises AssertionError on a protocol violation.
    ``nslots`` is the number of payload slots per region (the kernel has 2; slot = epoch % nslots)."""
    acts = [_actions(r, world) for r in range(world)]
    # state: per rank (call index, action index, epoch, aborted); slots[r][2]; flags[q][r]
    init = (tuple((0, 0, 0, False) for _ in range(world)),
            tuple(tuple(None for _ in range(nslots)) for _ in range(world)),
            tuple(tuple(0 for _ in range(world)) for _ in range(world)))
    seen = {init}
    stack = [init]
    terminals = 0
    while stack:
        ranks, slots, flags = stack.pop()
        moved = False
        for r in range(world):
            call, ai, epoch, aborted = ranks[r]
            if call == calls or aborted:
                continue
            act = acts[r][ai]
            nslot_l, nflags = [list(s) for s in slots], [list(f) for f in flags]
            nepoch, nabort = epoch, aborted
            if act[0] == "bump":
                nepoch = epoch + 1
            elif act[0] == "stage":
                nslot_l[r][epoch % nslots] = (r, epoch)
            elif act[0] == "pub":
                nflags[act[1]][r] = epoch
            elif act[0] == "wait":
                ready = all(flags[r][q] >= epoch for q in range(world) if q != r)
                if not ready:
                    if not allow_timeout:
                        continue
                    nabort = True  # the time limit ran out: give up, output unwritten, sticky
            elif act[0] == "read":
                got = slots[act[1]][epoch % nslots]
                assert got == (act[1], epoch), (
                    f"rank {r} call {epoch} read slot {epoch % nslots} of rank {act[1]} and saw {got}")
            nai, ncall = ai + 1, call
            if nai == len(acts[r]):
                nai, ncall = 0, call + 1
            if nabort:
                nai, ncall = ai, call
            nranks = list(ranks)
            nranks[r] = (ncall, nai, nepoch, nabort)
            state = (tuple(nranks), tuple(tuple(x) for x in nslot_l), tuple(tuple(f) for f in nflags))
            moved = True
            if state not in seen:
                seen.add(state)
                stack.append(state)
        if not moved:
            terminals += 1
            if not allow_timeout:
                assert all(c == calls for c, _, _, _ in ranks), f"stuck: {ranks}"
    return len(seen), terminals


@pytest.mark.parametrize("world,calls", [(2, 1), (2, 2), (2, 4), (3, 3)])
def test_no_slot_is_read_stale_or_overwritten(world, calls):
    states, terminals = _explore(world, calls)
    assert terminals == 1 and states > 1


@pytest.mark.parametrize("world,calls", [(2, 3), (3, 2)])
def test_time_limit_never_corrupts_a_completed_read(world, calls):
    states, terminals = _explore(world, calls, allow_timeout=True)
    assert terminals >= 2 and states > 1


def test_one_slot_would_be_wrong():
    # The check has teeth: with a single payload slot a rank that finished its reads of call e
    # stages call e + 1 over the partial a slower peer has not read yet.
    with pytest.raises(AssertionError, match="saw"):
        _explore(2, 2, nslots=1)


# ---- low-latency variant (``allreduce_ll_kernel``): the epoch travels with the data ----------


def _explore_ll(world, calls, nslots=2):
    """Per call and rank: bump the epoch; push (rank, epoch) into slot epoch % nslots of every
    peer's inbox line for this rank (one action per peer); then for each peer, in rank order, wait
    until the own inbox line from that peer carries the epoch and read it. The check: every read
    sees exactly (peer, epoch) -- the line is never overwritten by the peer's next-but-one call
    before it is read -- and no state is stuck."""
    acts = []
    for r in range(world):
        a = [("bump",)] + [("push", q) for q in range(world) if q != r] + [("pull", q) for q in range(world) if q != r]
        acts.append(a)
    # state: per rank (call, action index, epoch); inbox[dst][src][slot] = (src, epoch) or None
    init = (tuple((0, 0, 0) for _ in range(world)),
            tuple(tuple(tuple(None for _ in range(nslots)) for _ in range(world)) for _ in range(world)))
    seen, stack = {init}, [init]
    while stack:
        ranks, inbox = stack.pop()
        moved = False
        for r in range(world):
            call, ai, epoch = ranks[r]
            if call == calls:
                continue
            act = acts[r][ai]
            box = [[list(sl) for sl in dst] for dst in inbox]
            nepoch = epoch
            if act[0] == "bump":
                nepoch = epoch + 1
            elif act[0] == "push":
                box[act[1]][r][epoch % nslots] = (r, epoch)
            elif act[0] == "pull":
                line = inbox[r][act[1]][epoch % nslots]
                if line is None or line[1] != epoch:
                    assert line is None or line[1] < epoch, f"rank {r} call {epoch} saw a newer line {line}"
                    continue  # still waiting: the epoch is not there yet
            nai, ncall = ai + 1, call
            if nai == len(acts[r]):
                nai, ncall = 0, call + 1
            nr = list(ranks)
            nr[r] = (ncall, nai, nepoch)
            state = (tuple(nr), tuple(tuple(tuple(sl) for sl in dst) for dst in box))
            moved = True
            if state not in seen:
                seen.add(state)
                stack.append(state)
        if not moved:
            assert all(c == calls for c, _, _ in ranks), f"stuck: {ranks}"
    return len(seen)


@pytest.mark.parametrize("world,calls", [(2, 1), (2, 3), (2, 5), (3, 3), (4, 2)])
def test_ll_lines_are_read_before_they_are_overwritten(world, calls):
    assert _explore_ll(world, calls) > 1


def test_ll_one_slot_would_lose_lines():
    # With one slot a fast rank's next call overwrites a line a slow peer has not read yet, and the
    # slow peer then waits for an epoch that is gone.
    with pytest.raises(AssertionError):
        _explore_ll(2, 3, nslots=1)
