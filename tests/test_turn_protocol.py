"""CPU: the turn protocol of the two-group kernels (bwd_pingpong, fwd_pingpong,
head_pingpong in flashns_b200/csrc/eval.cu) never deadlocks and leaves no barrier with
pending arrivals, for every number of half tiles a CTA can own.

The kernels' barrier sequence, per group (group 0 takes the CTA's even half tiles, group
1 the odd ones, n0 = ceil(m / 2) and n1 = floor(m / 2)):

    group 1 first arrives on "turn 0";
    for each of its half tiles: sync on its own turn barrier, MMAs, arrive on the other's;
    closing: group 0 syncs "turn 0" once more when n0 == n1,
             group 1 syncs "turn 1" once more when n0 == n1 + 1.

A barrier generation completes when both groups have arrived (one syncing, one arriving
or syncing).  The model also rejects a group arriving twice in one generation, which on
the hardware would complete the barrier without the other group.
"""

import pytest


def program(group, n0, n1):
    ops = [("arrive", "turn0")] if group == 1 else []
    own, other = ("turn0", "turn1") if group == 0 else ("turn1", "turn0")
    for _ in range(n0 if group == 0 else n1):
        ops += [("sync", own), ("arrive", other)]
    if group == 0 and n0 == n1:
        ops.append(("sync", "turn0"))
    if group == 1 and n0 == n1 + 1:
        ops.append(("sync", "turn1"))
    return ops


def run(m, prefer):
    """Execute both programs, always advancing group `prefer` while it can."""
    n0, n1 = (m + 1) // 2, m // 2
    progs = [program(0, n0, n1), program(1, n0, n1)]
    pc, waiting = [0, 0], [None, None]
    pending = {"turn0": set(), "turn1": set()}
    generation = {"turn0": 0, "turn1": 0}

    def step(u):
        if waiting[u] is not None:
            bar, gen = waiting[u]
            if generation[bar] > gen:
                waiting[u] = None
                pc[u] += 1
                return True
            return False
        if pc[u] >= len(progs[u]):
            return False
        op, bar = progs[u][pc[u]]
        assert u not in pending[bar], f"m={m}: group {u} arrives twice in one generation of {bar}"
        pending[bar].add(u)
        gen = generation[bar]
        if len(pending[bar]) == 2:
            pending[bar] = set()
            generation[bar] += 1
        if op == "arrive":
            pc[u] += 1
        else:
            waiting[u] = (bar, gen)
        return True

    order = (prefer, 1 - prefer)
    while step(order[0]) or step(order[1]):
        pass
    assert pc == [len(progs[0]), len(progs[1])], f"m={m}: deadlock at {pc}"
    assert not pending["turn0"] and not pending["turn1"], f"m={m}: pending arrivals {pending}"


@pytest.mark.parametrize("prefer", [0, 1])
def test_turn_barriers_balance_for_every_tile_count(prefer):
    for m in range(0, 65):
        run(m, prefer)


def test_model_catches_an_unbalanced_closing():
    """The closing sync is what balances "turn 0" when the groups own as many tiles."""
    global program
    original = program

    def without_closing(group, n0, n1):
        ops = original(group, n0, n1)
        return ops[:-1] if group == 0 and n0 == n1 else ops

    program = without_closing
    try:
        with pytest.raises(AssertionError):
            run(4, 0)
    finally:
        program = original
