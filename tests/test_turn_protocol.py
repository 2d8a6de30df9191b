"""CPU: the turn protocol of the turn-taking kernels in flashns_b200/csrc/eval.cu never
deadlocks and leaves no barrier with pending arrivals, for every number of tiles a CTA can
own.  Two groups with a hand-written closing: bwd_pingpong, fwd_pingpong; the ring
`Ring<NG>` of head_pingpong and head_pingpong_staged: four groups (kHeadGroups).

The barrier sequence, per group g of NG (group g takes the CTA's tiles k = g, g + NG, ...,
so it owns n_g = ceil((m - g) / NG) of m):

    group NG - 1 first arrives on "turn 0";
    for each of its tiles: sync on "turn g", MMAs, arrive on "turn (g + 1) % NG";
    closing: one more sync on "turn g" when its predecessor arrived there more often
             than it synced (n_{NG-1} + 1 arrivals for group 0, n_{g-1} for the others).

For two groups this is the kernels' hand-written form: group 0 syncs "turn 0" once more
when n0 == n1, group 1 syncs "turn 1" once more when n0 == n1 + 1.

A barrier generation completes when two groups have arrived (one syncing, one arriving
or syncing).  The model also rejects a group arriving twice in one generation, which on
the hardware would complete the barrier without the other group.
"""

import itertools

import pytest


def count(m, g, ng):
    return (m - 1 - g) // ng + 1 if m > g else 0


def program(g, m, ng):
    ops = [("arrive", 0)] if g == ng - 1 else []
    for _ in range(count(m, g, ng)):
        ops += [("sync", g), ("arrive", (g + 1) % ng)]
    arrivals = count(m, ng - 1, ng) + 1 if g == 0 else count(m, g - 1, ng)
    if arrivals > count(m, g, ng):
        ops.append(("sync", g))
    return ops


def run(m, order, ng, make=None):
    """Execute every group's program, always advancing the first group of `order` that can."""
    make = make or program
    progs = [make(g, m, ng) for g in range(ng)]
    pc, waiting = [0] * ng, [None] * ng
    pending = {b: set() for b in range(ng)}
    generation = dict.fromkeys(range(ng), 0)

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
        assert u not in pending[bar], f"m={m}: group {u} arrives twice in one generation of turn {bar}"
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

    while any(step(u) for u in order):
        pass
    assert pc == [len(p) for p in progs], f"m={m}: deadlock at {pc}"
    assert not any(pending.values()), f"m={m}: pending arrivals {pending}"


@pytest.mark.parametrize("ng", [2, 4])
def test_turn_barriers_balance_for_every_tile_count(ng):
    for order in itertools.permutations(range(ng)):
        for m in range(0, 65):
            run(m, order, ng)


@pytest.mark.parametrize("ng", [2, 4])
def test_groups_take_every_tile_once(ng):
    for m in range(0, 65):
        assert sum(count(m, g, ng) for g in range(ng)) == m


def test_two_group_ring_is_the_hand_written_closing():
    """For NG = 2 the ring's closing syncs are the two-group kernels' explicit conditions."""
    for m in range(0, 65):
        n0, n1 = (m + 1) // 2, m // 2
        assert (program(0, m, 2)[-1:] == [("sync", 0)] and len(program(0, m, 2)) % 2 == 1) == (n0 == n1)
        assert (len(program(1, m, 2)) % 2 == 0) == (n0 == n1 + 1)


@pytest.mark.parametrize("ng", [2, 4])
def test_model_catches_an_unbalanced_closing(ng):
    """The closing sync is what balances a turn whose predecessor owns one tile more."""

    def without_closing(g, m, n):
        ops = program(g, m, n)
        return ops[:-1] if len(ops) % 2 == (0 if g == n - 1 else 1) else ops

    with pytest.raises(AssertionError):
        for m in range(0, 2 * ng + 1):
            run(m, tuple(range(ng)), ng, without_closing)
