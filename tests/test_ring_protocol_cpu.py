"""The decode kernel's shared-memory ring protocol, modelled on the CPU.

``decode_kernel`` (``solort_b200/csrc/decode.cu``) streams a split's tiles through ``nst`` stages
(7, or 6 when a long block-table slice needs the room). Warp pair ``g`` takes tiles ``g, g+2, ...``
and owns stages ``g, g+2, ...`` (``ns_g = (nst + 1 - g) // 2`` of them): its ``j``-th tile uses stage
``g + 2 * (j % ns_g)`` and waits for parity ``(j // ns_g) & 1``; after consuming tile ``it`` the pair
refills that stage with tile ``it + 2 * ns_g``; tiles ``0 .. nst - 1`` are issued up front into
stages ``0 .. nst - 1``. The model runs the two pairs in random interleavings and checks that every
tile is issued once, that each stage's fills are consumed in issue order by one pair with the wait
parity equal to the fill's phase, and the abort-drain parity of each stage's last fill.
"""

from __future__ import annotations

import random

import pytest


def _run(nst: int, ntiles: int, seed: int) -> None:
    fills = {s: [] for s in range(nst)}
    issued = set()

    def issue(t, s):
        assert t not in issued
        issued.add(t)
        fills[s].append(t)

    for i in range(min(ntiles, nst)):
        issue(i, i)
    consumed = {s: 0 for s in range(nst)}
    state = {0: (0, 0), 1: (1, 0)}
    done = {0: False, 1: False}
    rnd = random.Random(seed)
    spins = 0
    while not all(done.values()):
        g = rnd.choice([p for p in (0, 1) if not done[p]])
        it, j = state[g]
        if it >= ntiles:
            done[g] = True
            continue
        ns = (nst + 1 - g) >> 1
        s = g + 2 * (j % ns)
        k = j // ns
        if len(fills[s]) <= k:  # this pair waits; the other must be able to progress
            assert not done[1 - g], f"deadlock nst={nst} ntiles={ntiles}"
            spins += 1
            assert spins < 100000
            continue
        assert fills[s][k] == it and consumed[s] == k
        assert (k & 1) == ((j // ns) & 1)
        consumed[s] += 1
        if it + 2 * ns < ntiles:
            issue(it + 2 * ns, s)
        state[g] = (it + 2, j + 1)
    assert issued == set(range(ntiles))
    for s in range(nst):
        if fills[s]:
            t = fills[s][-1]
            drain_parity = ((t >> 1) // ((nst + 1 - (t & 1)) >> 1)) & 1
            assert drain_parity == (len(fills[s]) - 1) & 1


@pytest.mark.parametrize("nst", [6, 7])
def test_ring_protocol_every_interleaving_sample(nst):
    for ntiles in range(0, 300):
        for seed in range(3):
            _run(nst, ntiles, seed * 1000 + ntiles)
