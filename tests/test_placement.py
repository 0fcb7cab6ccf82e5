"""CPU tests of the expert-placement helper (hymoe_balance_placement, no device needed):
a permutation with exactly E/N experts per rank, equal to a restatement of the greedy rule,
better balanced than the contiguous split on skewed loads, and argument errors as status."""
import ctypes as C
import math

import numpy as np
import pytest

import hymoe


def greedy(load, N):
    """Restatement: heaviest first (ties: lower expert), least-loaded rank with a free slot
    (ties: lower rank), that rank's next slot."""
    E = len(load)
    el = E // N
    order = sorted(range(E), key=lambda e: (-load[e], e))
    tot, used, slot = [0.0] * N, [0] * N, [0] * E
    for e in order:
        r = min((r for r in range(N) if used[r] < el), key=lambda r: (tot[r], r))
        slot[e] = r * el + used[r]
        used[r] += 1
        tot[r] += load[e]
    return slot


def rank_loads(slot, load, N):
    el = len(load) // N
    out = [0.0] * N
    for e, s in enumerate(slot):
        out[s // el] += load[e]
    return out


@pytest.mark.parametrize("N", [1, 2, 4, 8, 64])
@pytest.mark.parametrize("kind", ["zipf", "uniform", "ties", "zeros"])
def test_balance_placement_is_the_greedy_permutation(N, kind):
    E = 64
    rng = np.random.default_rng(N)
    if kind == "zipf":
        load = (np.arange(1, E + 1) ** -1.1)[rng.permutation(E)] * 1e5
    elif kind == "uniform":
        load = rng.integers(0, 1000, E).astype(float)
    elif kind == "ties":
        load = np.repeat([5.0, 3.0, 1.0, 0.0], E // 4)
    else:
        load = np.zeros(E)
    slot = hymoe.balance_placement(list(load), N)
    assert sorted(slot) == list(range(E))
    assert slot == greedy(list(load), N)
    el = E // N
    assert all(sum(1 for s in slot if s // el == r) == el for r in range(N))
    if kind == "zeros":  # every tie resolved in order: the identity
        assert slot == list(range(E))


def test_balanced_placement_beats_the_contiguous_split_on_skewed_loads():
    E, N = 64, 8
    rng = np.random.default_rng(3)
    load = list((np.arange(1, E + 1) ** -1.1)[rng.permutation(E)] * 1e5)
    contiguous = max(rank_loads(list(range(E)), load, N))
    balanced = rank_loads(hymoe.balance_placement(load, N), load, N)
    assert max(balanced) < contiguous
    assert max(balanced) <= sum(load) / N + max(load)  # the greedy bound


def test_balance_placement_rejects_bad_arguments():
    L = hymoe.lib()
    out = (C.c_int32 * 64)()
    ok = (C.c_double * 64)(*([1.0] * 64))
    assert L.hymoe_balance_placement(64, 3, ok, out) == 1        # 64 % 3 != 0
    assert L.hymoe_balance_placement(64, 0, ok, out) == 1
    assert L.hymoe_balance_placement(0, 1, ok, out) == 1
    assert L.hymoe_balance_placement(64, 8, None, out) == 1
    assert L.hymoe_balance_placement(64, 8, ok, None) == 1
    for bad in (-1.0, math.nan):
        v = [1.0] * 64
        v[17] = bad
        assert L.hymoe_balance_placement(64, 8, (C.c_double * 64)(*v), out) == 1
    with pytest.raises(hymoe.HymoeError):
        hymoe.balance_placement([1.0] * 60, 8)
    assert L.hymoe_set_placement(None, 0, None) == 1
