"""CPU check of the tensor-core GEMM's work schedule on one GPU (restating
csrc/dispatch.cu build_items for the size-ordered list and csrc/gemm_tc.cu gemm_item for the
snake dealing): every (segment, row block, token tile) is one item, every item goes to exactly
one SM pair, and on routings with the benchmark's skew the busiest pair's work stays within a
few percent of the mean (it is 7-18 % above with plain striding of the segment-major list)."""
import itertools

import numpy as np
import pytest


def build_items_sized(segs, n_rb, tn=256):
    """segs: rows per segment.  Full tiles segment-major (then row block, tile); then partial
    tiles, segments by decreasing rows (ties: lower index), row block inside."""
    items = []
    for i, n in enumerate(segs):
        for rb in range(n_rb):
            for tt in range(n // tn):
                items.append((i, rb, tt * tn, tn))
    part = sorted((i for i, n in enumerate(segs) if n % tn), key=lambda i: (-(segs[i] % tn), i))
    for i in part:
        for rb in range(n_rb):
            items.append((i, rb, segs[i] // tn * tn, segs[i] % tn))
    return items


def gemm_item(j, cid, ncl):
    return j * ncl + ((ncl - 1 - cid) if (j & 1) else cid)


def deal(n_items, ncl):
    owner = {}
    for cid in range(ncl):
        for j in itertools.count():
            w = gemm_item(j, cid, ncl)
            if w >= n_items:
                break
            assert w not in owner
            owner[w] = cid
    assert sorted(owner) == list(range(n_items))
    return owner


@pytest.mark.parametrize("seed", range(6))
def test_items_cover_every_tile_once_and_pairs_stay_balanced(seed):
    rng = np.random.default_rng(seed)
    T, E, K = int(rng.choice([65, 300, 1000, 4096, 8192])), 64, 8
    counts = rng.multinomial(T * K, rng.dirichlet(np.full(E, rng.uniform(0.5, 3.0))))
    segs = [T] + [int(c) for c in counts]
    for n_rb in (24, 16):
        items = build_items_sized(segs, n_rb)
        cover = {}
        for i, rb, r0, n in items:
            assert 0 < n <= 256
            for r in range(r0, r0 + n):
                assert (i, rb, r) not in cover
                cover[(i, rb, r)] = 1
        assert len(cover) == n_rb * sum(segs)
        for ncl in (1, 73, 74):
            owner = deal(len(items), ncl)
            if ncl == 74 and T >= 4096:
                load = np.zeros(ncl)
                for w, cid in owner.items():
                    load[cid] += max(items[w][3], 64)  # MMA work, with a per-item floor
                assert load.max() / load.mean() < 1.05, load.max() / load.mean()
