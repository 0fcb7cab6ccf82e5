"""CPU check of the tensor-core GEMM's work schedule (restating csrc/dispatch.cu build_items and
csrc/gemm_tc.cu gemm_item): every (segment, row block, token tile) is one item, the snake
dealing gives every item to exactly one SM pair for any pair count, and each pair's items come
in increasing list order (so with expert parallelism the local source's rows still come
first)."""
import itertools

import numpy as np
import pytest


def build_items(segs, n_rb, tn=256):
    """Segment-major, then row block, then token tile."""
    items = []
    for i, n in enumerate(segs):
        nt = (n + tn - 1) // tn if n > 0 else 0
        for rb in range(n_rb):
            for tt in range(nt):
                items.append((i, rb, tt * tn, min(tn, n - tt * tn)))
    return items


def gemm_item(j, cid, ncl):
    return j * ncl + ((ncl - 1 - cid) if (j & 1) else cid)


def deal(n_items, ncl):
    owner, seq = {}, {}
    for cid in range(ncl):
        seq[cid] = []
        for j in itertools.count():
            w = gemm_item(j, cid, ncl)
            if w >= n_items:
                break
            assert w not in owner
            owner[w] = cid
            seq[cid].append(w)
    assert sorted(owner) == list(range(n_items))
    return owner, seq


@pytest.mark.parametrize("seed", range(6))
def test_items_cover_every_tile_once_and_each_pair_walks_forward(seed):
    rng = np.random.default_rng(seed)
    T, E, K = int(rng.choice([65, 300, 1000, 4096, 8192])), 64, 8
    counts = rng.multinomial(T * K, rng.dirichlet(np.full(E, rng.uniform(0.5, 3.0))))
    segs = [T] + [int(c) for c in counts]
    for n_rb, tn in ((24, 256), (16, 256), (24, 192)):
        items = build_items(segs, n_rb, tn)
        cover = set()
        for i, rb, r0, n in items:
            assert 0 < n <= tn
            for r in range(r0, r0 + n):
                assert (i, rb, r) not in cover
                cover.add((i, rb, r))
        assert len(cover) == n_rb * sum(segs)
        for ncl in (1, 73, 74):
            _, seq = deal(len(items), ncl)
            for ws in seq.values():
                assert ws == sorted(ws)

