"""CPU check of the fused expert-parallel layout (tests/ep_layout.py restates the kernels'
index arithmetic): on simulated ranks with random routings (a rank without tokens, skewed
counts, an expert placement), every received row of every owner lies in exactly one fused
segment of its (source, local expert); the segment's return row plus the row's offset is the
source's expert-sorted position of the pair that landed there (where the owner's result must
go back, and where the source's combine reads it); work items cover every row once and carry
the same return rows."""
import numpy as np
import pytest

from ep_layout import build_items, fused_segments, send_rows, sort_positions

E, K = 64, 8


@pytest.mark.parametrize("N,tokens,place", [(2, [300, 0], False), (4, [257, 64, 1, 900], True),
                                            (8, [513] * 8, False), (8, [0, 3, 70, 129, 256, 300, 5, 1024], True)])
def test_fused_segments_and_items_return_every_row_to_its_source_position(N, tokens, place):
    el = E // N
    rng = np.random.default_rng(N * 7 + len(tokens))
    slot_of = rng.permutation(E) if place else np.arange(E)
    p = rng.dirichlet(np.full(E, 0.4))
    topk = []
    for T in tokens:
        ex = np.stack([rng.choice(E, K, replace=False, p=p) for _ in range(T)]) if T else np.zeros((0, K), np.int64)
        topk.append(slot_of[ex])
    C = np.stack([np.bincount(t.ravel(), minlength=E) for t in topk])
    # where every source stores each pair, and its sorted position (the return row)
    landed = {}  # (owner, row) -> (source, sorted position)
    slot = {}    # (owner, row) -> the pair's placement slot
    for s in range(N):
        owner, row = send_rows(topk[s], C, tokens, s, el)
        _, pos = sort_positions(topk[s], E)
        for t in range(tokens[s]):
            for k in range(K):
                key = (int(owner[t, k]), int(row[t, k]))
                assert key not in landed
                landed[key] = (s, int(pos[t, k]))
                slot[key] = int(topk[s][t, k])
    for d in range(N):
        segs = fused_segments(C, tokens, d, el)
        assert segs[1][3] == d  # the owner's own rows are listed first
        seen = set()
        for g, r0, n, src, ret in segs[1:]:
            for i in range(n):
                got = landed[(d, r0 + i)]
                assert got == (src, ret + i), (d, r0 + i)
                assert slot[(d, r0 + i)] == d * el + g  # the segment's weights are the pair's expert
                seen.add(r0 + i)
        assert seen == {r for (o, r) in landed if o == d}
        items = build_items(segs, n_rb=12)
        cover = {}
        for g, rb, r0, n, src, ret in items:
            for i in range(n):
                cover[(rb, r0 + i)] = cover.get((rb, r0 + i), 0) + 1
                if r0 + i >= tokens[d]:
                    assert landed[(d, r0 + i)] == (src, ret + i)
        total_rows = tokens[d] + len(seen)
        assert len(cover) == 12 * total_rows and set(cover.values()) == {1}
