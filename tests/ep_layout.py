"""Specification of the expert-parallel row layout (test helper).

The CUDA path (csrc/dispatch.cu plan/ep_segments, csrc/ep_p2p.cu ep_scatter) implements this
layout; the gloo tests check its properties on CPU ranks.  Rank r owns experts
[r*el, (r+1)*el), el = E/N.

- Each rank sorts its T*K (token, rank-k) pairs by global expert, stably by token:
  position pos(t, k) = goff[e] + #{earlier tokens choosing e}.
- Owner d's receive matrix: rows [0, T_d) its own tokens (shared expert), then the rows of
  source 0, 1, ..., each in (local expert, source token) order.
- Source s stores its pair (t, k) with expert e (owner d = e // el) at
      row = base(d, s) + pos(t, k) - goff[d*el],   base(d, s) = T_d + sum_{s'<s} sum_le C[s'][d*el+le]
  where C[s'] are the per-expert pair counts of source s'.
"""
import numpy as np


def sort_positions(topk_idx: np.ndarray, E: int):
    """(goff[E+1], pos[T, K]) of the stable counting sort of the pairs by expert."""
    T, K = topk_idx.shape
    counts = np.bincount(topk_idx.ravel(), minlength=E)
    goff = np.concatenate([[0], np.cumsum(counts)])
    pos = np.empty((T, K), np.int64)
    seen = np.zeros(E, np.int64)
    for t in range(T):
        for k in range(K):
            e = topk_idx[t, k]
            pos[t, k] = goff[e] + seen[e]
            seen[e] += 1
    return goff, pos


def send_rows(topk_idx: np.ndarray, C: np.ndarray, Ts, me: int, el: int):
    """(owner[T, K], row[T, K]): where source `me` stores each of its pairs."""
    E = C.shape[1]
    goff, pos = sort_positions(topk_idx, E)
    owner = topk_idx // el
    N = C.shape[0]
    base = np.array([Ts[d] + sum(int(C[s, d * el:(d + 1) * el].sum()) for s in range(me)) for d in range(N)])
    row = base[owner] + pos - goff[owner * el]
    return owner, row


def recv_segments(C: np.ndarray, Ts, d: int, el: int):
    """Owner d's segments: (group, first row, rows, source); the shared expert first."""
    segs = [(el, 0, Ts[d], -1)]
    row = Ts[d]
    for s in range(C.shape[0]):
        for le in range(el):
            cnt = int(C[s, d * el + le])
            segs.append((le, row, cnt, s))
            row += cnt
    return segs


def rows_cap(max_tokens: int, N: int, K: int, el: int) -> int:
    """Receive capacity the library allocates: T + N*T*min(K, el) rows (N = 1: T + T*K)."""
    return max_tokens + (max_tokens * K if N == 1 else N * max_tokens * min(K, el))


def fused_segments(C: np.ndarray, Ts, d: int, el: int):
    """Owner d's segments as the fused expert-parallel path lists them (csrc/dispatch.cu
    ep_segments_fused_kernel): shared first, then sources d, d-1, d-2, ... (rows stay
    source-major); each (group, first row, rows, source, return row), where the return row is
    the source's expert-sorted position of the segment's first row."""
    N = C.shape[0]
    segs = [(el, 0, Ts[d], d, 0)]
    for j in range(N):
        s = (d - j) % N
        row = Ts[d] + sum(int(C[s2, d * el:(d + 1) * el].sum()) for s2 in range(s))
        ret = int(C[s, :d * el].sum())
        for le in range(el):
            cnt = int(C[s, d * el + le])
            segs.append((le, row, cnt, s, ret))
            row += cnt
            ret += cnt
    return segs


def build_items(segs, n_rb: int, tile_n: int = 256):
    """Work items of the tensor-core path (csrc/dispatch.cu build_items): segment-major, then
    row block, then token tile; each (group, row block, first row, rows, source, return row)."""
    items = []
    for g, r0, n, src, ret in segs:
        ntt = (n + tile_n - 1) // tile_n if n > 0 else 0
        for rb in range(n_rb):
            for tt in range(ntt):
                items.append((g, rb, r0 + tt * tile_n, min(tile_n, n - tt * tile_n), src, ret + tt * tile_n))
    return items
