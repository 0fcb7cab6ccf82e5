"""Expert-parallel host logic on CPU: world-size-2 (and 4) gloo process groups exchange the
per-expert counts the way the library's count exchange does, compute the row layout of
tests/ep_layout.py, and check it end to end:

- every pair of every source lands on a distinct row of its owner, and the rows an owner
  receives are exactly [T_d, T_d + received) — no gaps, no overlaps, within capacity;
- each received row falls in the segment (source, local expert) of its pair;
- routing results back by the same rows reproduces every source's own pairs (the combine's
  inputs), whatever the token counts (including a rank with no tokens);
- with an expert placement (top-K slots instead of expert ids; the owner computes the expert
  its slot holds), every source still gets back the results of its own experts.

Failure detection: a rank that stops taking part makes the others' next collective end with
an error within a short process-group timeout (no hang).
"""
import datetime
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from ep_layout import recv_segments, rows_cap, send_rows

E, K = 64, 8


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, tokens, q, place=False):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        el = E // world
        T = tokens[rank]
        rng = np.random.default_rng(100 + rank)
        experts = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]) if T else np.zeros((0, K), np.int64)
        # placement: the same seeded permutation on every rank (identity without one)
        slot_of = np.random.default_rng(5).permutation(E) if place else np.arange(E)
        expert_of = np.argsort(slot_of)
        topk = slot_of[experts]  # what the top-K step hands on: slots
        counts = torch.from_numpy(np.bincount(topk.ravel(), minlength=E).astype(np.int64))
        allc = [torch.zeros(E, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(allc, counts)  # the count exchange
        C = torch.stack(allc).numpy()
        Ts = [int(c.sum()) // K for c in C]
        assert Ts == list(tokens)
        owner, row = send_rows(topk, C, Ts, rank, el)
        # every rank learns every source's (owner, row, expert, token id) of every pair
        mine = np.stack([owner.ravel(), row.ravel(), topk.ravel(),
                         np.repeat(np.arange(T), K) + 10000 * rank]).astype(np.int64) if T else np.zeros((4, 0), np.int64)
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, torch.tensor([mine.shape[1]]))
        n_max = max(int(s) for s in sizes)
        pad = np.full((4, n_max), -1, np.int64)
        pad[:, :mine.shape[1]] = mine
        got = [torch.zeros(4, n_max, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(got, torch.from_numpy(pad))
        # as owner `rank`: the rows this rank receives
        recv = []
        for s, g in enumerate(got):
            g = g.numpy()[:, :int(sizes[s])]
            sel = g[0] == rank
            recv.append((s, g[1, sel], g[2, sel], g[3, sel]))
        rows = np.concatenate([r[1] for r in recv]) if recv else np.zeros(0, np.int64)
        total = sum(len(r[1]) for r in recv)
        assert np.array_equal(np.sort(rows), np.arange(Ts[rank], Ts[rank] + total)), "rows not a bijection"
        assert Ts[rank] + total <= rows_cap(max(tokens), world, K, el)
        segs = recv_segments(C, Ts, rank, el)
        assert segs[-1][1] + segs[-1][2] == Ts[rank] + total
        for s, rr, ee, _ in recv:
            for r, e in zip(rr, ee):
                hit = [g for g in segs[1:] if g[1] <= r < g[1] + g[2]]
                assert len(hit) == 1 and hit[0][3] == s and hit[0][0] == e - rank * el
        # results back: owner returns row r's "result" (the pair's id) to its source; each
        # source must see exactly its own pairs in (t, k) order
        # the owner runs the expert its slot holds
        result = {int(r): int(tid) * 100 + int(expert_of[e]) for s, rr, ee, tt in recv for r, e, tid in zip(rr, ee, tt)}
        res_all = [None] * world
        dist.all_gather_object(res_all, result)
        if T:
            back = np.array([res_all[o][int(r)] for o, r in zip(owner.ravel(), row.ravel())]).reshape(T, K)
            expect = (np.arange(T)[:, None] + 10000 * rank) * 100 + experts
            assert np.array_equal(back, expect)
        q.put((rank, "ok"))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, f"error: {e!r}"))
    finally:
        dist.destroy_process_group()


def _run(world, tokens, place=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, tokens, q, place)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
    return res


@pytest.mark.parametrize("world,tokens", [(2, [37, 20]), (2, [16, 0]), (4, [9, 0, 33, 4])])
def test_ep_row_layout_over_gloo(world, tokens):
    res = _run(world, tokens)
    assert all(v == "ok" for v in res.values()), res


@pytest.mark.parametrize("world,tokens", [(2, [29, 11]), (4, [7, 25, 0, 16])])
def test_ep_row_layout_with_expert_placement_over_gloo(world, tokens):
    res = _run(world, tokens, place=True)
    assert all(v == "ok" for v in res.values()), res


def _leaver(rank, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=3))
    t = torch.ones(4)
    dist.all_reduce(t)  # both ranks take part once
    if rank == 1:
        q.put((1, "left"))  # stops taking part between steps
        return
    try:
        dist.all_reduce(t)  # the next collective must end with an error, not hang
        q.put((0, "no error"))
    except Exception as e:
        q.put((0, f"error: {type(e).__name__}"))


def test_rank_that_leaves_ends_the_next_collective_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_leaver, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("error"), res
