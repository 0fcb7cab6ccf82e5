"""Capacity-limited routing across expert-parallel ranks, on CPU gloo ranks (world 2 and 4):
each rank routes its own tokens, the ranks all-gather their per-(choice, expert) pair counts,
and each rank decides which of its pairs are kept by the specification in
tests/capacity_layout.py.  The union must equal one topkgating_full call (the oracle, pinned to
the reference) over the job's tokens in rank order: same experts, same capacity, same kept
pairs — ranks with no tokens included.  Also checks the single-rank case directly."""
import datetime
import multiprocessing as mp
import os
import socket
import sys

import numpy as np
import pytest

from capacity_layout import capacity, choice_counts, priorities

E, K = 64, 8
HERE = os.path.dirname(os.path.abspath(__file__))


def _logits(rank: int, T: int) -> np.ndarray:
    rng = np.random.default_rng(900 + rank)
    return (np.round(rng.standard_normal((T, E)) * 4) / 4).astype(np.float32)  # ties included


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, tokens, opts, q):
    sys.path[:0] = [os.path.join(os.path.dirname(HERE), "oracle"), HERE]
    import torch
    import torch.distributed as dist
    import oracle as O2
    from capacity_layout import capacity as cap_fn, choice_counts as cc, priorities as pr
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        orc = O2.Oracle(nthreads=1)
        T = tokens[rank]
        route = {k: v for k, v in opts.items() if k not in ("drop", "min_capacity")}
        idx = orc.topkgating_full(_logits(rank, T), K, **route)["idx"] if T else np.zeros((0, K), np.int32)
        C = torch.from_numpy(cc(idx, E))
        allC = [torch.zeros_like(C) for _ in range(world)]
        dist.all_gather(allC, C)
        C_all = torch.stack(allC).numpy()
        cap = cap_fn(sum(tokens), K, E, C_all.sum(axis=(0, 1)), opts.get("drop"), opts.get("min_capacity", 8))
        keep = pr(idx, C_all, rank) < cap
        q.put((rank, "ok", idx, keep, cap))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, f"error: {e!r}", None, None, None))
    finally:
        dist.destroy_process_group()


def _run(world, tokens, opts):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, tokens, opts, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        rank, status, idx, keep, cap = q.get(timeout=300)
        assert status == "ok", f"rank {rank}: {status}"
        res[rank] = (idx, keep, cap)
    for p in ps:
        p.join(timeout=60)
    return res


@pytest.mark.parametrize("world,tokens,opts", [
    (2, [40, 23], {"drop": 1.0}),
    (2, [70, 0], {"drop": 0.5, "min_capacity": 2}),
    (4, [9, 30, 0, 17], {"drop": 1.0, "group": (8, 3)}),
    (4, [12, 12, 12, 12], {"drop": 2.0, "min_capacity": 4, "norm_topk_prob": False, "scale": 2.0}),
])
def test_capacity_over_ranks_equals_one_call_over_the_job(orc, world, tokens, opts):
    res = _run(world, tokens, opts)
    logits = np.concatenate([_logits(r, t) for r, t in enumerate(tokens)])
    want = orc.topkgating_full(logits, K, **opts)
    assert all(res[r][2] == want["capacity"] for r in range(world))
    idx = np.concatenate([res[r][0] for r in range(world)])
    keep = np.concatenate([res[r][1] for r in range(world)])
    assert np.array_equal(idx, want["idx"])
    assert np.array_equal(keep, want["keep"])
    assert 0 < keep.mean() < 1.0 or opts.get("drop", 0) >= 2.0  # some pairs dropped in the tight cases


@pytest.mark.parametrize("opts", [{"drop": 1.0}, {"drop": 0.75, "group": (4, 2)}, {}])
def test_single_rank_priorities_equal_the_oracle(orc, opts):
    lg = _logits(7, 200)
    a = orc.topkgating_full(lg, K, **opts)
    C = choice_counts(a["idx"], E)[None]
    cap = capacity(200, K, E, C.sum(axis=(0, 1)), opts.get("drop"), opts.get("min_capacity", 8))
    assert cap == a["capacity"]
    assert np.array_equal(priorities(a["idx"], C, 0) < cap, a["keep"])
