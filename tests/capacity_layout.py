"""Specification of capacity-limited routing across expert-parallel ranks (test helper).

topkgating_full (src/hunyuan_moe_full.cpp:182-316) keeps a (token, choice k) pair when its
position among its expert's pairs, in k-major order over the call's tokens (every token's
first choice, then every token's second, ...), is below the capacity.  Spread over ranks, the
job's tokens are taken in rank order (rank 0's tokens first), so each rank needs only the
per-(choice, expert) pair counts of every rank:

    priority(t, k) = sum_{k' < k} sum_r C[r][k'][e]        (earlier choices, whole job)
                   + sum_{r < me} C[r][k][e]                (earlier ranks, same choice)
                   + #{t' < t on this rank : idx[t', k] = e}  (earlier local tokens)

with capacity max(K, (uint32)(capacity_factor * K * T_job / E)) (at least min_capacity) when
dropping, else the largest job-wide expert count (nothing dropped).  One rank (N = 1) is the
single-call case.  The device plan implements this as one more counting pass per choice k.
"""
import numpy as np


def choice_counts(idx: np.ndarray, E: int) -> np.ndarray:
    """C[k][e]: pairs of this rank whose k-th choice is expert e."""
    T, K = idx.shape
    C = np.zeros((K, E), np.int64)
    for k in range(K):
        C[k] = np.bincount(idx[:, k], minlength=E) if T else 0
    return C


def capacity(T_job: int, K: int, E: int, counts_job: np.ndarray, drop: float | None,
             min_capacity: int) -> int:
    if drop is not None:
        f = int(np.float32(np.float32(drop) * np.float32(K) * np.float32(T_job) / np.float32(E)))
        cap = max(K, f)
    else:
        cap = int(counts_job.max()) if counts_job.size else 0
    return max(cap, min_capacity)


def priorities(idx: np.ndarray, C_all: np.ndarray, me: int) -> np.ndarray:
    """Priority of every local pair; C_all [N][K][E] = every rank's choice_counts."""
    T, K = idx.shape
    E = C_all.shape[2]
    job = C_all.sum(axis=0)                                  # [K][E]
    before_k = np.vstack([np.zeros((1, E), np.int64), np.cumsum(job, axis=0)[:-1]])
    before_r = C_all[:me].sum(axis=0) if me else np.zeros((K, E), np.int64)
    prio = np.empty((T, K), np.int64)
    for k in range(K):
        seen = np.zeros(E, np.int64)
        for t in range(T):
            e = idx[t, k]
            prio[t, k] = before_k[k, e] + before_r[k, e] + seen[e]
            seen[e] += 1
    return prio
