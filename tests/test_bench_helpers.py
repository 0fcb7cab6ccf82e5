"""CPU tests of bench.py's parity statistics (the `parity` object of the bench line): output
relative L2 against its tolerance, top-K agreement, and near ties (K-th/(K+1)-th logit gap at
most 1e-4) excluded rather than counted as mismatches."""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def _case(T=4, E=16, K=4, seed=0):
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    idx = np.argsort(-logits, axis=1)[:, :K].astype(np.int32)
    out = rng.standard_normal((T, 32)).astype(np.float32)
    return logits, idx, out


def test_identical_outputs_pass():
    logits, idx, out = _case()
    p = bench.parity_stats({"out": out, "idx": idx, "logits": logits}, out, idx, 4)
    assert p["ok"] and p["rel_l2"] == 0.0 and p["topk_match"] == 1.0
    assert p["near_ties_excluded"] == 0 and p["topk_mismatches"] == 0


def test_mismatch_outside_a_near_tie_fails():
    logits, idx, out = _case()
    bad = idx.copy()
    bad[1, -1] = np.argsort(-logits[1])[4]  # the 5th expert instead of the 4th
    p = bench.parity_stats({"out": out, "idx": bad, "logits": logits}, out, idx, 4)
    assert not p["ok"] and p["topk_mismatches"] == 1 and p["topk_match"] == 0.75


def test_mismatch_at_a_near_tie_is_excluded():
    logits, idx, out = _case()
    order = np.argsort(-logits[2])
    logits[2, order[4]] = logits[2, order[3]] - 5e-5  # 4th/5th gap below 1e-4
    bad = idx.copy()
    bad[2, -1] = order[4]
    p = bench.parity_stats({"out": out, "idx": bad, "logits": logits}, out, idx, 4)
    assert p["ok"] and p["near_ties_excluded"] == 1 and p["topk_mismatches"] == 0


def test_output_error_above_tolerance_fails():
    logits, idx, out = _case()
    noisy = out * np.float32(1.01)
    p = bench.parity_stats({"out": noisy, "idx": idx, "logits": logits}, out, idx, 4)
    assert not p["ok"] and abs(p["rel_l2"] - 0.01) < 1e-4


def test_workload_zipf_bias_equals_the_oracle_restatement():
    """The package's Zipf(1.1) router bias (what bench.py feeds the GPU) is the oracle's
    zipf_bias (what the parity tests feed the checker)."""
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
    import hymoe
    import oracle as O
    for seed in (0, 5, 104):
        assert np.array_equal(hymoe.zipf_router_bias(seed, 64), O.zipf_bias(seed, 64))
