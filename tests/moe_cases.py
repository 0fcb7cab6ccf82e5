"""Shared builders and metrics for the parity tests (test infrastructure).

Weights and activations come from the seeded synthetic generator (Philox4x32-10 +
Irwin-Hall) that the oracle and the library implement independently; parity metrics
follow the acceptance criteria: expert sets equal wherever the K-th / (K+1)-th logit gap
exceeds 1e-4, output relative L2 error <= 1e-3 against the reference.
"""
from __future__ import annotations

import os

import numpy as np

import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
REL_L2_TOL = 1e-3     # output tolerance (fp16 tensor-core operands, fp32 accumulate)
GAP_TOL = 1e-4        # logit gap above which the selected expert set must match exactly


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def topk_mismatches(idx_a, idx_b, logits, K: int) -> tuple[int, int]:
    """(#tokens whose expert sets differ although the gap exceeds GAP_TOL, #near ties)."""
    srt = -np.sort(-logits, axis=1)
    gap = srt[:, K - 1] - srt[:, K] if logits.shape[1] > K else np.full(len(logits), np.inf)
    bad = ties = 0
    for t in range(len(idx_a)):
        if gap[t] > GAP_TOL:
            bad += set(idx_a[t].tolist()) != set(idx_b[t].tolist())
        else:
            ties += 1
    return bad, ties


def host_layer(orc: O.Oracle, seed: int, layer: int, H: int, I: int, E: int, wtype: int,
               std: float = 0.02):
    """GGUF bytes for every tensor of a synthetic layer, plus the F32 tensors the oracle
    consumes (quantised then dequantised with the standard GGUF rule)."""
    sid = O.stream_id
    rw = orc.fill_normal(E * H, seed, sid(layer, O.KIND_ROUTER), std).reshape(E, H)

    def pair(kind, idx, n):
        raw = orc.synth_tensor(wtype, n, seed, sid(layer, kind, idx), std)
        f32 = (raw.view(np.float32).copy() if wtype == O.F32 else orc.dequantize(wtype, raw, n))
        return raw, f32

    sgu, sgu_f = pair(O.KIND_GATE_UP, O.SHARED_INDEX, 2 * I * H)
    sdn, sdn_f = pair(O.KIND_DOWN, O.SHARED_INDEX, H * I)
    egu, edn, egu_f, edn_f = [], [], [], []
    for e in range(E):
        a, af = pair(O.KIND_GATE_UP, e, 2 * I * H)
        b, bf = pair(O.KIND_DOWN, e, H * I)
        egu.append(a)
        edn.append(b)
        egu_f.append(af)
        edn_f.append(bf)
    return dict(router=rw, sgu=sgu, sdn=sdn, egu=egu, edn=edn, sgu_f=sgu_f, sdn_f=sdn_f,
                egu_f=egu_f, edn_f=edn_f)


def load_fixture(name: str) -> dict:
    d = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    H, I, E, K, T, wt, seed = (int(v) for v in d["meta"])
    return dict(H=H, I=I, E=E, K=K, T=T, wt=wt, seed=seed, out=d["out"], probs=d["probs"],
                w=d["w"], idx=d["idx"], checksum=d["checksum"])


SMALL_FIXTURES = ["small_f32", "small_q4_0", "small_q8_0", "ragged_q4_0", "multitile_q8_0",
                  "topk4_f16"]
FULL_FIXTURES = ["full_f32_t2", "full_q4_0_t2", "full_q8_0_t1"]


def input_checksum(x: np.ndarray, rw: np.ndarray) -> np.ndarray:
    return np.array([np.float64(x).sum(), np.float64(np.abs(x)).sum(), np.float64(rw).sum()])


def fixture_inputs(orc: O.Oracle, fx: dict):
    """Regenerates a golden case's inputs as tests/golden/make_golden.py made them: x, and
    F32 weights for the shared expert and the experts the tokens select."""
    H, I, E, K, T, wt, seed = (fx[k] for k in ("H", "I", "E", "K", "T", "wt", "seed"))
    x = O.synth_x(orc, seed, T, H)
    rw = orc.fill_normal(E * H, seed, O.stream_id(0, O.KIND_ROUTER), 0.02).reshape(E, H)
    _, _, _, ti = orc.router(x, rw, K)
    w = O.synth_layer_f32(orc, seed, 0, H, I, E, wt, experts=np.unique(ti))
    return x, w, input_checksum(x, rw)


def check_full_routing(mine: dict, ref: dict, K: int) -> None:
    """The FULL-mode routing restatement (idx, w, keep per pair) against the reference's
    topkgating_full outputs (probs, dispatch mask and combine weights [T, E, capacity],
    expert counts, capacity, capacity rate): every kept pair has exactly one mask entry whose
    combine weight is its w; dropped and unselected (token, expert) pairs have none."""
    T, E = ref["probs"].shape
    assert np.array_equal(mine["probs"], ref["probs"])
    assert mine["capacity"] == ref["capacity"]
    assert np.array_equal(mine["exp_counts"], ref["exp_counts"])
    m, cw = ref["mask"], ref["combine"]
    assert m.shape == (T, E, ref["capacity"])
    seen = np.zeros((T, E), bool)
    for t in range(T):
        for k in range(K):
            e = int(mine["idx"][t, k])
            assert not seen[t, e], "an expert chosen twice"
            seen[t, e] = True
            hits = np.nonzero(m[t, e])[0]
            if mine["keep"][t, k]:
                assert len(hits) == 1 and cw[t, e, hits[0]] == mine["w"][t, k], (t, k)
            else:
                assert len(hits) == 0, (t, k)
    assert not m[~seen].any()
    # the reference divides in single precision: kept pairs / (T * K)
    assert np.float32(mine["keep"].sum()) / np.float32(T * K) == np.float32(ref["rate"])
