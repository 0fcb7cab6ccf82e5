"""Generate the golden fixtures under tests/golden/ by running the REFERENCE's own
moe_forward_cpu (src/attention.cpp:191-313), compiled from the reference sources into
oracle/_ref/libhyref.so by oracle/Makefile.

Inputs are never stored for the full-shape cases: weights and activations are
regenerated from (seed, layer, stream) by the synthetic generator (Philox4x32-10 +
Irwin-Hall), whose known-answer vectors tests/test_oracle.py pins.  Each fixture
records the case parameters, the reference outputs and a checksum of the inputs so a
drifting generator is caught.

Run (needs the reference tree, i.e. only in the build container):
    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402

# name, H, I, E, K, T, weight type, seed
CASES = [
    ("small_f32", 256, 192, 64, 8, 16, O.F32, 0),
    ("small_q4_0", 512, 384, 64, 8, 32, O.Q4_0, 1),
    ("small_q8_0", 512, 256, 64, 8, 24, O.Q8_0, 2),
    ("ragged_q4_0", 384, 128, 16, 8, 7, O.Q4_0, 3),
    ("multitile_q8_0", 256, 128, 8, 8, 300, O.Q8_0, 4),
    ("topk4_f16", 256, 64, 32, 4, 40, O.F16, 5),
    ("full_f32_t2", 4096, 3072, 64, 8, 2, O.F32, 0),
    ("full_q4_0_t2", 4096, 3072, 64, 8, 2, O.Q4_0, 0),
    ("full_q8_0_t1", 4096, 3072, 64, 8, 1, O.Q8_0, 0),
]


def input_checksum(x: np.ndarray, rw: np.ndarray) -> np.ndarray:
    return np.array([np.float64(x).sum(), np.float64(np.abs(x)).sum(), np.float64(rw).sum()])


def run_case(orc: O.Oracle, ref: O.RefMoE, name, H, I, E, K, T, wt, seed):
    x = O.synth_x(orc, seed, T, H)
    rw = orc.fill_normal(E * H, seed, O.stream_id(0, O.KIND_ROUTER), 0.02).reshape(E, H)
    _, _, _, ti = orc.router(x, rw, K)
    rw, sgu, sdn, egu, edn = O.synth_layer_f32(orc, seed, 0, H, I, E, wt,
                                               experts=np.unique(ti))
    h = ref.weights(H, I, rw, sgu, sdn, egu, edn)
    t0 = time.time()
    r = ref.moe_forward(x, h, E, H, I, K)
    dt = time.time() - t0
    ref.free(h)
    meta = np.array([H, I, E, K, T, wt, seed], dtype=np.int64)
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, meta=meta, out=r["out"], probs=r["probs"], w=r["w"], idx=r["idx"],
                        checksum=input_checksum(x, rw))
    print(f"{name}: reference {dt:.2f}s -> {os.path.getsize(path)} bytes")


def run_rms_norm(orc: O.Oracle, ref: O.RefMoE) -> None:
    """rms_norm_f32 (src/rms_norm.cpp:9-33) on rows of very different scales, with the inputs
    stored (they are small)."""
    rng = np.random.default_rng(7)
    cases = {}
    for name, T, H, eps in (("h512", 9, 512, 1e-5), ("h4096", 3, 4096, 1e-6)):
        x = O.synth_x(orc, 31 + H, T, H)
        x *= np.float32(10.0) ** rng.integers(-6, 5, size=(T, 1)).astype(np.float32)
        w = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        cases[name] = (x, w, eps, ref.rms_norm(x, w, eps))
    path = os.path.join(HERE, "rms_norm.npz")
    np.savez_compressed(path, **{f"{n}_{k}": v for n, (x, w, eps, out) in cases.items()
                                 for k, v in (("x", x), ("w", w), ("eps", np.float32(eps)), ("out", out))})
    print(f"rms_norm: {os.path.getsize(path)} bytes")


# FULL-mode routing cases: name, T, E, K, options of topkgating_full
ROUTING_CASES = [
    ("plain", 37, 64, 8, {}),
    ("group", 37, 64, 8, {"group": (8, 3)}),
    ("drop", 64, 64, 8, {"drop": 1.0}),
    ("group_drop_scaled", 20, 16, 4, {"group": (4, 2), "drop": 1.25, "norm_topk_prob": False, "scale": 2.5}),
    ("top1_drop", 9, 64, 1, {"drop": 1.0, "min_capacity": 1}),
]


def routing_options(opts: dict) -> np.ndarray:
    g = opts.get("group") or (0, 0)
    return np.array([1 if opts.get("group") else 0, g[0], g[1], 0 if opts.get("drop") is None else 1,
                     opts.get("drop") or 1.0, opts.get("min_capacity", 8),
                     1 if opts.get("norm_topk_prob", True) else 0, opts.get("scale", 1.0)], np.float64)


def run_routing_full(ref: O.RefMoE) -> None:
    """topkgating_full (src/hunyuan_moe_full.cpp:119-350) on seeded logits, half of them
    rounded to steps of 0.5 so that ties occur."""
    rng = np.random.default_rng(17)
    arrays = {}
    for name, T, E, K, opts in ROUTING_CASES:
        for tie in (False, True):
            lg = (rng.standard_normal((T, E)) * 2).astype(np.float32)
            if tie:
                lg = (np.round(lg * 2) / 2).astype(np.float32)
            r = ref.topkgating_full(lg, K, **opts)
            key = f"{name}{'_ties' if tie else ''}"
            arrays.update({f"{key}_logits": lg, f"{key}_k": np.int64(K), f"{key}_opts": routing_options(opts),
                           f"{key}_probs": r["probs"], f"{key}_mask": r["mask"], f"{key}_combine": r["combine"],
                           f"{key}_counts": r["exp_counts"], f"{key}_capacity": np.int64(r["capacity"]),
                           f"{key}_rate": np.float32(r["rate"])})
    path = os.path.join(HERE, "routing_full.npz")
    np.savez_compressed(path, **arrays)
    print(f"routing_full: {os.path.getsize(path)} bytes")


def main():
    orc = O.Oracle()
    ref = O.RefMoE()
    only = set(sys.argv[1:])
    for c in CASES:
        if not only or c[0] in only:
            run_case(orc, ref, *c)
    if not only or "rms_norm" in only:
        run_rms_norm(orc, ref)
    if not only or "routing_full" in only:
        run_routing_full(ref)


if __name__ == "__main__":
    main()
