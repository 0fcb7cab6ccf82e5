"""CPU tests of the oracle (the checker): generator known answers, binary16 and GGUF
block formats against numpy / gguf-py, and the MoE restatement against the golden
fixtures produced by the reference's own moe_forward_cpu."""
import os

import numpy as np
import pytest

import oracle as O
from moe_cases import FULL_FIXTURES, SMALL_FIXTURES, fixture_inputs, load_fixture


def test_philox_known_answers(orc):
    # Known-answer vectors of Philox4x32-10 (Random123 kat_vectors).
    assert [hex(v) for v in orc.philox([0, 0, 0, 0], [0, 0])] == [
        "0x6627e8d5", "0xe169c58d", "0xbc57ac4c", "0x9b00dbd8"]
    assert [hex(v) for v in orc.philox([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2)] == [
        "0x408f276d", "0x41c83b0e", "0xa20bc7c6", "0x6d5451fd"]
    assert [hex(v) for v in orc.philox([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344],
                                       [0xA4093822, 0x299F31D0])] == [
        "0xd16cfe09", "0x94fdcceb", "0x5001e420", "0x24126ea1"]


def test_generator_moments(orc):
    x = orc.fill_normal(1 << 20, 0, 123, 0.02)
    assert abs(float(x.mean())) < 1e-4
    assert abs(float(x.std()) - 0.02) < 2e-4
    # deterministic and thread-count independent
    y = O.Oracle(nthreads=1).fill_normal(1 << 12, 0, 123, 0.02)
    assert np.array_equal(x[: 1 << 12], y)


def test_f16_conversion_matches_numpy(orc):
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(4000).astype(np.float32) * s
                           for s in (1e-8, 6e-8, 1e-6, 1e-4, 1.0, 100.0, 6.5e4)])
    vals = np.concatenate([vals, np.float32([0.0, -0.0, 65504.0, 65519.0, 65520.0, np.inf])])
    mine = np.array([orc.L.oracle_f32_to_f16(float(v)) for v in vals], dtype=np.uint16)
    with np.errstate(over="ignore"):
        ref = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(mine, ref)
    back = np.array([orc.L.oracle_f16_to_f32(int(h)) for h in ref[:3000]], dtype=np.float32)
    assert np.array_equal(back, ref[:3000].view(np.float16).astype(np.float32))


@pytest.mark.parametrize("t", [O.Q4_0, O.Q8_0])
def test_gguf_blocks_match_gguf_py(orc, t):
    gq = pytest.importorskip("gguf.quants")
    from gguf import GGMLQuantizationType as QT
    qt = {O.Q4_0: QT.Q4_0, O.Q8_0: QT.Q8_0}[t]
    w = orc.fill_normal(32 * 2048, 1, 7, 0.02)
    w[:32] = 0.0                      # all-zero block: d = 0
    w[32:64] = np.linspace(-1, 1, 32)  # exact extremes
    a = orc.quantize(t, w)
    b = gq.quantize(w.reshape(-1, 32 * 16), qt).ravel()
    assert np.array_equal(a, b)
    assert np.array_equal(orc.dequantize(t, a, w.size), gq.dequantize(b.reshape(1, -1), qt).ravel())


def test_synth_tensor_equals_fill_then_quantize(orc):
    n = 32 * 300
    raw = orc.synth_tensor(O.Q4_0, n, 9, 42, 0.02)
    assert np.array_equal(raw, orc.quantize(O.Q4_0, orc.fill_normal(n, 9, 42, 0.02)))
    f = orc.synth_tensor_f32(O.Q8_0, n, 9, 42, 0.02)
    assert np.array_equal(f, orc.dequantize(O.Q8_0, orc.quantize(O.Q8_0, orc.fill_normal(n, 9, 42, 0.02)), n))


@pytest.mark.parametrize("name", SMALL_FIXTURES + FULL_FIXTURES)
def test_restatement_matches_reference_golden(orc, name):
    fx = load_fixture(name)
    x, w, ck = fixture_inputs(orc, fx)
    np.testing.assert_allclose(ck, fx["checksum"], rtol=1e-12)
    r = orc.moe_forward(x, w[0], w[1], w[2], w[3], w[4], fx["K"], fx["I"])
    assert np.array_equal(r["idx"], fx["idx"])
    assert np.array_equal(r["w"], fx["w"])
    assert np.array_equal(r["probs"], fx["probs"])
    assert np.array_equal(r["out"], fx["out"])  # bit-identical to the reference


def test_router_ties_pick_lower_expert(orc):
    """Equal probabilities: the reference's insertion keeps the lower expert first."""
    H, E, K = 64, 16, 8
    rw = np.zeros((E, H), np.float32)
    rw[:, 0] = np.float32([1, 2, 2, 3, 3, 3, 0, 0, 1, 1, 2, 0, 3, 1, 2, 0]) * 0.1
    x = np.ones((1, H), np.float32)
    _, _, tw, ti = orc.router(x, rw, K)
    assert ti[0].tolist() == [3, 4, 5, 12, 1, 2, 10, 14]
    if O.RefMoE.available():
        ref = O.RefMoE()
        I = 64
        z = np.zeros(2 * I * H, np.float32)
        d = np.zeros(H * I, np.float32)
        h = ref.weights(H, I, rw, z, d, [z] * E, [d] * E)
        r = ref.moe_forward(x, h, E, H, I, K)
        ref.free(h)
        assert r["idx"][0].tolist() == ti[0].tolist()
        assert np.array_equal(r["w"], tw)


def test_bias_zero_equals_no_bias(orc):
    H, I, E, K, T = 128, 64, 16, 8, 5
    rw, sgu, sdn, egu, edn = O.synth_layer_f32(orc, 3, 0, H, I, E, O.Q8_0)
    x = O.synth_x(orc, 3, T, H)
    a = orc.moe_forward(x, rw, sgu, sdn, egu, edn, K, I)
    b = orc.moe_forward(x, rw, sgu, sdn, egu, edn, K, I, bias=np.zeros(E, np.float32))
    assert np.array_equal(a["out"], b["out"])


@pytest.mark.skipif(not O.RefMoE.available(), reason="reference checker not built here")
@pytest.mark.parametrize("seed,H,I,E,K,T", [(11, 256, 128, 32, 8, 13), (12, 256, 128, 32, 8, 13),
                                            (13, 128, 64, 8, 1, 5), (14, 384, 192, 16, 2, 33),
                                            (15, 128, 128, 32, 6, 1), (16, 256, 64, 64, 8, 9)])
def test_restatement_matches_compiled_reference(orc, seed, H, I, E, K, T):
    """Every output of moe_forward_cpu (output, probabilities, top-K weights and indices) is
    bit-identical between the restatement and the reference compiled from its sources, over
    expert counts 8..64, K 1..8, hidden sizes 128..384 and 1..33 tokens."""
    rw, sgu, sdn, egu, edn = O.synth_layer_f32(orc, seed, 0, H, I, E, O.Q4_0)
    x = O.synth_x(orc, seed, T, H)
    ref = O.RefMoE()
    h = ref.weights(H, I, rw, sgu, sdn, egu, edn)
    r = ref.moe_forward(x, h, E, H, I, K)
    ref.free(h)
    o = orc.moe_forward(x, rw, sgu, sdn, egu, edn, K, I)
    for k in ("out", "idx", "w", "probs"):
        assert np.array_equal(r[k], o[k]), k


def test_rms_norm_restatement_matches_reference_golden(orc):
    """oracle_rms_norm against the reference's rms_norm_f32 (src/rms_norm.cpp:9-33) outputs
    stored in tests/golden/rms_norm.npz: bit-identical, rows spanning 1e-6 .. 1e4 in scale."""
    d = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "rms_norm.npz"))
    for n in ("h512", "h4096"):
        got = orc.rms_norm(d[f"{n}_x"], d[f"{n}_w"], float(d[f"{n}_eps"]))
        assert np.array_equal(got, d[f"{n}_out"]), n


@pytest.mark.skipif(not O.RefMoE.available(), reason="reference checker not built here")
def test_rms_norm_restatement_matches_compiled_reference(orc):
    ref = O.RefMoE()
    rng = np.random.default_rng(5)
    for T, H, eps in ((1, 128, 1e-5), (17, 384, 1e-6), (4, 4096, 0.0)):
        x = (rng.standard_normal((T, H)) * 10.0 ** rng.integers(-5, 5, size=(T, 1))).astype(np.float32)
        w = rng.standard_normal(H).astype(np.float32)
        assert np.array_equal(orc.rms_norm(x, w, eps), ref.rms_norm(x, w, eps))


def _routing_opts(v: np.ndarray) -> dict:
    opts = {"min_capacity": int(v[5]), "norm_topk_prob": bool(v[6]), "scale": float(v[7])}
    if v[0]:
        opts["group"] = (int(v[1]), int(v[2]))
    if v[3]:
        opts["drop"] = float(v[4])
    return opts


def test_full_routing_restatement_matches_reference_golden(orc):
    """FULL-mode routing (topkgating_full, src/hunyuan_moe_full.cpp:119-350: group-limited
    greedy, capacity with k-major drop priority, renormalisation or scaling) against the
    reference's outputs stored in tests/golden/routing_full.npz, ties included."""
    from moe_cases import check_full_routing
    d = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "routing_full.npz"))
    keys = sorted({k[: -len("_logits")] for k in d.files if k.endswith("_logits")})
    assert len(keys) == 10
    for key in keys:
        K = int(d[f"{key}_k"])
        mine = orc.topkgating_full(d[f"{key}_logits"], K, **_routing_opts(d[f"{key}_opts"]))
        ref = {"probs": d[f"{key}_probs"], "mask": d[f"{key}_mask"], "combine": d[f"{key}_combine"],
               "exp_counts": d[f"{key}_counts"], "capacity": int(d[f"{key}_capacity"]),
               "rate": float(d[f"{key}_rate"])}
        check_full_routing(mine, ref, K)


@pytest.mark.skipif(not O.RefMoE.available(), reason="reference checker not built here")
@pytest.mark.parametrize("opts", [{}, {"group": (8, 3)}, {"drop": 1.0}, {"drop": 0.5, "min_capacity": 2},
                                  {"group": (4, 1), "drop": 2.0, "norm_topk_prob": False, "scale": 0.7}])
def test_full_routing_restatement_matches_compiled_reference(orc, opts):
    from moe_cases import check_full_routing
    ref = O.RefMoE()
    rng = np.random.default_rng(len(opts))
    for T in (1, 16, 130):
        lg = (rng.standard_normal((T, 64)) * 3).astype(np.float32)
        check_full_routing(orc.topkgating_full(lg, 8, **opts), ref.topkgating_full(lg, 8, **opts), 8)
