"""GPU tests of the one-kernel decode path (csrc/decode.cu): 1..8 tokens on one GPU, Q4_0 or
Q8_0 experts, the whole block (router chains, top-K, both experts' weight streams, combine) in
one cooperative kernel.

The one-kernel path is enabled per context with HYMOE_DECODE_FUSED=1 at creation; the
multi-kernel path (HYMOE_DECODE_FUSED=0, the default) computes every logit,
selection, weight and output with the same arithmetic in the same order, so the two must agree
bit for bit; against the oracle (the C restatement of moe_forward_cpu, src/attention.cpp:191-313)
the usual tolerances hold: experts equal outside 1e-4 logit gaps, relative L2 <= 1e-3.
Repeated and graph-replayed calls check that the kernel leaves its counters at zero.
"""
import os

import numpy as np
import pytest

import hymoe
import oracle as O
from moe_cases import REL_L2_TOL, host_layer, rel_l2, topk_mismatches

pytestmark = pytest.mark.gpu


def _ctx_with(flag, H, I, E, K, T, layers):
    old = os.environ.get("HYMOE_DECODE_FUSED")
    os.environ["HYMOE_DECODE_FUSED"] = flag
    try:
        return hymoe.MoE(H, I, E, K, layers, max(T, 16))
    finally:
        if old is None:
            del os.environ["HYMOE_DECODE_FUSED"]
        else:
            os.environ["HYMOE_DECODE_FUSED"] = old


def _pair(H, I, E, K, T, layers=1):
    """(one-kernel context, multi-kernel context) of the same shape."""
    return _ctx_with("1", H, I, E, K, T, layers), _ctx_with("0", H, I, E, K, T, layers)


def _load(m, lay, wt, layer=0):
    m.load_layer(layer, lay["router"], lay["sgu"], lay["sdn"], lay["egu"], lay["edn"], wt)


def _same(a, b):
    for k in ("logits", "probs", "w", "idx", "out"):
        assert np.array_equal(a[k], b[k]), k


SMALL = {
    # H, I, E, K, wtype, T, router bias, pre-norm
    "q4_0_t1_bias": (512, 256, 64, 8, O.Q4_0, 1, True, False),
    "q4_0_t3": (512, 256, 64, 8, O.Q4_0, 3, False, False),
    "q8_0_t8_bias": (512, 256, 64, 8, O.Q8_0, 8, True, False),
    "q8_0_t5_prenorm": (512, 384, 64, 8, O.Q8_0, 5, True, True),
    "q4_0_e16_k4_t2": (256, 128, 16, 4, O.Q4_0, 2, False, False),
    "q8_0_e40_k6_t7": (384, 256, 40, 6, O.Q8_0, 7, True, False),
}


@pytest.mark.parametrize("case", list(SMALL))
def test_one_kernel_decode_equals_multi_kernel_and_oracle(orc, case):
    H, I, E, K, wt, T, with_bias, pre_norm = SMALL[case]
    seed = 300 + sum(map(ord, case))
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    x = O.synth_x(orc, seed, T, H)
    bias = O.synth_bias(orc, seed, E) if with_bias else None
    fused, multi = _pair(H, I, E, K, T)
    for m in (fused, multi):
        _load(m, lay, wt)
    xn = x
    if pre_norm:
        w = (1.0 + 0.1 * np.random.default_rng(seed).standard_normal(H)).astype(np.float32)
        for m in (fused, multi):
            m.set_norm(0, w, 1e-5)
        xn = orc.rms_norm(x, w, 1e-5)
    got = fused.forward_host(0, x, resid="x", bias=bias, debug=True, pre_norm=pre_norm)
    want = multi.forward_host(0, x, resid="x", bias=bias, debug=True, pre_norm=pre_norm)
    _same(got, want)
    o = orc.moe_forward(xn, lay["router"], lay["sgu_f"], lay["sdn_f"], lay["egu_f"], lay["edn_f"], K, I,
                        bias=bias, resid=x)
    assert np.array_equal(got["logits"], o["logits"])
    bad, _ = topk_mismatches(got["idx"], o["idx"], o["logits"], K)
    assert bad == 0
    assert rel_l2(got["out"], o["out"]) <= REL_L2_TOL
    fused.close()
    multi.close()


def test_routing_variants_and_placement_equal_multi_kernel(orc):
    """Group-limited routing (n_group 8, topk_group 3) and an expert placement (slots != expert
    ids): the one-kernel path routes with the same step and lists slots in the same order."""
    H, I, E, K, wt, T, seed = 512, 256, 64, 8, O.Q4_0, 6, 411
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    x = O.synth_x(orc, seed, T, H)
    perm = np.random.default_rng(seed).permutation(E)
    fused, multi = _pair(H, I, E, K, T)
    for m in (fused, multi):
        m.set_routing(group=(8, 3))
        m.set_placement(0, perm)
        _load(m, lay, wt)
    _same(fused.forward_host(0, x, debug=True), multi.forward_host(0, x, debug=True))
    for m in (fused, multi):
        m.set_routing(plain=True)
    _same(fused.forward_host(0, x, debug=True), multi.forward_host(0, x, debug=True))
    fused.close()
    multi.close()


def test_repeated_eager_graph_and_in_place_calls(orc):
    """30 device calls of 1, 8 and 3 tokens, eager and graph-replayed, one of them in place
    (x, residual and out one buffer): each gives the multi-kernel path's bits, so every call
    starts from zeroed counters."""
    torch = pytest.importorskip("torch")
    H, I, E, K, wt, seed = 512, 256, 64, 8, O.Q8_0, 421
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    fused, multi = _pair(H, I, E, K, 8)
    for m in (fused, multi):
        _load(m, lay, wt)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        fused.set_stream(st.cuda_stream)
        for call in range(30):
            T = (1, 8, 3)[call % 3]
            x = O.synth_x(orc, seed + call, T, H)
            want = multi.forward_host(0, x, resid="x")["out"]
            xd = torch.from_numpy(x).cuda()
            if call % 5 == 4:
                fused.forward_device(0, xd.data_ptr(), xd.data_ptr(), T, resid_ptr=xd.data_ptr())
                fused.synchronize()
                assert np.array_equal(xd.cpu().numpy(), want), f"in place, call {call}"
                continue
            od = torch.empty_like(xd)
            fused.forward_device(0, xd.data_ptr(), od.data_ptr(), T, resid_ptr=xd.data_ptr(), graph=call % 2 == 1)
            fused.synchronize()
            assert np.array_equal(od.cpu().numpy(), want), f"call {call}"
    fused.close()
    multi.close()


@pytest.mark.parametrize("wt,T", [(O.Q8_0, 1), (O.Q8_0, 8), (O.Q4_0, 4)])
def test_full_shape_one_kernel_decode(orc, wt, T):
    """The benchmark shape (H 4096, I 3072, E 64, K 8): bits of the multi-kernel path, and the
    oracle's experts and output within tolerance."""
    H, I, E, K, seed = 4096, 3072, 64, 8, 431 + T
    bias = O.synth_bias(orc, seed, E)
    fused, multi = _pair(H, I, E, K, T)
    for m in (fused, multi):
        m.synth_layer(0, wt, seed, 0.02)
    x = O.synth_x(orc, seed, T, H)
    got = fused.forward_host(0, x, bias=bias, debug=True)
    _same(got, multi.forward_host(0, x, bias=bias, debug=True))
    fused.close()
    multi.close()
    rw = orc.fill_normal(E * H, seed, O.stream_id(0, O.KIND_ROUTER), 0.02).reshape(E, H)
    logits, _, _, ti = orc.router(x, rw, K, bias=bias)
    assert np.array_equal(got["logits"], logits)
    w = O.synth_layer_f32(orc, seed, 0, H, I, E, wt, experts=np.unique(ti))
    o = orc.moe_forward(x, *w, K, I, bias=bias)
    bad, _ = topk_mismatches(got["idx"], o["idx"], logits, K)
    assert bad == 0
    assert rel_l2(got["out"], o["out"]) <= REL_L2_TOL


def test_near_tie_falls_back_to_the_router_chains(orc):
    """A router bias that puts the K-th and (K+1)-th logits of every token 1e-6 apart: the
    one-kernel path's certified pass cannot decide those selections, so the plan comes from
    the bit-exact chains; results still equal the multi-kernel path's bits.  A second call
    without the bias (every token certified) gives the multi-kernel bits too."""
    H, I, E, K, wt, T, seed = 512, 256, 64, 8, O.Q8_0, 1, 441
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    x = O.synth_x(orc, seed, T, H)
    logits = orc.router(x, lay["router"], K)[0][0].astype(np.float64)
    order = np.argsort(-logits, kind="stable")
    bias = np.zeros(E, np.float32)
    bias[order[K]] = np.float32(logits[order[K - 1]] - logits[order[K]] - 1e-6)
    fused, multi = _pair(H, I, E, K, T)
    for m in (fused, multi):
        _load(m, lay, wt)
    _same(fused.forward_host(0, x, bias=bias, debug=True), multi.forward_host(0, x, bias=bias, debug=True))
    _same(fused.forward_host(0, x, debug=True), multi.forward_host(0, x, debug=True))
    fused.close()
    multi.close()
