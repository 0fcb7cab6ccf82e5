"""GPU parity at the benchmark shapes (H=4096, I=3072, E=64, K=8) on the tensor-core path.

Every call here has more than 64 tokens, so the grouped tcgen05 GEMM (not the decode
kernels) computes gate_up and down, with the same per-expert raggedness, K-stage count and
row-block pairs as the benchmark.  The GPU runs all T tokens in one call.  Checked against
the oracle (the C restatement, itself bit-identical to the reference's moe_forward_cpu,
src/attention.cpp:191-313):
  - the router logits of all T tokens, bit for bit (pre-softmax, with the bias);
  - the selected experts of all T tokens, equal wherever the K-th/(K+1)-th logit gap
    exceeds 1e-4;
  - the output of a seeded sample of 32 tokens within relative L2 1e-3.  moe_forward_cpu
    treats every token independently (src/attention.cpp:246-309: no capacity, no cross-token
    state), so the oracle's rows for the sample are exactly the rows of a full-T run.
Weights come from the device generator (hymoe_synth_layer), which is byte-identical to the
oracle's host generator.
"""
import numpy as np
import pytest

import hymoe
import oracle as O
from moe_cases import GAP_TOL, REL_L2_TOL, rel_l2, topk_mismatches

pytestmark = pytest.mark.gpu

H, I, E, K = 4096, 3072, 64, 8
SAMPLE = 32

CASES = {
    # BASELINE cfg3: Q4_0 prefill, 4096 tokens, router bias ~N(0, 0.5)
    "cfg3_q4_0_t4096_bias": (O.Q4_0, 4096, "normal", 101),
    # BASELINE cfg1: F32 weights (stored as F16 tiles), 256 tokens, no bias
    "cfg1_f32_t256": (O.F32, 256, None, 0),
    # a ragged token count: partial token tiles in every expert, Q8_0
    "ragged_q8_0_t1000": (O.Q8_0, 1000, None, 103),
    # cfg4's token count on one GPU with its Zipf(1.1) skew: hot experts of >1000 rows
    "cfg4_q4_0_t8192_zipf": (O.Q4_0, 8192, "zipf", 104),
    # the smallest call that takes the tensor-core path, F16 weights
    "f16_t65": (O.F16, 65, None, 105),
}


@pytest.mark.parametrize("case", list(CASES))
def test_headline_shape_tensor_core_vs_oracle(orc, case):
    wt, T, bias_kind, seed = CASES[case]
    bias = None
    if bias_kind == "normal":
        bias = O.synth_bias(orc, seed, E)
    elif bias_kind == "zipf":
        bias = O.zipf_bias(seed, E)
    m = hymoe.MoE(H, I, E, K, 1, T)
    m.synth_layer(0, wt, seed, 0.02)
    x = O.synth_x(orc, seed, T, H)
    r = m.forward_host(0, x, bias=bias, debug=True)  # one call over all T tokens
    m.close()

    rw = orc.fill_normal(E * H, seed, O.stream_id(0, O.KIND_ROUTER), 0.02).reshape(E, H)
    logits, probs, tw, ti = orc.router(x, rw, K, bias=bias)
    assert np.array_equal(r["logits"], logits), "router logits differ from the reference chain"
    bad, ties = topk_mismatches(r["idx"], ti, logits, K)
    assert bad == 0, f"{bad} of {T} tokens select different experts (gap > {GAP_TOL})"
    same = (r["idx"] == ti).all(axis=1)
    np.testing.assert_allclose(r["w"][same], tw[same], rtol=2e-6)

    sample = np.sort(np.random.default_rng(seed).choice(T, size=min(SAMPLE, T), replace=False))
    xs = np.ascontiguousarray(x[sample])
    w = O.synth_layer_f32(orc, seed, 0, H, I, E, wt, experts=np.unique(ti[sample]))
    o = orc.moe_forward(xs, *w, K, I, bias=bias)
    assert np.array_equal(o["idx"], ti[sample])
    err = rel_l2(r["out"][sample], o["out"])
    assert err <= REL_L2_TOL, f"{case}: rel L2 {err:.3e} over {len(sample)} sampled tokens"
