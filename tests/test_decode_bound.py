"""CPU check of the bound the one-kernel decode path uses to certify a routing selection before
the bit-exact router chains finish (csrc/decode.cu, "certified routing").

The router logit is the reference's sequential fp32 chain acc = fl(acc + fl(x_k * w_k)) over k
(src/attention.cpp:213-222).  From the same rounded products p_k the kernel computes in fp64 the
sum L, P = sum |p_k| and S = sum_k |prefix_k|, and bounds the chain by
    |chain - L| <= u/(1-u) * (S + H * gamma_H * P) (+ fp64 slack),  u = 2^-24.
Here the chain is run exactly as the reference does (numpy's add.accumulate is sequential in
float32) on seeded inputs of many scales, with heavy cancellation and with a large constant
offset, and the bound must hold every time; it must also be far tighter than the worst case
gamma_H * P, which is what makes the certification succeed for almost every token.
"""
import numpy as np

U = 2.0 ** -24


def chain_and_bound(x, w):
    p = (x.astype(np.float32) * w.astype(np.float32)).astype(np.float32)  # each product rounded
    chain = np.add.accumulate(p, dtype=np.float32)[-1]
    pd = p.astype(np.float64)
    L = pd.sum()
    P = np.abs(pd).sum()
    S = np.abs(np.cumsum(pd)).sum()
    H = len(p)
    gH = H * U / (1.0 - H * U)
    bound = U / (1.0 - U) * (S + H * gH * P) + 1e-9 * (P + abs(L))
    return float(chain), L, bound, gH * P


def test_chain_bound_holds_on_seeded_inputs():
    rng = np.random.default_rng(2026)
    worst = 0.0
    for case in range(300):
        H = int(rng.choice([256, 512, 4096]))
        scale = 10.0 ** rng.uniform(-4, 4)
        x = (rng.standard_normal(H) * scale).astype(np.float32)
        w = (rng.standard_normal(H) * 0.02).astype(np.float32)
        if case % 3 == 1:  # heavy cancellation: pairs of opposite products
            x[1::2] = -x[0::2][: H // 2]
            w[1::2] = w[0::2][: H // 2]
        if case % 3 == 2:  # a large offset the chain carries along
            x[0] = np.float32(1e4 * scale)
            w[0] = np.float32(1.0)
        chain, L, bound, crude = chain_and_bound(x, w)
        err = abs(chain - L)
        assert err <= bound, (case, err, bound)
        worst = max(worst, err / bound if bound else 0.0)
        if case % 3 == 0:  # random inputs: the running-sum bound is far tighter than gamma_H * P
            assert bound < crude / 5, (case, bound, crude)
    assert worst > 0.0


def test_bound_is_zero_slack_only_for_exact_sums():
    # products that are small integers add exactly in fp32: the chain equals the fp64 sum
    x = np.arange(1, 129, dtype=np.float32)
    w = np.ones(128, np.float32)
    chain, L, bound, _ = chain_and_bound(x, w)
    assert chain == L
    assert bound >= 0.0
