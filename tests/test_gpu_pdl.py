"""GPU tests of programmatic dependent launch in the decode chains (1..64 tokens on one GPU).

A context created with HYMOE_PDL=1 (the default) launches the router, top-K, plan, scatter,
both weight streams and the combine with the programmatic-serialisation attribute, each kernel
waiting for its predecessor before it reads that predecessor's output; HYMOE_PDL=0 launches
them the ordinary way.  The arithmetic is the same, so every logit, selection, weight and
output must be bit-identical between the two, eagerly and under graph replay, and repeated
calls must not see a previous call's rows.  Oracle agreement of this path is covered by the
parity tests (same kernels).
"""
import os

import numpy as np
import pytest

import hymoe
import oracle as O
from moe_cases import host_layer

pytestmark = pytest.mark.gpu


def _ctx(pdl, H, I, E, K, T):
    old = os.environ.get("HYMOE_PDL")
    os.environ["HYMOE_PDL"] = pdl
    try:
        return hymoe.MoE(H, I, E, K, 1, max(T, 16))
    finally:
        if old is None:
            del os.environ["HYMOE_PDL"]
        else:
            os.environ["HYMOE_PDL"] = old


@pytest.mark.parametrize("wt,T,pre_norm", [(O.Q8_0, 1, False), (O.Q4_0, 3, True), (O.Q8_0, 8, False),
                                           (O.Q4_0, 13, False), (O.Q8_0, 40, True), (O.Q4_0, 64, False)])
def test_programmatic_launch_gives_the_ordinary_launch_bits(orc, wt, T, pre_norm):
    H, I, E, K = 512, 256, 64, 8
    seed = 500 + T
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    bias = O.synth_bias(orc, seed, E)
    on, off = _ctx("1", H, I, E, K, T), _ctx("0", H, I, E, K, T)
    for m in (on, off):
        m.load_layer(0, lay["router"], lay["sgu"], lay["sdn"], lay["egu"], lay["edn"], wt)
        if pre_norm:
            w = (1.0 + 0.1 * np.random.default_rng(seed).standard_normal(H)).astype(np.float32)
            m.set_norm(0, w, 1e-5)
    for call in range(3):
        x = O.synth_x(orc, seed + call, T, H)
        a = on.forward_host(0, x, resid="x", bias=bias, debug=True, pre_norm=pre_norm)
        b = off.forward_host(0, x, resid="x", bias=bias, debug=True, pre_norm=pre_norm)
        for k in ("logits", "probs", "w", "idx", "out"):
            assert np.array_equal(a[k], b[k]), (call, k)
    on.close()
    off.close()


def test_programmatic_launch_under_graph_replay(orc):
    """Device calls of 1, 8 and 40 tokens replayed from CUDA graphs on a side stream: the
    programmatic edges captured in the graph give the ordinary launches' bits."""
    torch = pytest.importorskip("torch")
    H, I, E, K, wt, seed = 512, 256, 64, 8, O.Q8_0, 611
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    on, off = _ctx("1", H, I, E, K, 64), _ctx("0", H, I, E, K, 64)
    for m in (on, off):
        m.load_layer(0, lay["router"], lay["sgu"], lay["sdn"], lay["egu"], lay["edn"], wt)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        on.set_stream(st.cuda_stream)
        for call in range(12):
            T = (1, 8, 40)[call % 3]
            x = O.synth_x(orc, seed + call, T, H)
            want = off.forward_host(0, x, resid="x")["out"]
            xd = torch.from_numpy(x).cuda()
            od = torch.empty_like(xd)
            on.forward_device(0, xd.data_ptr(), od.data_ptr(), T, resid_ptr=xd.data_ptr(), graph=True)
            on.synchronize()
            assert np.array_equal(od.cpu().numpy(), want), f"call {call}"
    on.close()
    off.close()
