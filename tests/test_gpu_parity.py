"""GPU parity tests: the CUDA path through the C ABI against the reference's golden
fixtures and the oracle, on the same seeded inputs.

Tolerances (north star): selected experts equal wherever the K-th/(K+1)-th logit gap
exceeds 1e-4; output relative L2 error <= 1e-3.  The router logits are additionally
required to be bit-identical to the reference (the kernel performs the reference's
sequential multiply-add chain).
"""
import numpy as np
import pytest

import hymoe
import oracle as O
from moe_cases import (FULL_FIXTURES, REL_L2_TOL, SMALL_FIXTURES, host_layer, load_fixture,
                       rel_l2, topk_mismatches)

pytestmark = pytest.mark.gpu


def _ctx(H, I, E, K, T, layers=1):
    return hymoe.MoE(H, I, E, K, layers, max(T, 16))


def _load(m, lay, wt, layer=0):
    m.load_layer(layer, lay["router"], lay["sgu"], lay["sdn"], lay["egu"], lay["edn"], wt)


def _oracle(orc, lay, x, K, I, bias=None, resid=None):
    return orc.moe_forward(x, lay["router"], lay["sgu_f"], lay["sdn_f"], lay["egu_f"],
                           lay["edn_f"], K, I, bias=bias, resid=resid)


def _check(r, ref_out, ref_idx, logits, K, tol=REL_L2_TOL):
    bad, _ = topk_mismatches(r["idx"], ref_idx, logits, K)
    assert bad == 0, f"{bad} tokens select different experts"
    err = rel_l2(r["out"], ref_out)
    assert err <= tol, f"rel L2 {err:.3e} > {tol}"
    return err


@pytest.mark.parametrize("name", SMALL_FIXTURES)
def test_small_shapes_vs_reference_golden(orc, name):
    fx = load_fixture(name)
    H, I, E, K, T, wt, seed = (fx[k] for k in ("H", "I", "E", "K", "T", "wt", "seed"))
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    x = O.synth_x(orc, seed, T, H)
    m = _ctx(H, I, E, K, T)
    _load(m, lay, wt)
    r = m.forward_host(0, x, debug=True)
    logits = orc.router(x, lay["router"], K)[0]
    assert np.array_equal(r["logits"], logits)
    np.testing.assert_allclose(r["probs"], fx["probs"], rtol=2e-6, atol=1e-9)
    _check(r, fx["out"], fx["idx"], logits, K)
    same = (r["idx"] == fx["idx"]).all(axis=1)
    np.testing.assert_allclose(r["w"][same], fx["w"][same], rtol=2e-6)
    m.close()


@pytest.mark.parametrize("name", FULL_FIXTURES)
def test_full_shape_vs_reference_golden_device_weights(orc, name):
    """Weights generated on the device (hymoe_synth_layer); the golden output came from
    the reference on host-generated weights, so this also pins the device generator."""
    fx = load_fixture(name)
    H, I, E, K, T, wt, seed = (fx[k] for k in ("H", "I", "E", "K", "T", "wt", "seed"))
    m = _ctx(H, I, E, K, T)
    m.synth_layer(0, wt, seed, 0.02)
    x = O.synth_x(orc, seed, T, H)
    r = m.forward_host(0, x, debug=True)
    rw = orc.fill_normal(E * H, seed, O.stream_id(0, O.KIND_ROUTER), 0.02).reshape(E, H)
    logits = orc.router(x, rw, K)[0]
    assert np.array_equal(r["logits"], logits)
    _check(r, fx["out"], fx["idx"], logits, K)
    m.close()


@pytest.mark.parametrize("wt", [O.Q4_0, O.Q8_0])
@pytest.mark.parametrize("T", [1, 3, 8, 9, 16, 24, 33, 64, 65, 257, 600])
def test_token_counts_vs_oracle(orc, wt, T):
    """Decode (weight-streaming kernel, T <= 64: activation boxes of 8/16/32/64 rows) and
    tensor-core paths (T > 64), single and multiple token tiles per expert, ragged tails."""
    H, I, E, K, seed = 512, 256, 64, 8, 21
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    x = O.synth_x(orc, seed + T, T, H)
    m = _ctx(H, I, E, K, T)
    _load(m, lay, wt)
    r = m.forward_host(0, x, debug=True)
    o = _oracle(orc, lay, x, K, I)
    assert np.array_equal(r["logits"], o["logits"])
    _check(r, o["out"], o["idx"], o["logits"], K)
    m.close()


@pytest.mark.parametrize("kind", ["normal", "zipf"])
def test_router_bias_and_residual_vs_oracle(orc, kind):
    H, I, E, K, T, seed, wt = 512, 256, 64, 8, 300, 5, O.Q4_0
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    x = O.synth_x(orc, seed, T, H)
    resid = O.synth_x(orc, seed + 1, T, H)
    bias = O.synth_bias(orc, seed, E) if kind == "normal" else O.zipf_bias(seed, E)
    m = _ctx(H, I, E, K, T)
    _load(m, lay, wt)
    r = m.forward_host(0, x, resid=resid, bias=bias, debug=True)
    o = _oracle(orc, lay, x, K, I, bias=bias, resid=resid)
    assert np.array_equal(r["logits"], o["logits"])
    _check(r, o["out"], o["idx"], o["logits"], K)
    m.close()


def test_full_shape_prefill_vs_oracle(orc):
    """Full HunyuanImage-3 shapes through the tensor-core path, Q4_0, router bias."""
    H, I, E, K, T, seed, wt = 4096, 3072, 64, 8, 24, 7, O.Q4_0
    m = _ctx(H, I, E, K, T)
    m.synth_layer(0, wt, seed, 0.02)
    x = O.synth_x(orc, seed, T, H)
    bias = O.synth_bias(orc, seed, E)
    r = m.forward_host(0, x, bias=bias, debug=True)
    rw = orc.fill_normal(E * H, seed, O.stream_id(0, O.KIND_ROUTER), 0.02).reshape(E, H)
    logits, _, _, ti = orc.router(x, rw, K, bias=bias)
    assert np.array_equal(r["logits"], logits)
    _, sgu, sdn, egu, edn = O.synth_layer_f32(orc, seed, 0, H, I, E, wt, experts=np.unique(ti))
    o = orc.moe_forward(x, rw, sgu, sdn, egu, edn, K, I, bias=bias)
    _check(r, o["out"], o["idx"], logits, K)
    m.close()


def test_device_pointers_and_aliased_residual(orc):
    torch = pytest.importorskip("torch")
    H, I, E, K, T, seed, wt = 512, 256, 64, 8, 40, 9, O.Q8_0
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    x = O.synth_x(orc, seed, T, H)
    resid = O.synth_x(orc, seed + 1, T, H)
    m = _ctx(H, I, E, K, T)
    _load(m, lay, wt)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        xd = torch.from_numpy(x).cuda()
        rd = torch.from_numpy(resid).cuda()
        m.set_stream(st.cuda_stream)
        m.forward_device(0, xd.data_ptr(), rd.data_ptr(), T, resid_ptr=rd.data_ptr())  # in place
    m.synchronize()
    o = _oracle(orc, lay, x, K, I, resid=resid)
    assert rel_l2(rd.cpu().numpy(), o["out"]) <= REL_L2_TOL
    host = m.forward_host(0, x, resid=resid)["out"]
    assert np.array_equal(host, rd.cpu().numpy())  # same kernels, same bits
    m.close()


def test_deterministic_and_empty(orc):
    H, I, E, K, T, seed, wt = 256, 128, 16, 8, 77, 3, O.Q4_0
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    x = O.synth_x(orc, seed, T, H)
    m = _ctx(H, I, E, K, T)
    _load(m, lay, wt)
    a = m.forward_host(0, x)["out"]
    b = m.forward_host(0, x)["out"]
    assert np.array_equal(a, b)
    e = m.forward_host(0, np.zeros((0, H), np.float32))["out"]
    assert e.shape == (0, H)
    with pytest.raises(hymoe.HymoeError):
        m.forward_host(0, np.zeros((T + 1, H), np.float32))  # above max_tokens
    m.close()


def test_errors_are_statuses(orc):
    m = _ctx(256, 128, 16, 8, 8)
    with pytest.raises(hymoe.HymoeError) as ei:
        m.forward_host(0, np.zeros((4, 256), np.float32))
    assert ei.value.status == 7  # layer not loaded
    with pytest.raises(hymoe.HymoeError) as ei:
        m.forward_host(0, np.zeros((17, 256), np.float32))
    assert ei.value.status in (1, 7)
    m.close()


@pytest.mark.parametrize("T", [3, 6, 40])
def test_graph_replay_matches_eager(orc, T):
    """HYMOE_USE_GRAPH: the captured graph reads the buffers' current contents on every
    replay, giving the same bits as the eager call."""
    torch = pytest.importorskip("torch")
    H, I, E, K, seed, wt = 512, 256, 64, 8, 17, O.Q8_0
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    m = _ctx(H, I, E, K, T)
    _load(m, lay, wt)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        m.set_stream(st.cuda_stream)
        xd = torch.empty(T, H, device="cuda")
        od = torch.empty_like(xd)
        for call in range(3):
            x = O.synth_x(orc, seed + call, T, H)
            xd.copy_(torch.from_numpy(x))
            m.forward_device(0, xd.data_ptr(), od.data_ptr(), T, graph=True)
            m.synchronize()
            got = od.cpu().numpy()
            eager = m.forward_host(0, x)["out"]
            assert np.array_equal(got, eager), f"call {call}"
    m.close()


def test_host_pointer_call_in_chunks_is_bit_identical(orc):
    """Host-pointer calls of >= 2048 tokens run as pipelined token chunks (copies on a second
    stream beside the compute); the output must equal one device-pointer call bit for bit."""
    torch = pytest.importorskip("torch")
    H, I, E, K, T, seed, wt = 256, 128, 16, 8, 6149, 17, O.Q4_0  # 3 chunks, the last one shorter
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    x = O.synth_x(orc, seed, T, H)
    resid = O.synth_x(orc, seed + 1, T, H)
    bias = O.synth_bias(orc, seed, E)
    m = _ctx(H, I, E, K, T)
    _load(m, lay, wt)
    host = m.forward_host(0, x, resid=resid, bias=bias)["out"]
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        xd, rd = torch.from_numpy(x).cuda(), torch.from_numpy(resid).cuda()
        bd, od = torch.from_numpy(bias).cuda(), torch.empty(T, H, device="cuda")
        m.set_stream(st.cuda_stream)
        m.forward_device(0, xd.data_ptr(), od.data_ptr(), T, resid_ptr=rd.data_ptr(), bias_ptr=bd.data_ptr())
    m.synchronize()
    assert np.array_equal(host, od.cpu().numpy())
    o = _oracle(orc, lay, x, K, I, bias=bias, resid=resid)
    assert rel_l2(host, o["out"]) <= REL_L2_TOL
    m.close()


def test_expert_placement_keeps_outputs_and_expert_ids(orc):
    """hymoe_set_placement: the same layer loaded under a permuted placement gives the same
    bits (outputs, weights) and the same expert ids in the debug indices, on every path
    (fused top-K + plan at T <= 16, the decode kernels, the tensor-core GEMM); a placement
    marks the layer unloaded; a non-permutation is refused."""
    H, I, E, K, seed, wt = 512, 256, 64, 8, 23, O.Q4_0
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    m = _ctx(H, I, E, K, 300)
    _load(m, lay, wt)
    bias = O.zipf_bias(seed, E)
    xs = {T: O.synth_x(orc, seed + T, T, H) for T in (5, 40, 300)}
    ref = {T: m.forward_host(0, x, bias=bias, debug=True) for T, x in xs.items()}
    perm = list(np.random.default_rng(9).permutation(E))
    m.set_placement(0, perm)
    with pytest.raises(hymoe.HymoeError) as ei:
        m.forward_host(0, xs[5])
    assert ei.value.status == 7  # load again after a placement
    _load(m, lay, wt)
    for T, x in xs.items():
        got = m.forward_host(0, x, bias=bias, debug=True)
        assert np.array_equal(got["idx"], ref[T]["idx"]), T
        assert np.array_equal(got["w"], ref[T]["w"]), T
        assert np.array_equal(got["out"], ref[T]["out"]), T
    with pytest.raises(hymoe.HymoeError):
        m.set_placement(0, [0] * E)
    m.set_placement(0, None)
    _load(m, lay, wt)
    assert np.array_equal(m.forward_host(0, xs[40], bias=bias)["out"], ref[40]["out"])
    m.close()


@pytest.mark.parametrize("router_type", [O.F32, O.Q8_0])
def test_load_layer_from_gguf_file_matches_load_layer(orc, tmp_path, router_type):
    """hymoe_load_layer_gguf: a layer written under the reference converter's names gives
    the same bits as hymoe_load_layer of the same blocks.  A router stored as Q8_0 is decoded
    on the host with the standard rule (gguf-py's dequantize)."""
    gguf = pytest.importorskip("gguf")
    from gguf_layer import write_moe_layer
    H, I, E, K, seed, wt = 512, 256, 64, 8, 29, O.Q4_0
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    path = str(tmp_path / "layer7.gguf")
    write_moe_layer(path, 7, H, I, lay["router"], lay["sgu"], lay["sdn"], lay["egu"], lay["edn"], wt,
                    router_type=router_type)
    router = lay["router"]
    if router_type != O.F32:
        qt = gguf.GGMLQuantizationType(router_type)
        router = gguf.quants.dequantize(gguf.quants.quantize(router, qt), qt).astype(np.float32)
    x = O.synth_x(orc, seed, 200, H)
    ref = hymoe.MoE(H, I, E, K, 1, 200)
    ref.load_layer(0, router, lay["sgu"], lay["sdn"], lay["egu"], lay["edn"], wt)
    want = ref.forward_host(0, x, debug=True)
    ref.close()
    m = hymoe.MoE(H, I, E, K, 2, 200)
    with hymoe.GGUF(path) as f:
        m.load_layer_gguf(1, f, 7)
        with pytest.raises(hymoe.HymoeError):
            m.load_layer_gguf(0, f, 6)  # no such layer in the file
    got = m.forward_host(1, x, debug=True)
    assert np.array_equal(got["logits"], want["logits"])
    assert np.array_equal(got["out"], want["out"])
    m.close()


@pytest.mark.parametrize("T", [1, 5, 40, 300])
def test_pre_norm_is_the_reference_rms_norm_then_the_block(orc, T):
    """HYMOE_PRE_NORM with residual = x is decoder_layer's out = h + moe(rms_norm(h))
    (src/decoder_layer.cpp:34-42).  The device RMSNorm keeps the reference's rounding, so the
    call gives the same bits (logits, routing, output) as the block run on the oracle's
    rms_norm (itself pinned bit-exactly to the reference's rms_norm_f32 on the CPU)."""
    H, I, E, K, seed, wt = 512, 256, 64, 8, 31, O.Q4_0
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    m = _ctx(H, I, E, K, T)
    _load(m, lay, wt)
    rng = np.random.default_rng(T)
    h = (O.synth_x(orc, seed + T, T, H) * 10.0 ** rng.integers(-3, 3, size=(T, 1))).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    eps = 1e-5
    with pytest.raises(hymoe.HymoeError) as ei:
        m.forward_host(0, h, pre_norm=True)
    assert ei.value.status == 7  # no RMSNorm weights yet
    m.set_norm(0, w, eps)
    xn = orc.rms_norm(h, w, eps)
    want = m.forward_host(0, xn, resid=h, debug=True)
    got = m.forward_host(0, h, resid="x", debug=True, pre_norm=True)
    for k in ("logits", "idx", "w", "out"):
        assert np.array_equal(got[k], want[k]), k
    o = _oracle(orc, lay, xn, K, I, resid=h)
    assert rel_l2(got["out"], o["out"]) <= REL_L2_TOL
    m.close()


def test_pre_norm_chunked_host_call_and_graph_replay(orc):
    """The pipelined host-pointer call (>= 2048 tokens, x uploaded once as its own residual)
    and a replayed CUDA graph give the same bits as the eager device call."""
    torch = pytest.importorskip("torch")
    H, I, E, K, seed, wt = 512, 256, 64, 8, 37, O.Q8_0
    T = 4200
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    m = _ctx(H, I, E, K, T)
    _load(m, lay, wt)
    rng = np.random.default_rng(3)
    w = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    m.set_norm(0, w, 1e-6)
    h = O.synth_x(orc, seed, T, H)
    host = m.forward_host(0, h, resid="x", pre_norm=True)["out"]
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        m.set_stream(st.cuda_stream)
        xd = torch.from_numpy(h).cuda()
        od = torch.empty_like(xd)
        m.forward_device(0, xd.data_ptr(), od.data_ptr(), T, resid_ptr=xd.data_ptr(), pre_norm=True)
        m.synchronize()
        assert np.array_equal(od.cpu().numpy(), host)
        t = 6
        xs = torch.empty(t, H, device="cuda")
        os_ = torch.empty_like(xs)
        for call in range(3):
            xs.copy_(torch.from_numpy(O.synth_x(orc, seed + call, t, H)))
            m.forward_device(0, xs.data_ptr(), os_.data_ptr(), t, resid_ptr=xs.data_ptr(), graph=True,
                             pre_norm=True)
            m.synchronize()
            eager = m.forward_host(0, xs.cpu().numpy(), resid="x", pre_norm=True)["out"]
            assert np.array_equal(os_.cpu().numpy(), eager), f"call {call}"
    m.close()


def test_layer_stack_in_place_matches_the_oracle(orc):
    """The cfg5 recurrence x <- x + MoE_l(RMSNorm_l(x)) over 4 layers, in place on the device
    (x, residual and out one buffer, HYMOE_PRE_NORM): every layer gives the bits of the same
    call with separate buffers, and the stack stays within the parity tolerance of the
    oracle's recurrence."""
    torch = pytest.importorskip("torch")
    H, I, E, K, T, L, wt, seed = 512, 256, 64, 8, 40, 4, O.Q4_0, 51
    lays = [host_layer(orc, seed, l, H, I, E, wt) for l in range(L)]
    rng = np.random.default_rng(seed)
    ws = [(1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32) for _ in range(L)]
    m = _ctx(H, I, E, K, T, layers=L)
    for l in range(L):
        _load(m, lays[l], wt, layer=l)
        m.set_norm(l, ws[l], 1e-5)
    x0 = O.synth_x(orc, seed, T, H)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        m.set_stream(st.cuda_stream)
        xd = torch.from_numpy(x0).cuda()
        for l in range(L):
            sep_in = xd.clone()
            sep_out = torch.empty_like(xd)
            m.forward_device(l, sep_in.data_ptr(), sep_out.data_ptr(), T, resid_ptr=sep_in.data_ptr(),
                             pre_norm=True)
            m.forward_device(l, xd.data_ptr(), xd.data_ptr(), T, resid_ptr=xd.data_ptr(), pre_norm=True)
            m.synchronize()
            assert torch.equal(xd, sep_out), f"layer {l}"
        got = xd.cpu().numpy()
    m.close()
    x = x0.copy()
    for l in range(L):
        x = _oracle(orc, lays[l], orc.rms_norm(x, ws[l], 1e-5), K, I, resid=x)["out"]
    assert rel_l2(got, x) <= REL_L2_TOL


def _block_with_routing(orc, lay, x, idx, w, I):
    """shared(x) + sum_k w[t,k] * expert_{idx[t,k]}(x[t]) through the oracle's FFN."""
    out = orc.swiglu_ffn(x, lay["sgu_f"], lay["sdn_f"], I).astype(np.float64)
    for e in np.unique(idx):
        rows = np.nonzero((idx == e).any(axis=1))[0]
        y = orc.swiglu_ffn(np.ascontiguousarray(x[rows]), lay["egu_f"][e], lay["edn_f"][e], I)
        wk = np.where(idx[rows] == e, w[rows], 0).sum(axis=1)
        out[rows] += wk[:, None] * y
    return out.astype(np.float32)


@pytest.mark.parametrize("opts", [{"group": (8, 3)}, {"norm_topk_prob": False, "scale": 2.5},
                                  {"group": (4, 1), "norm_topk_prob": False, "scale": 0.7}])
@pytest.mark.parametrize("T", [5, 40, 300])
def test_full_mode_routing_variants_vs_oracle(orc, opts, T):
    """hymoe_set_routing (group-limited greedy, unnormalised scaling) against the oracle's
    topkgating_full on the GPU's own logits (bit-identical to the reference's): same experts in
    the same rank order (a difference only where two probabilities lie within 1e-6 of each
    other, expf's last place), same weights within 1e-5; the output equals the block under
    that routing within the parity tolerance; the plain routing comes back bit-identical."""
    H, I, E, K, seed, wt = 512, 256, 64, 8, 61, O.Q4_0
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    m = _ctx(H, I, E, K, T)
    _load(m, lay, wt)
    x = O.synth_x(orc, seed + T, T, H)
    plain = m.forward_host(0, x)["out"]
    m.set_routing(**opts)
    r = m.forward_host(0, x, debug=True)
    a = orc.topkgating_full(r["logits"], K, **opts)
    np.testing.assert_allclose(r["probs"], a["probs"], rtol=1e-6, atol=1e-12)
    for t in range(T):
        if not np.array_equal(r["idx"][t], a["idx"][t]):
            diff = set(r["idx"][t]) ^ set(a["idx"][t])
            kth = a["probs"][t, a["idx"][t]].min()
            assert all(abs(a["probs"][t, e] - kth) <= 1e-6 * kth for e in diff), f"token {t}"
        else:
            np.testing.assert_allclose(r["w"][t], a["w"][t], rtol=1e-5)
    ref = _block_with_routing(orc, lay, x, r["idx"], r["w"], I)
    assert rel_l2(r["out"], ref) <= REL_L2_TOL
    m.set_routing(plain=True)
    assert np.array_equal(m.forward_host(0, x)["out"], plain)
    m.close()


@pytest.mark.parametrize("opts", [{"drop": 1.0}, {"drop": 0.5, "group": (8, 3)},
                                  {"drop": 1.25, "min_capacity": 4, "norm_topk_prob": False, "scale": 1.5}])
@pytest.mark.parametrize("T", [5, 17, 300, 700])
def test_capacity_drops_vs_oracle(orc, opts, T):
    """hymoe_set_routing with drop_tokens: the capacity floor(cf * K * T / E) (at least K and
    min_capacity), each expert's first pairs in k-major order kept, the others dropped — the
    same pairs as the oracle's topkgating_full (pinned to the reference's), their debug weight
    0, their rows out of the GEMMs; the output equals the block over the kept pairs.  T = 5 and
    17 run the decode kernels (17: more than one router chunk), 300 and 700 the tensor cores."""
    H, I, E, K, seed, wt = 512, 256, 64, 8, 67, O.Q4_0
    lay = host_layer(orc, seed, 0, H, I, E, wt)
    m = _ctx(H, I, E, K, T)
    _load(m, lay, wt)
    x = O.synth_x(orc, seed + T, T, H)
    bias = O.zipf_bias(seed, E)  # skewed load: hot experts overflow their capacity
    m.set_routing(**opts)
    r = m.forward_host(0, x, bias=bias, debug=True)
    a = orc.topkgating_full(r["logits"], K, **opts)
    assert np.array_equal(r["idx"], a["idx"])
    np.testing.assert_allclose(r["w"], a["w"] * a["keep"], rtol=1e-5, atol=0)
    assert np.array_equal(r["w"] == 0, ~a["keep"])
    if T >= 300 and opts["drop"] <= 1.0:
        assert (~a["keep"]).any()  # the case really drops pairs
    ref = _block_with_routing(orc, lay, x, r["idx"], r["w"], I)
    assert rel_l2(r["out"], ref) <= REL_L2_TOL
    m.set_routing(plain=True)
    assert (m.forward_host(0, x, bias=bias, debug=True)["w"] > 0).all()
    m.close()


@pytest.mark.parametrize("H,I,E,K,wt,Ts", [(256, 128, 8, 1, O.Q4_0, (1, 7, 100)),
                                             (384, 192, 16, 2, O.Q8_0, (3, 70)),
                                             (256, 128, 32, 6, O.Q4_0, (1, 33, 130))])
def test_other_expert_counts_and_top_k_vs_oracle(orc, H, I, E, K, wt, Ts):
    """Expert counts 8/16/32 with K = 1/2/6 on the decode and tensor-core paths: logits
    bit-identical, experts equal outside near ties, output within the parity tolerance."""
    lay = host_layer(orc, 71 + E, 0, H, I, E, wt)
    m = _ctx(H, I, E, K, max(Ts))
    _load(m, lay, wt)
    for T in Ts:
        x = O.synth_x(orc, 71 + T, T, H)
        r = m.forward_host(0, x, debug=True)
        o = _oracle(orc, lay, x, K, I)
        assert np.array_equal(r["logits"], o["logits"]), T
        _check(r, o["out"], o["idx"], o["logits"], K)
    m.close()
