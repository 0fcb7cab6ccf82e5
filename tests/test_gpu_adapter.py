"""GPU tests of the drop-in at the reference's own call site.

oracle/_ref/libhyref_gpu.so holds the reference's unmodified src/decoder_layer.cpp compiled
twice: as written (MoE = moe_forward_cpu), and with its MoE call (src/decoder_layer.cpp:38)
bound at compile time to the C++ adapter hymoe_moe_forward_cpu, which runs the MoE on the GPU
through libhymoe.so.  Both layers run on the same weights and inputs; the GPU MoE must agree
within the parity tolerance and select the same experts.  Skipped when the checker was not
built (it needs the reference sources at build time).
"""
import ctypes as C
import os

import numpy as np
import pytest

import oracle as O
from moe_cases import REL_L2_TOL, rel_l2, topk_mismatches

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(O.__file__), "_ref", "libhyref_gpu.so")
_fp = C.POINTER(C.c_float)


def _lib():
    L = C.CDLL(LIB)
    u32 = C.c_uint32
    L.hyref_layer_create.restype = C.c_void_p
    L.hyref_layer_create.argtypes = [u32, u32, u32] + [_fp] * 9 + [C.POINTER(_fp), C.POINTER(_fp)]
    L.hyref_layer_destroy.argtypes = [C.c_void_p]
    L.hyref_layer_forward.argtypes = [_fp, C.c_void_p, u32, u32, u32, u32, C.c_int, _fp]
    L.hyref_moe_forward.argtypes = [_fp, C.c_void_p, u32, u32, u32, u32, C.c_int, _fp, _fp, _fp,
                                    C.POINTER(C.c_int32)]
    L.hyref_layer_reload_moe.argtypes = [C.c_void_p, u32, u32, u32, _fp, _fp, _fp, C.POINTER(_fp),
                                         C.POINTER(_fp), C.c_int]
    return L


def _p(a):
    return a.ctypes.data_as(_fp)


@pytest.fixture(scope="module")
def layer(orc):
    if not os.path.exists(LIB):
        pytest.skip("integration checker not built (needs the reference sources)")
    H, I, E, K, seed = 256, 128, 16, 8, 13
    L = _lib()
    rw, sgu, sdn, egu, edn = O.synth_layer_f32(orc, seed, 0, H, I, E, O.F32)
    n = lambda cnt, s, std: orc.fill_normal(cnt, seed, O.stream_id(7, 6, s), std)
    in_ln = 1.0 + n(H, 0, 0.1)
    post_ln = 1.0 + n(H, 1, 0.1)
    qkv = n(6144 * H, 2, 0.02)
    o = n(H * 4096, 3, 0.02)
    qn = 1.0 + n(128, 4, 0.1)
    kn = 1.0 + n(128, 5, 0.1)
    keep = (rw, sgu, sdn, egu, edn, in_ln, post_ln, qkv, o, qn, kn)
    h = L.hyref_layer_create(H, I, E, _p(in_ln), _p(post_ln), _p(qkv), _p(o), _p(qn), _p(kn),
                             _p(rw), _p(sgu), _p(sdn), (_fp * E)(*[_p(a) for a in egu]),
                             (_fp * E)(*[_p(a) for a in edn]))
    yield dict(L=L, h=h, H=H, I=I, E=E, K=K, seed=seed, keep=keep)
    L.hyref_release()
    L.hyref_layer_destroy(h)


def test_adapter_moe_matches_moe_forward_cpu(orc, layer):
    L, h, H, I, E, K = (layer[k] for k in ("L", "h", "H", "I", "E", "K"))
    T = 21
    x = O.synth_x(orc, layer["seed"], T, H)
    res = {}
    for which in (0, 1):
        out = np.empty((T, H), np.float32)
        probs = np.empty((T, E), np.float32)
        w = np.empty((T, K), np.float32)
        idx = np.empty((T, K), np.int32)
        rc = L.hyref_moe_forward(_p(x), h, T, H, I, K, which, _p(out), _p(probs), _p(w),
                                 idx.ctypes.data_as(C.POINTER(C.c_int32)))
        assert rc == 0
        res[which] = dict(out=out, probs=probs, w=w, idx=idx)
    logits = orc.router(x, np.ascontiguousarray(layer["keep"][0]), K)[0]
    bad, _ = topk_mismatches(res[1]["idx"], res[0]["idx"], logits, K)
    assert bad == 0
    np.testing.assert_allclose(res[1]["probs"], res[0]["probs"], rtol=2e-6, atol=1e-9)
    assert rel_l2(res[1]["out"], res[0]["out"]) <= REL_L2_TOL


def test_reference_decoder_layer_with_gpu_moe(orc, layer):
    L, h, H, I, K = (layer[k] for k in ("L", "h", "H", "I", "K"))
    T = 9
    x = O.synth_x(orc, layer["seed"] + 1, T, H)
    outs = []
    for which in (0, 1):
        out = np.empty((T, H), np.float32)
        assert L.hyref_layer_forward(_p(x), h, T, H, I, K, which, _p(out)) == 0
        outs.append(out)
    # Attention, norms and residuals are the same compiled reference code on both sides;
    # only the MoE differs, so the layer agrees to the MoE tolerance.
    assert rel_l2(outs[1], outs[0]) <= REL_L2_TOL
    assert rel_l2(outs[1] - x, outs[0] - x) <= 2 * REL_L2_TOL


def _moe_both(L, h, x, H, I, E, K):
    """moe_forward_cpu (0) and the adapter (1) on the same MoEWeights object."""
    T = x.shape[0]
    res = {}
    for which in (0, 1):
        out = np.empty((T, H), np.float32)
        probs = np.empty((T, E), np.float32)
        w = np.empty((T, K), np.float32)
        idx = np.empty((T, K), np.int32)
        rc = L.hyref_moe_forward(_p(x), h, T, H, I, K, which, _p(out), _p(probs), _p(w),
                                 idx.ctypes.data_as(C.POINTER(C.c_int32)))
        assert rc == 0
        res[which] = dict(out=out, probs=probs, w=w, idx=idx)
    return res


@pytest.mark.parametrize("in_place", [0, 1])
def test_adapter_follows_a_weight_object_refilled_layer_by_layer(orc, layer, in_place):
    """The reference's layer-streaming loop keeps ONE DecoderLayerWeights object and refills
    it for every layer (src/hunyuan_full_model.cpp:195-207; release_layer's clear +
    shrink_to_fit at :119-130), so consecutive layers' weights often sit at the same
    addresses.  in_place=1 forces that case (new values written over the old ones).  The
    adapter must run each layer on that layer's weights: after the refill it matches
    moe_forward_cpu on the new weights, and its output differs from the previous layer's."""
    L, h, H, I, E, K, seed = (layer[k] for k in ("L", "h", "H", "I", "E", "K", "seed"))
    x = O.synth_x(orc, seed + 2, 17, H)
    first = _moe_both(L, h, x, H, I, E, K)
    assert rel_l2(first[1]["out"], first[0]["out"]) <= REL_L2_TOL
    keep = O.synth_layer_f32(orc, seed, 1, H, I, E, O.F32)  # decoder layer 1 of the same seed
    rw, sgu, sdn, egu, edn = keep
    same_addr = L.hyref_layer_reload_moe(h, H, I, E, _p(rw), _p(sgu), _p(sdn),
                                         (_fp * E)(*[_p(a) for a in egu]),
                                         (_fp * E)(*[_p(a) for a in edn]), in_place)
    if in_place:
        assert same_addr == 1
    second = _moe_both(L, h, x, H, I, E, K)
    logits = orc.router(x, np.ascontiguousarray(rw), K)[0]
    bad, _ = topk_mismatches(second[1]["idx"], second[0]["idx"], logits, K)
    assert bad == 0
    assert rel_l2(second[1]["out"], second[0]["out"]) <= REL_L2_TOL
    assert rel_l2(second[0]["out"], first[0]["out"]) > 0.1  # the layers really differ
    # put layer 0 back for the other tests of this module
    rw0, sgu0, sdn0, egu0, edn0 = layer["keep"][:5]
    L.hyref_layer_reload_moe(h, H, I, E, _p(rw0), _p(sgu0), _p(sdn0), (_fp * E)(*[_p(a) for a in egu0]),
                             (_fp * E)(*[_p(a) for a in edn0]), 1)


def test_adapter_takes_more_tokens_than_one_context(orc, layer):
    """moe_forward_cpu accepts any n_tokens; the adapter runs calls above the context's
    8192-token bound as 8192-token chunks (output and every debug array sliced alike)."""
    L, h, H, I, E, K, seed = (layer[k] for k in ("L", "h", "H", "I", "E", "K", "seed"))
    x = O.synth_x(orc, seed + 3, 8192 + 131, H)
    r = _moe_both(L, h, x, H, I, E, K)
    logits = orc.router(x, np.ascontiguousarray(layer["keep"][0]), K)[0]
    bad, _ = topk_mismatches(r[1]["idx"], r[0]["idx"], logits, K)
    assert bad == 0
    np.testing.assert_allclose(r[1]["probs"], r[0]["probs"], rtol=2e-6, atol=1e-9)
    same = (r[1]["idx"] == r[0]["idx"]).all(axis=1)
    np.testing.assert_allclose(r[1]["w"][same], r[0]["w"][same], rtol=2e-6)
    assert rel_l2(r[1]["out"], r[0]["out"]) <= REL_L2_TOL
    tail = slice(8192, None)  # the second chunk on its own
    assert rel_l2(r[1]["out"][tail], r[0]["out"][tail]) <= REL_L2_TOL
