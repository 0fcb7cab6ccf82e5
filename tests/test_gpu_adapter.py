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
