"""GPU test of hymoe_ffn_noalloc, the entry point for callers that cannot allocate device
memory (code inside CUDA stream capture, engines whose device memory belongs to another
allocator, decode loops that must not allocate per step).  It must give the same answer as
the regular entry point.

Comparisons: (1) a layer whose routed experts are all zero makes hymoe_forward return
exactly the shared expert's SwiGLU FFN, which is what hymoe_ffn_noalloc computes from the
same GGUF bytes; (2) the oracle's swiglu_ffn (the C restatement of the reference's
swiglu_ffn_f32, src/rms_norm.cpp:39-91) on the dequantised weights, for every GGUF type the
entry point reads (F32, F16, Q4_0, Q8_0) and for a shape whose sizes are multiples of 32 but
of nothing larger.  Two calls in a row are checked, so a call that depends on what the
previous call left in the shared static scratch array would be caught.  This file is
collected last and builds everything it needs itself, so it passes alone in a fresh process
too.
"""
import ctypes as C

import numpy as np
import pytest

import hymoe
import oracle as O
from moe_cases import REL_L2_TOL, rel_l2

pytestmark = pytest.mark.gpu


def _device_tensor(torch, raw: np.ndarray, wt: int, rows: int, cols: int):
    d = torch.from_numpy(raw).cuda()
    return d, hymoe.Tensor(d.data_ptr(), wt, (C.c_int64 * 2)(cols, rows), raw.nbytes)


@pytest.mark.parametrize("wt", [O.Q4_0, O.Q8_0])
def test_ffn_noalloc_matches_hymoe_forward(orc, wt):
    torch = pytest.importorskip("torch")
    H, I, E, K, T, seed = 512, 256, 16, 8, 6, 31
    rw = orc.fill_normal(E * H, seed, O.stream_id(0, O.KIND_ROUTER), 0.02).reshape(E, H)
    sgu = orc.synth_tensor(wt, 2 * I * H, seed, O.stream_id(0, O.KIND_GATE_UP, O.SHARED_INDEX), 0.02)
    sdn = orc.synth_tensor(wt, H * I, seed, O.stream_id(0, O.KIND_DOWN, O.SHARED_INDEX), 0.02)
    zgu = orc.quantize(wt, np.zeros(2 * I * H, np.float32))
    zdn = orc.quantize(wt, np.zeros(H * I, np.float32))
    m = hymoe.MoE(H, I, E, K, 1, 16)
    m.load_layer(0, rw, sgu, sdn, [zgu] * E, [zdn] * E, wt)

    L = hymoe.lib()
    gu_d, tg = _device_tensor(torch, sgu, wt, 2 * I, H)
    dn_d, td = _device_tensor(torch, sdn, wt, H, I)
    for call in range(2):
        x = O.synth_x(orc, seed + call, T, H)
        want = m.forward_host(0, x)["out"]
        xd = torch.from_numpy(x).cuda()
        yd = torch.full_like(xd, float("nan"))
        torch.cuda.synchronize()
        st = L.hymoe_ffn_noalloc(C.byref(tg), C.byref(td), xd.data_ptr(), yd.data_ptr(), T, None)
        assert st == 0, L.hymoe_last_error(None)
        torch.cuda.synchronize()
        err = rel_l2(yd.cpu().numpy(), want)
        assert err <= REL_L2_TOL, f"call {call}: rel L2 {err:.3e}"
    m.close()


@pytest.mark.parametrize("wt", [O.F32, O.F16, O.Q4_0, O.Q8_0])
@pytest.mark.parametrize("H,I,T", [(512, 256, 8), (160, 96, 3)])
def test_ffn_noalloc_matches_the_oracle_swiglu_ffn(orc, wt, H, I, T):
    torch = pytest.importorskip("torch")
    seed = 41 + wt
    gu = orc.synth_tensor(wt, 2 * I * H, seed, O.stream_id(0, O.KIND_GATE_UP, 3), 0.02)
    dn = orc.synth_tensor(wt, H * I, seed, O.stream_id(0, O.KIND_DOWN, 3), 0.02)
    deq = lambda raw, n: raw.view(np.float32).copy() if wt == O.F32 else orc.dequantize(wt, raw, n)
    gu_f, dn_f = deq(gu, 2 * I * H), deq(dn, H * I)
    L = hymoe.lib()
    gu_d, tg = _device_tensor(torch, gu, wt, 2 * I, H)
    dn_d, td = _device_tensor(torch, dn, wt, H, I)
    for call in range(2):
        x = O.synth_x(orc, seed + call, T, H)
        want = orc.swiglu_ffn(x, gu_f, dn_f, I)
        xd = torch.from_numpy(x).cuda()
        yd = torch.full_like(xd, float("nan"))
        torch.cuda.synchronize()
        st = L.hymoe_ffn_noalloc(C.byref(tg), C.byref(td), xd.data_ptr(), yd.data_ptr(), T, None)
        assert st == 0, L.hymoe_last_error(None)
        torch.cuda.synchronize()
        err = rel_l2(yd.cpu().numpy(), want)
        assert err <= REL_L2_TOL, f"call {call}: rel L2 {err:.3e}"


def test_ffn_noalloc_rejects_sizes_beyond_its_scratch(orc):
    torch = pytest.importorskip("torch")
    L = hymoe.lib()
    H, I, wt = 256, 128, O.Q8_0
    gu_d, tg = _device_tensor(torch, orc.quantize(wt, np.zeros(2 * I * H, np.float32)), wt, 2 * I, H)
    dn_d, td = _device_tensor(torch, orc.quantize(wt, np.zeros(H * I, np.float32)), wt, H, I)
    x = torch.zeros(16, H, device="cuda")
    y = torch.zeros(16, H, device="cuda")
    st = L.hymoe_ffn_noalloc(C.byref(tg), C.byref(td), x.data_ptr(), y.data_ptr(),
                             9, None)
    assert st == 1 and b"HYMOE_NOALLOC_MAX_TOKENS" in L.hymoe_last_error(None)
    big_i = 16384 + 32  # claims an intermediate size larger than the static array
    tbig = hymoe.Tensor(gu_d.data_ptr(), wt, (C.c_int64 * 2)(H, 2 * big_i),
                        2 * big_i * H // 32 * 34)
    dbig = hymoe.Tensor(dn_d.data_ptr(), wt, (C.c_int64 * 2)(big_i, H), big_i * H // 32 * 34)
    st = L.hymoe_ffn_noalloc(C.byref(tbig), C.byref(dbig), x.data_ptr(), y.data_ptr(), 1, None)
    assert st == 1 and b"HYMOE_NOALLOC_MAX_INTERMEDIATE" in L.hymoe_last_error(None)
    xh = np.zeros((1, H), np.float32)
    st = L.hymoe_ffn_noalloc(C.byref(tg), C.byref(td), xh.ctypes.data, y.data_ptr(), 1, None)
    assert st == 1 and b"device memory" in L.hymoe_last_error(None)
    if torch.cuda.device_count() > 1:  # another GPU's memory: refused, not read over the link
        x1 = torch.zeros(1, H, device="cuda:1")
        st = L.hymoe_ffn_noalloc(C.byref(tg), C.byref(td), x1.data_ptr(), y.data_ptr(), 1, None)
        assert st == 1 and b"current device" in L.hymoe_last_error(None)
