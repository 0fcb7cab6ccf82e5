"""GPU tests of asynchronous layer loading (hymoe_load_layer_async, hymoe_load_layer_gguf_async,
hymoe_wait_layer): the reference's layer-streaming loop (load a layer, run it, release it;
src/hunyuan_full_model.cpp:195-207) through two layer slots, the next layer's upload queued
before the current layer runs.  Every result must equal the same loop with synchronous loads
bit for bit (the same kernels on the same bytes)."""
import numpy as np
import pytest

import hymoe
import oracle as O
from moe_cases import REL_L2_TOL, host_layer, rel_l2

pytestmark = pytest.mark.gpu

H, I, E, K, WT = 512, 256, 64, 8, O.Q4_0


def _load(m, slot, lay, asynchronous):
    f = m.load_layer_async if asynchronous else m.load_layer
    f(slot, lay["router"], lay["sgu"], lay["sdn"], lay["egu"], lay["edn"], WT)


def test_two_slot_streaming_equals_synchronous_loads(orc):
    """x <- x + MoE_l(x) over 5 layers: synchronous loads into 5 slots against asynchronous loads
    into 2 alternating slots, layer l+1 queued before layer l runs; host-pointer calls."""
    T, seed, n = 300, 91, 5
    lays = [host_layer(orc, seed, l, H, I, E, WT) for l in range(n)]
    x0 = O.synth_x(orc, seed, T, H)
    ref = hymoe.MoE(H, I, E, K, n, T)
    for l in range(n):
        _load(ref, l, lays[l], False)
    want, x = [], x0
    for l in range(n):
        x = ref.forward_host(l, x, resid=x)["out"]
        want.append(x)
    ref.close()

    m = hymoe.MoE(H, I, E, K, 2, T)
    _load(m, 0, lays[0], True)
    x = x0
    for l in range(n):
        if l + 1 < n:
            _load(m, (l + 1) % 2, lays[l + 1], True)  # overlaps layer l's compute
        x = m.forward_host(l % 2, x, resid=x)["out"]
        assert np.array_equal(x, want[l]), f"layer {l}"
        m.wait_layer(l % 2)
    m.wait_layer((n - 1) % 2)
    m.close()
    o = x0
    for l in range(n):
        lay = lays[l]
        o = orc.moe_forward(o, lay["router"], lay["sgu_f"], lay["sdn_f"], lay["egu_f"], lay["edn_f"], K, I,
                            resid=o)["out"]
    assert rel_l2(x, o) <= REL_L2_TOL


def test_device_call_right_after_queueing_waits_on_the_gpu(orc):
    """A device-pointer forward issued right after hymoe_load_layer_async (no host wait in
    between) computes with the new weights: its stream waits for the load on the GPU."""
    torch = pytest.importorskip("torch")
    T, seed = 70, 93
    a, b = host_layer(orc, seed, 0, H, I, E, WT), host_layer(orc, seed, 1, H, I, E, WT)
    x = O.synth_x(orc, seed, T, H)
    ref = hymoe.MoE(H, I, E, K, 1, T)
    _load(ref, 0, b, False)
    want = ref.forward_host(0, x)["out"]
    ref.close()
    m = hymoe.MoE(H, I, E, K, 1, T)
    _load(m, 0, a, False)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        m.set_stream(st.cuda_stream)
        xd = torch.from_numpy(x).cuda()
        od = torch.empty_like(xd)
        m.forward_device(0, xd.data_ptr(), od.data_ptr(), T)  # layer a, queued before the load
        first = torch.empty_like(xd)
        first.copy_(od)
        _load(m, 0, b, True)                                   # rewrites the slot after that call
        m.forward_device(0, xd.data_ptr(), od.data_ptr(), T)  # must see layer b
    m.synchronize()
    m.wait_layer(0)
    assert np.array_equal(od.cpu().numpy(), want)
    ref_a = hymoe.MoE(H, I, E, K, 1, T)
    _load(ref_a, 0, a, False)
    assert np.array_equal(first.cpu().numpy(), ref_a.forward_host(0, x)["out"])
    ref_a.close()
    m.close()


def test_gguf_async_load_matches_synchronous(orc, tmp_path):
    pytest.importorskip("gguf")
    from gguf_layer import write_moe_layer
    T, seed = 130, 95
    lay = host_layer(orc, seed, 0, H, I, E, WT)
    path = str(tmp_path / "layer3.gguf")
    write_moe_layer(path, 3, H, I, lay["router"], lay["sgu"], lay["sdn"], lay["egu"], lay["edn"], WT)
    x = O.synth_x(orc, seed, T, H)
    m = hymoe.MoE(H, I, E, K, 2, T)
    with hymoe.GGUF(path) as f:
        m.load_layer_gguf(0, f, 3)
        m.load_layer_gguf_async(1, f, 3)
        got = m.forward_host(1, x)["out"]
        m.wait_layer(1)
    assert np.array_equal(got, m.forward_host(0, x)["out"])
    m.wait_layer(0)  # no asynchronous load queued: returns at once
    m.close()
