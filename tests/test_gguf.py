"""CPU tests of the library's GGUF reader (hymoe_gguf_*, no device): files written by gguf-py
(the package the reference's converter uses) under the reference's tensor names, read back
as views of their raw blocks and compared with gguf-py's own reader; malformed files give a
status, never a crash."""
import os

import numpy as np
import pytest

import hymoe
import oracle as O
from gguf_layer import write_moe_layer
from moe_cases import host_layer

gguf = pytest.importorskip("gguf")

H, I, E = 256, 128, 8


def _write(tmp_path, wtype, layer_idx=3, router_type=O.F32, alignment=None, extra=None, name="l.gguf"):
    orc = O.Oracle()
    lay = host_layer(orc, 11, 0, H, I, E, wtype)
    path = str(tmp_path / name)
    write_moe_layer(path, layer_idx, H, I, lay["router"], lay["sgu"], lay["sdn"], lay["egu"],
                    lay["edn"], wtype, router_type=router_type, alignment=alignment, extra=extra)
    return path, lay


@pytest.mark.parametrize("wtype", [O.Q4_0, O.Q8_0, O.F16, O.F32])
def test_moe_tensors_are_the_written_blocks(tmp_path, wtype):
    path, lay = _write(tmp_path, wtype)
    with hymoe.GGUF(path) as f:
        assert f.get_u32("hunyuan.num_experts") == E
        assert f.get_u32("hunyuan.layer_idx") == 3
        m = f.moe_tensors(3, E)
    assert m["router"]["type"] == O.F32 and m["router"]["ne"] == (H, E)
    assert np.array_equal(m["router"]["bytes"].view(np.float32), lay["router"].ravel())
    for key, rows, cols in (("sgu", 2 * I, H), ("sdn", H, I)):
        assert m[key]["type"] == wtype and m[key]["ne"] == (cols, rows)
        assert np.array_equal(m[key]["bytes"], lay[key].view(np.uint8).ravel())
    for e in range(E):
        assert np.array_equal(m["egu"][e]["bytes"], lay["egu"][e].view(np.uint8).ravel())
        assert np.array_equal(m["edn"][e]["bytes"], lay["edn"][e].view(np.uint8).ravel())
        assert m["edn"][e]["ne"] == (I, H)


def test_views_match_gguf_py_reader_and_other_tensors_are_skipped(tmp_path):
    extra = {"blk.3.attn_qkv.weight": np.arange(24, dtype=np.float32).reshape(2, 3, 4),  # 3 dims
             "blk.3.ffn_norm.weight": np.linspace(-1, 1, H).astype(np.float32),           # 1 dim
             "blk.3.pos": np.arange(10, dtype=np.int32)}                                   # I32
    path, _ = _write(tmp_path, O.Q4_0, extra=extra)
    rd = gguf.GGUFReader(path)
    with hymoe.GGUF(path) as f:
        for t in rd.tensors:
            raw = np.asarray(t.data).view(np.uint8).ravel()
            if t.name == "blk.3.attn_qkv.weight" or t.name == "blk.3.pos":
                with pytest.raises(hymoe.HymoeError) as ei:
                    f.tensor(t.name)
                assert ei.value.status == 4  # unsupported rank / type
                continue
            v = f.tensor(t.name)
            assert v["type"] == int(t.tensor_type)
            assert v["nbytes"] == raw.size and np.array_equal(v["bytes"], raw), t.name
        with pytest.raises(hymoe.HymoeError):
            f.tensor("blk.3.no_such.weight")
        with pytest.raises(hymoe.HymoeError):
            f.get_u32("general.architecture")  # a string, not u32
        with pytest.raises(hymoe.HymoeError):
            f.moe_tensors(4, E)  # another layer's names


def test_float_weights_are_quantised_with_the_standard_blocks(tmp_path):
    rng = np.random.default_rng(0)
    wf = [(rng.standard_normal((2 * I, H)) * 0.02).astype(np.float32) for _ in range(E)]
    df = [(rng.standard_normal((H, I)) * 0.02).astype(np.float32) for _ in range(E)]
    rw = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    path = str(tmp_path / "f.gguf")
    write_moe_layer(path, 0, H, I, rw, wf[0], df[0], wf, df, O.Q4_0)
    orc = O.Oracle()
    with hymoe.GGUF(path) as f:
        m = f.moe_tensors(0, E)
    for e in (0, E - 1):
        q = gguf.quants.quantize(wf[e], gguf.GGMLQuantizationType.Q4_0).ravel()
        assert np.array_equal(m["egu"][e]["bytes"], q)
        # the oracle's standard decode of those blocks equals gguf-py's
        ref = gguf.quants.dequantize(q.reshape(2 * I, -1), gguf.GGMLQuantizationType.Q4_0).ravel()
        assert np.array_equal(orc.dequantize(O.Q4_0, q, 2 * I * H), ref.astype(np.float32))


def test_custom_alignment(tmp_path):
    path, lay = _write(tmp_path, O.Q8_0, alignment=256)
    with hymoe.GGUF(path) as f:
        assert np.array_equal(f.tensor("blk.3.ffn_expert_5_down.weight")["bytes"], lay["edn"][5])


def _expect_error(path, data):
    with open(path, "wb") as fh:
        fh.write(data)
    with pytest.raises(hymoe.HymoeError) as ei:
        hymoe.GGUF(path)
    assert ei.value.status in (1, 4)


def test_malformed_files_give_a_status(tmp_path):
    path, _ = _write(tmp_path, O.Q4_0)
    good = open(path, "rb").read()
    bad = str(tmp_path / "bad.gguf")
    _expect_error(bad, b"")
    _expect_error(bad, b"GGML" + good[4:])
    for version in (1, 4):
        _expect_error(bad, good[:4] + version.to_bytes(4, "little") + good[8:])
    _expect_error(bad, good[:8] + (1 << 62).to_bytes(8, "little") + good[16:])   # tensor count
    _expect_error(bad, good[:16] + (1 << 62).to_bytes(8, "little") + good[24:])  # key count
    first_key_len = good[24:32]
    assert int.from_bytes(first_key_len, "little") < 100
    _expect_error(bad, good[:24] + (1 << 63).to_bytes(8, "little") + good[32:])  # string length
    _expect_error(bad, good[: len(good) - 1])                                     # data past the end
    with pytest.raises(hymoe.HymoeError):
        hymoe.GGUF(str(tmp_path / "missing.gguf"))


def test_every_truncated_header_gives_a_status(tmp_path):
    path, _ = _write(tmp_path, O.Q4_0)
    good = open(path, "rb").read()
    rd = gguf.GGUFReader(path)
    data_start = min(int(t.data_offset) for t in rd.tensors)
    bad = str(tmp_path / "cut.gguf")
    for n in range(0, data_start + 64):
        _expect_error(bad, good[:n])


def test_flipped_header_bytes_never_crash(tmp_path):
    """Seeded byte corruption of the header region: open either fails with a status or
    succeeds with every MoE view readable inside the mapping."""
    path, _ = _write(tmp_path, O.Q8_0)
    good = bytearray(open(path, "rb").read())
    rd = gguf.GGUFReader(path)
    data_start = min(int(t.data_offset) for t in rd.tensors)
    rng = np.random.default_rng(1)
    bad = str(tmp_path / "flip.gguf")
    opened = 0
    for _ in range(300):
        b = bytearray(good)
        for p in rng.integers(0, data_start, size=int(rng.integers(1, 4))):
            b[p] = int(rng.integers(0, 256))
        with open(bad, "wb") as fh:
            fh.write(b)
        try:
            f = hymoe.GGUF(bad)
        except hymoe.HymoeError as e:
            assert e.status in (1, 4)
            continue
        opened += 1
        try:
            f.moe_tensors(3, E)
        except hymoe.HymoeError:
            pass
        f.close()
    assert opened > 0  # some flips hit bytes the reader does not depend on


def test_null_arguments():
    L = hymoe.lib()
    assert L.hymoe_gguf_open(None, None) == 1
    assert L.hymoe_gguf_tensor(None, b"x", None) == 1
    assert L.hymoe_load_layer_gguf(None, 0, None, 0) == 1
    L.hymoe_gguf_close(None)
    assert os.path.exists(hymoe.LIB_PATH)
