"""Writes one decoder layer's MoE tensors as a GGUF file that hymoe_gguf_open /
hymoe_load_layer_gguf read: the reference converter's tensor names and metadata keys
(scripts/convert_to_gguf.py:70-137, 183-200), PyTorch [out, in] layout (no transpose), and
weights quantised with gguf-py's standard block quantisation.  (The reference converter hands
float32 data to gguf-py with a Q4_0/Q8_0 label, which stores the float bytes themselves rather
than quantised blocks; this writer quantises.)  Needs the `gguf` package.
"""
from __future__ import annotations

import numpy as np

TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q8_0 = 0, 1, 2, 8


def _encode(gguf, arr: np.ndarray, rows: int, cols: int, wtype: int):
    """(array, raw_dtype) for GGUFWriter.add_tensor.  float32 [rows, cols] is converted to
    wtype; uint8 holds raw GGUF blocks of wtype already."""
    qt = gguf.GGMLQuantizationType
    if arr.dtype == np.uint8:
        raw = np.ascontiguousarray(arr).reshape(rows, -1)
        return raw, qt(wtype)
    w = np.ascontiguousarray(arr, dtype=np.float32).reshape(rows, cols)
    if wtype == TYPE_F32:
        return w, None
    if wtype == TYPE_F16:
        return w.astype(np.float16), None
    return gguf.quants.quantize(w, qt(wtype)), qt(wtype)


def write_moe_layer(path: str, layer_idx: int, H: int, I: int, router, shared_gate_up,
                    shared_down, experts_gate_up, experts_down, wtype: int,
                    router_type: int = TYPE_F32, moe_topk: int = 8, alignment: int | None = None,
                    extra: dict | None = None) -> None:
    """router [E, H] float32; every other weight float32 [rows, cols] or raw GGUF bytes (uint8)
    of `wtype`.  extra: more tensors {name: ndarray} written as they are."""
    import gguf
    E = len(experts_gate_up)
    w = gguf.GGUFWriter(path, "hunyuan3")
    if alignment is not None:
        w.add_custom_alignment(alignment)
    w.add_uint32("hunyuan.hidden_size", H)
    w.add_uint32("hunyuan.moe_intermediate_size", I)
    w.add_uint32("hunyuan.num_experts", E)
    w.add_uint32("hunyuan.moe_topk", moe_topk)
    w.add_uint32("hunyuan.layer_idx", layer_idx)
    p = f"blk.{layer_idx}."
    tensors = {p + "ffn_gate.weight": _encode(gguf, np.asarray(router, np.float32), E, H, router_type),
               p + "ffn_shared_gate_up.weight": _encode(gguf, shared_gate_up, 2 * I, H, wtype),
               p + "ffn_shared_down.weight": _encode(gguf, shared_down, H, I, wtype)}
    for e in range(E):
        tensors[p + f"ffn_expert_{e}_gate_up.weight"] = _encode(gguf, experts_gate_up[e], 2 * I, H, wtype)
        tensors[p + f"ffn_expert_{e}_down.weight"] = _encode(gguf, experts_down[e], H, I, wtype)
    for name, arr in (extra or {}).items():
        tensors[name] = (arr, None)
    for name in sorted(tensors):
        arr, raw_dtype = tensors[name]
        if raw_dtype is None:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=raw_dtype)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
