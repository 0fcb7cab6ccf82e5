"""ctypes bindings of libhymoe.so (the C ABI in include/hymoe.h).

This is how the test-suite and bench.py drive the library; a C++ host uses the header
directly (see the adapter in csrc/adapter/).  The module fails loudly when the CUDA
library is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
# HYMOE_LIB: load another build of the library (e.g. to compare two builds on one machine)
LIB_PATH = os.environ.get("HYMOE_LIB") or os.path.join(HERE, "libhymoe.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "hymoe.h")

TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q8_0 = 0, 1, 2, 8
HOST_PTRS = 1
USE_GRAPH = 2
PRE_NORM = 4

STATUS = {0: "OK", 1: "INVALID_ARG", 2: "CUDA", 3: "OOM", 4: "UNSUPPORTED", 5: "NCCL",
          6: "TIMEOUT", 7: "STATE"}
STATUS_TIMEOUT = 6

# Every function include/hymoe.h declares.
EXPORTS = ["hymoe_version", "hymoe_nccl_unique_id", "hymoe_create", "hymoe_destroy",
           "hymoe_last_error", "hymoe_set_stream", "hymoe_synchronize", "hymoe_load_layer",
           "hymoe_synth_layer", "hymoe_forward", "hymoe_profile", "hymoe_profile_read",
           "hymoe_ffn_noalloc", "hymoe_set_placement", "hymoe_balance_placement",
           "hymoe_gguf_open", "hymoe_gguf_close", "hymoe_gguf_last_error", "hymoe_gguf_tensor",
           "hymoe_gguf_get_u32", "hymoe_gguf_moe_tensors", "hymoe_load_layer_gguf",
           "hymoe_set_norm", "hymoe_set_routing", "hymoe_load_layer_async", "hymoe_wait_layer",
           "hymoe_load_layer_gguf_async"]

PHASES = ["router", "plan", "dispatch", "gate_up", "down", "combine", "ep_dispatch",
          "ep_combine", "copy_in", "copy_out"]


class Config(C.Structure):
    _fields_ = [("hidden_size", C.c_uint32), ("moe_intermediate_size", C.c_uint32),
                ("num_experts", C.c_uint32), ("moe_topk", C.c_uint32), ("num_layers", C.c_uint32),
                ("max_tokens", C.c_uint32), ("device", C.c_int32), ("ep_rank", C.c_int32),
                ("ep_size", C.c_int32), ("nccl_unique_id", C.c_void_p)]


class Tensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("ggml_type", C.c_int32), ("ne", C.c_int64 * 2),
                ("nbytes", C.c_size_t)]


class Routing(C.Structure):
    _fields_ = [("group_limited_greedy", C.c_int32), ("n_group", C.c_uint32), ("topk_group", C.c_uint32),
                ("drop_tokens", C.c_int32), ("capacity_factor", C.c_float), ("min_capacity", C.c_uint32),
                ("norm_topk_prob", C.c_int32), ("routed_scaling_factor", C.c_float)]


class Debug(C.Structure):
    _fields_ = [("router_logits", C.c_void_p), ("router_probs", C.c_void_p),
                ("topk_weights", C.c_void_p), ("topk_indices", C.c_void_p)]


class HymoeError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"hymoe {STATUS.get(status, status)}: {msg}")
        self.status = status


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE, "-j8"], check=True)


_LIB = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built (run make -C {HERE})")
        L = C.CDLL(LIB_PATH)
        vp, i32, u32, u64 = C.c_void_p, C.c_int32, C.c_uint32, C.c_uint64
        L.hymoe_version.restype = C.c_char_p
        L.hymoe_nccl_unique_id.argtypes = [vp]
        L.hymoe_create.argtypes = [C.POINTER(Config), C.POINTER(vp)]
        L.hymoe_destroy.argtypes = [vp]
        L.hymoe_destroy.restype = None
        L.hymoe_last_error.argtypes = [vp]
        L.hymoe_last_error.restype = C.c_char_p
        L.hymoe_set_stream.argtypes = [vp, vp]
        L.hymoe_synchronize.argtypes = [vp]
        L.hymoe_load_layer.argtypes = [vp, u32, C.POINTER(Tensor), C.POINTER(Tensor),
                                       C.POINTER(Tensor), C.POINTER(Tensor), C.POINTER(Tensor),
                                       C.c_int]
        L.hymoe_synth_layer.argtypes = [vp, u32, i32, u64, C.c_float]
        L.hymoe_forward.argtypes = [vp, u32, vp, vp, vp, u32, vp, C.POINTER(Debug), C.c_int]
        L.hymoe_profile.argtypes = [vp, C.c_int]
        L.hymoe_ffn_noalloc.argtypes = [C.POINTER(Tensor), C.POINTER(Tensor), vp, vp, u32, vp]
        L.hymoe_profile_read.argtypes = [vp, C.POINTER(C.c_float), C.POINTER(C.c_int32), C.c_int]
        L.hymoe_set_placement.argtypes = [vp, u32, C.POINTER(C.c_int32)]
        L.hymoe_balance_placement.argtypes = [u32, u32, C.POINTER(C.c_double), C.POINTER(C.c_int32)]
        L.hymoe_gguf_open.argtypes = [C.c_char_p, C.POINTER(vp)]
        L.hymoe_gguf_close.argtypes = [vp]
        L.hymoe_gguf_close.restype = None
        L.hymoe_gguf_last_error.argtypes = []
        L.hymoe_gguf_last_error.restype = C.c_char_p
        L.hymoe_gguf_tensor.argtypes = [vp, C.c_char_p, C.POINTER(Tensor)]
        L.hymoe_gguf_get_u32.argtypes = [vp, C.c_char_p, C.POINTER(u32)]
        L.hymoe_gguf_moe_tensors.argtypes = [vp, u32, u32, C.POINTER(Tensor), C.POINTER(Tensor),
                                             C.POINTER(Tensor), C.POINTER(Tensor), C.POINTER(Tensor)]
        L.hymoe_load_layer_gguf.argtypes = [vp, u32, vp, u32]
        L.hymoe_load_layer_async.argtypes = [vp, u32, C.POINTER(Tensor), C.POINTER(Tensor),
                                             C.POINTER(Tensor), C.POINTER(Tensor), C.POINTER(Tensor)]
        L.hymoe_wait_layer.argtypes = [vp, u32]
        L.hymoe_load_layer_gguf_async.argtypes = [vp, u32, vp, u32]
        L.hymoe_set_norm.argtypes = [vp, u32, vp, C.c_float, C.c_int]
        L.hymoe_set_routing.argtypes = [vp, C.POINTER(Routing)]
        for f in EXPORTS:
            if f not in ("hymoe_version", "hymoe_destroy", "hymoe_last_error", "hymoe_gguf_close",
                         "hymoe_gguf_last_error"):
                getattr(L, f).restype = C.c_int
        _LIB = L
    return _LIB


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    st = lib().hymoe_nccl_unique_id(buf)
    if st != 0:
        raise HymoeError(st, "hymoe_nccl_unique_id failed")
    return buf.raw


def balance_placement(load, ep_size: int) -> list:
    """slot_of_expert (a list of E ints) balancing per-expert `load` over ep_size ranks
    (hymoe_balance_placement: greedy, heaviest expert first)."""
    E = len(load)
    buf = (C.c_double * E)(*[float(v) for v in load])
    out = (C.c_int32 * E)()
    st = lib().hymoe_balance_placement(E, ep_size, buf, out)
    if st != 0:
        raise HymoeError(st, f"hymoe_balance_placement: invalid arguments (E={E}, ep_size={ep_size})")
    return list(out)


class GGUF:
    """A GGUF weight file opened by the library (hymoe_gguf_*): parsed, mapped read-only."""

    def __init__(self, path: str):
        self.L = lib()
        h = C.c_void_p()
        st = self.L.hymoe_gguf_open(os.fsencode(path), C.byref(h))
        if st != 0:
            raise HymoeError(st, self.L.hymoe_gguf_last_error().decode(errors="replace"))
        self.h = h

    def _check(self, st: int) -> None:
        if st != 0:
            raise HymoeError(st, self.L.hymoe_gguf_last_error().decode(errors="replace"))

    def close(self) -> None:
        if getattr(self, "h", None):
            self.L.hymoe_gguf_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @staticmethod
    def _view(t: Tensor) -> dict:
        import numpy as np
        raw = np.ctypeslib.as_array(C.cast(t.data, C.POINTER(C.c_uint8)), shape=(t.nbytes,)).copy()
        return {"type": t.ggml_type, "ne": (t.ne[0], t.ne[1]), "nbytes": t.nbytes, "bytes": raw}

    def tensor(self, name: str) -> dict:
        """{type, ne (GGUF order), nbytes, bytes (a copy of the raw blocks)}."""
        t = Tensor()
        self._check(self.L.hymoe_gguf_tensor(self.h, name.encode(), C.byref(t)))
        return self._view(t)

    def get_u32(self, key: str) -> int:
        v = C.c_uint32()
        self._check(self.L.hymoe_gguf_get_u32(self.h, key.encode(), C.byref(v)))
        return v.value

    def moe_tensors(self, layer_idx: int, n_experts: int) -> dict:
        r, sg, sd = Tensor(), Tensor(), Tensor()
        eg, ed = (Tensor * n_experts)(), (Tensor * n_experts)()
        self._check(self.L.hymoe_gguf_moe_tensors(self.h, layer_idx, n_experts, C.byref(r), C.byref(sg),
                                                  C.byref(sd), eg, ed))
        return {"router": self._view(r), "sgu": self._view(sg), "sdn": self._view(sd),
                "egu": [self._view(t) for t in eg], "edn": [self._view(t) for t in ed]}


def gguf_nbytes(t: int, n: int) -> int:
    return {TYPE_F32: 4 * n, TYPE_F16: 2 * n, TYPE_Q4_0: n // 32 * 18, TYPE_Q8_0: n // 32 * 34}[t]


def _tensor(arr, t: int, rows: int, cols: int) -> Tensor:
    """arr: numpy uint8/float32 host array (GGUF bytes) or None."""
    if arr is None:
        return Tensor(None, t, (C.c_int64 * 2)(cols, rows), 0)
    return Tensor(arr.ctypes.data, t, (C.c_int64 * 2)(cols, rows), arr.nbytes)


class MoE:
    """One hymoe context: shapes of HunyuanConfig, layer slots, scratch for max_tokens."""

    def __init__(self, H=4096, I=3072, E=64, K=8, num_layers=1, max_tokens=4096, device=0,
                 ep_rank=0, ep_size=1, nccl_id: bytes | None = None):
        self.L = lib()
        self.H, self.I, self.E, self.K = H, I, E, K
        self._id = C.create_string_buffer(nccl_id, 128) if nccl_id else None
        cfg = Config(H, I, E, K, num_layers, max_tokens, device, ep_rank, ep_size,
                     C.cast(self._id, C.c_void_p) if self._id else None)
        h = C.c_void_p()
        st = self.L.hymoe_create(C.byref(cfg), C.byref(h))
        if st != 0:
            raise HymoeError(st, self.L.hymoe_last_error(None).decode())
        self.h = h

    def _check(self, st: int) -> None:
        if st != 0:
            raise HymoeError(st, self.L.hymoe_last_error(self.h).decode())

    def close(self) -> None:
        if getattr(self, "h", None):
            self.L.hymoe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream_ptr: int | None) -> None:
        self._check(self.L.hymoe_set_stream(self.h, stream_ptr))

    def synchronize(self) -> None:
        self._check(self.L.hymoe_synchronize(self.h))

    def profile(self, enable: bool) -> None:
        self._check(self.L.hymoe_profile(self.h, 1 if enable else 0))

    def profile_read(self) -> dict:
        """{phase: (total_ms, launches)} recorded since profile(True)."""
        n = len(PHASES)
        ms = (C.c_float * n)()
        cnt = (C.c_int32 * n)()
        self._check(self.L.hymoe_profile_read(self.h, ms, cnt, n))
        return {p: (float(ms[i]), int(cnt[i])) for i, p in enumerate(PHASES)}

    def load_layer(self, layer: int, router, shared_gu, shared_dn, experts_gu, experts_dn,
                   wtype: int) -> None:
        """Host numpy arrays: router float32 [E, H]; the others GGUF bytes of `wtype`
        (entries of experts_* may be None for experts another rank owns)."""
        H, I, E = self.H, self.I, self.E
        r = _tensor(router, TYPE_F32, E, H)
        sg = _tensor(shared_gu, wtype, 2 * I, H)
        sd = _tensor(shared_dn, wtype, H, I)
        eg = (Tensor * E)(*[_tensor(a, wtype, 2 * I, H) for a in experts_gu])
        ed = (Tensor * E)(*[_tensor(a, wtype, H, I) for a in experts_dn])
        self._check(self.L.hymoe_load_layer(self.h, layer, C.byref(r), C.byref(sg), C.byref(sd),
                                            eg, ed, HOST_PTRS))

    def load_layer_async(self, layer: int, router, shared_gu, shared_dn, experts_gu, experts_dn,
                         wtype: int) -> None:
        """hymoe_load_layer_async: returns at once; the arrays must stay alive and unchanged until
        wait_layer(layer) (this object keeps references to them until then)."""
        H, I, E = self.H, self.I, self.E
        r = _tensor(router, TYPE_F32, E, H)
        sg = _tensor(shared_gu, wtype, 2 * I, H)
        sd = _tensor(shared_dn, wtype, H, I)
        eg = (Tensor * E)(*[_tensor(a, wtype, 2 * I, H) for a in experts_gu])
        ed = (Tensor * E)(*[_tensor(a, wtype, H, I) for a in experts_dn])
        self._check(self.L.hymoe_load_layer_async(self.h, layer, C.byref(r), C.byref(sg), C.byref(sd), eg, ed))
        self._pending = getattr(self, "_pending", {})
        self._pending.setdefault(layer, []).append((router, shared_gu, shared_dn, experts_gu, experts_dn))

    def load_layer_gguf_async(self, layer: int, file: "GGUF", layer_idx: int) -> None:
        """hymoe_load_layer_gguf_async: keep `file` open until wait_layer(layer)."""
        self._check(self.L.hymoe_load_layer_gguf_async(self.h, layer, file.h, layer_idx))

    def wait_layer(self, layer: int) -> None:
        self._check(self.L.hymoe_wait_layer(self.h, layer))
        getattr(self, "_pending", {}).pop(layer, None)

    def set_placement(self, layer: int, slot_of_expert) -> None:
        """Expert placement (a permutation of 0..E-1, or None for identity); load the layer
        again afterwards."""
        if slot_of_expert is None:
            self._check(self.L.hymoe_set_placement(self.h, layer, None))
            return
        if len(slot_of_expert) != self.E:
            raise ValueError(f"placement needs {self.E} entries, got {len(slot_of_expert)}")
        arr = (C.c_int32 * self.E)(*[int(v) for v in slot_of_expert])
        self._check(self.L.hymoe_set_placement(self.h, layer, arr))

    def set_routing(self, group=None, drop=None, min_capacity: int = 8, norm_topk_prob: bool = True,
                    scale: float = 1.0, plain: bool = False) -> None:
        """FULL-mode routing variant (hymoe_set_routing); plain=True restores the default.
        group = (n_group, topk_group); drop = capacity_factor of capacity-limited routing (one
        GPU; the pairs beyond each expert's capacity in k-major order are dropped)."""
        if plain:
            self._check(self.L.hymoe_set_routing(self.h, None))
            return
        ng, tg = group if group else (0, 0)
        r = Routing(1 if group else 0, ng, tg, 0 if drop is None else 1, 1.0 if drop is None else drop,
                    min_capacity, 1 if norm_topk_prob else 0, scale)
        self._check(self.L.hymoe_set_routing(self.h, C.byref(r)))

    def set_norm(self, layer: int, weight, eps: float) -> None:
        """Post-attention RMSNorm weights [H] (host numpy float32; None removes them)."""
        import numpy as np
        if weight is None:
            self._check(self.L.hymoe_set_norm(self.h, layer, None, eps, HOST_PTRS))
            return
        w = np.ascontiguousarray(weight, dtype=np.float32)
        if w.shape != (self.H,):
            raise ValueError(f"norm weight must be [{self.H}], got {w.shape}")
        self._check(self.L.hymoe_set_norm(self.h, layer, w.ctypes.data, eps, HOST_PTRS))

    def load_layer_gguf(self, layer: int, file: GGUF, layer_idx: int) -> None:
        """Loads decoder layer `layer_idx` of an open GGUF file into layer slot `layer`."""
        self._check(self.L.hymoe_load_layer_gguf(self.h, layer, file.h, layer_idx))

    def synth_layer(self, layer: int, wtype: int, seed: int, std: float = 0.02) -> None:
        self._check(self.L.hymoe_synth_layer(self.h, layer, wtype, seed, std))

    def forward_host(self, layer: int, x, resid=None, bias=None, debug: bool = False,
                     pre_norm: bool = False) -> dict:
        """x (and resid) float32 [T, H] numpy; returns numpy outputs.  pre_norm: x is the
        un-normalised hidden state (HYMOE_PRE_NORM); resid="x" passes x itself as residual."""
        import numpy as np
        x = np.ascontiguousarray(x, dtype=np.float32)
        T = x.shape[0]
        out = np.empty_like(x)
        res = {"out": out}
        dbg = None
        if debug:
            res.update(logits=np.empty((T, self.E), np.float32),
                       probs=np.empty((T, self.E), np.float32),
                       w=np.empty((T, self.K), np.float32), idx=np.empty((T, self.K), np.int32))
            dbg = Debug(res["logits"].ctypes.data, res["probs"].ctypes.data,
                        res["w"].ctypes.data, res["idx"].ctypes.data)
        r = None if resid is None else x if isinstance(resid, str) and resid == "x" else \
            np.ascontiguousarray(resid, dtype=np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self._check(self.L.hymoe_forward(self.h, layer, x.ctypes.data,
                                         None if r is None else r.ctypes.data, out.ctypes.data, T,
                                         None if b is None else b.ctypes.data,
                                         C.byref(dbg) if dbg else None,
                                         HOST_PTRS | (PRE_NORM if pre_norm else 0)))
        return res

    def forward_device(self, layer: int, x_ptr: int, out_ptr: int, T: int, resid_ptr=None,
                       bias_ptr=None, dbg: Debug | None = None, host: bool = False,
                       graph: bool = False, pre_norm: bool = False) -> None:
        """Raw pointers (device memory unless host=True); asynchronous on the set stream.
        graph=True replays a captured CUDA graph for repeated (layer, T, pointers)."""
        flags = (HOST_PTRS if host else 0) | (USE_GRAPH if graph else 0) | (PRE_NORM if pre_norm else 0)
        self._check(self.L.hymoe_forward(self.h, layer, x_ptr, resid_ptr, out_ptr, T, bias_ptr,
                                         C.byref(dbg) if dbg else None, flags))


def zipf_router_bias(seed: int, E: int, s: float = 1.1):
    """Router bias of the skewed expert-parallel workload: expected load follows a Zipf(s) law
    over a seeded permutation of the experts, p_r ∝ r^-s, bias_e = ln(E * p_rank(e)).  A
    workload generator (no reference counterpart: the reference has no router bias)."""
    import numpy as np
    rng = np.random.Generator(np.random.Philox(seed))
    perm = rng.permutation(E)
    r = np.arange(1, E + 1, dtype=np.float64)
    p = r ** (-s)
    p /= p.sum()
    bias = np.empty(E, np.float64)
    bias[perm] = np.log(E * p)
    return bias.astype(np.float32)
