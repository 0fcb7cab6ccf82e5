"""ctypes bindings for the CPU checkers (TEST INFRASTRUCTURE ONLY).

`Oracle` wraps liboracle.so, the C restatement of the reference MoE path
(hymoe_oracle.c).  `RefMoE` wraps oracle/_ref/libhyref.so, the reference's own
src/attention.cpp + src/rms_norm.cpp compiled here (moe_forward_cpu,
src/attention.cpp:191-313).  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference legs import this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_ORACLE = os.path.join(HERE, "liboracle.so")
LIB_REF = os.path.join(HERE, "_ref", "libhyref.so")

F32, F16, Q4_0, Q8_0 = 0, 1, 2, 8
KIND_ROUTER, KIND_GATE_UP, KIND_DOWN, KIND_BIAS, KIND_X = 1, 2, 3, 4, 5
SHARED_INDEX = 0xFFFF

_fp = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)
_i32p = C.POINTER(C.c_int32)


def stream_id(layer: int, kind: int, index: int = 0) -> int:
    return (layer << 32) | (kind << 16) | index


def type_nbytes(t: int, n: int) -> int:
    return {F32: 4 * n, F16: 2 * n, Q4_0: n // 32 * 18, Q8_0: n // 32 * 34}[t]


def _ptr(a: np.ndarray | None, ty):
    if a is None:
        return None
    assert a.flags.c_contiguous
    return a.ctypes.data_as(ty)


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def reference_dir() -> str | None:
    """The reference checkout the checkers compile: $HYMOE_REFERENCE, else a checkout named
    `reference` beside this repository; None when neither holds the reference's src/."""
    env = os.environ.get("HYMOE_REFERENCE")
    cands = [env] if env else [os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")]
    for d in cands:
        if d and os.path.isdir(os.path.join(d, "src")):
            return d
    return None


def build(ref: bool | None = None) -> None:
    """Compile liboracle.so (and the reference checker when its sources exist)."""
    targets = ["oracle"]
    refdir = reference_dir()
    if ref is None:
        ref = refdir is not None
    if ref and refdir is None:
        raise RuntimeError("the reference checkout was not found: set HYMOE_REFERENCE")
    if ref:
        targets += ["ref", "ref-gpu"]
    subprocess.run(["make", "-s", "-C", HERE, *([f"REF={refdir}"] if ref else []), *targets], check=True)


class Oracle:
    def __init__(self, nthreads: int | None = None):
        if not os.path.exists(LIB_ORACLE):
            build(ref=False)
        L = C.CDLL(LIB_ORACLE)
        self.L = L
        self.nthreads = nthreads or default_threads()
        u64, u32, i32 = C.c_uint64, C.c_uint32, C.c_int
        L.oracle_philox4x32_10.argtypes = [C.POINTER(C.c_uint32)] * 3
        L.oracle_synth_scale.argtypes = [C.c_float]
        L.oracle_synth_scale.restype = C.c_float
        L.oracle_fill_normal.argtypes = [_fp, u64, u64, u64, C.c_float, i32]
        L.oracle_f32_to_f16.argtypes = [C.c_float]
        L.oracle_f32_to_f16.restype = C.c_uint16
        L.oracle_f16_to_f32.argtypes = [C.c_uint16]
        L.oracle_f16_to_f32.restype = C.c_float
        L.oracle_quantize.argtypes = [i32, _fp, _u8p, u64]
        L.oracle_dequantize.argtypes = [i32, _u8p, _fp, u64]
        L.oracle_synth_tensor.argtypes = [i32, _u8p, u64, u64, u64, C.c_float, i32]
        L.oracle_synth_tensor_f32.argtypes = [i32, _fp, u64, u64, u64, C.c_float, i32]
        L.oracle_rms_norm.argtypes = [_fp, _fp, _fp, u32, u32, C.c_float]
        L.oracle_topkgating_full.argtypes = [_fp, u32, u32, u32, C.c_int, u32, u32, C.c_int, C.c_float,
                                             u32, C.c_int, C.c_float, _fp, _i32p, _fp, _u8p, _i32p,
                                             C.POINTER(u32)]
        L.oracle_topkgating_full.restype = None
        L.oracle_swiglu_ffn.argtypes = [_fp, _fp, _fp, _fp, u32, u32, u32, i32]
        L.oracle_router.argtypes = [_fp, u32, u32, u32, u32, _fp, _fp, _fp, _fp, _fp, _i32p, i32]
        L.oracle_moe_forward.argtypes = [_fp, _fp, u32, u32, u32, u32, u32, _fp, _fp, _fp, _fp,
                                         C.POINTER(_fp), C.POINTER(_fp), _fp, _fp, _fp, _fp,
                                         _i32p, i32]
        L.oracle_moe_forward.restype = C.c_int

    # -- generator / formats -------------------------------------------------
    def philox(self, ctr, key) -> np.ndarray:
        c = (C.c_uint32 * 4)(*ctr)
        k = (C.c_uint32 * 2)(*key)
        o = (C.c_uint32 * 4)()
        self.L.oracle_philox4x32_10(c, k, o)
        return np.array(list(o), dtype=np.uint32)

    def fill_normal(self, n: int, seed: int, stream: int, std: float) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        self.L.oracle_fill_normal(_ptr(out, _fp), n, seed, stream, std, self.nthreads)
        return out

    def quantize(self, t: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        out = np.empty(type_nbytes(t, x.size), dtype=np.uint8)
        self.L.oracle_quantize(t, _ptr(x, _fp), _ptr(out, _u8p), x.size)
        return out

    def dequantize(self, t: int, raw: np.ndarray, n: int) -> np.ndarray:
        raw = np.ascontiguousarray(raw, dtype=np.uint8).ravel()
        out = np.empty(n, dtype=np.float32)
        self.L.oracle_dequantize(t, _ptr(raw, _u8p), _ptr(out, _fp), n)
        return out

    def synth_tensor(self, t: int, n: int, seed: int, stream: int, std: float) -> np.ndarray:
        out = np.empty(type_nbytes(t, n), dtype=np.uint8)
        self.L.oracle_synth_tensor(t, _ptr(out, _u8p), n, seed, stream, std, self.nthreads)
        return out

    def synth_tensor_f32(self, t: int, n: int, seed: int, stream: int, std: float) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        self.L.oracle_synth_tensor_f32(t, _ptr(out, _fp), n, seed, stream, std, self.nthreads)
        return out

    # -- maths ---------------------------------------------------------------
    def rms_norm(self, x: np.ndarray, w: np.ndarray, eps: float = 1e-5) -> np.ndarray:
        T, H = x.shape
        out = np.empty_like(x)
        self.L.oracle_rms_norm(_ptr(x, _fp), _ptr(w, _fp), _ptr(out, _fp), T, H, eps)
        return out

    def topkgating_full(self, logits: np.ndarray, K: int, group=None, drop=None, min_capacity: int = 8,
                        norm_topk_prob: bool = True, scale: float = 1.0) -> dict:
        """FULL-mode routing (topkgating_full, src/hunyuan_moe_full.cpp:119-350).
        group = (n_group, topk_group) for group-limited greedy; drop = capacity_factor to
        drop pairs beyond a fixed capacity (None: capacity = the largest expert count)."""
        logits = np.ascontiguousarray(logits, np.float32)
        T, E = logits.shape
        probs = np.empty((T, E), np.float32)
        idx = np.empty((T, K), np.int32)
        w = np.empty((T, K), np.float32)
        keep = np.empty((T, K), np.uint8)
        cnt = np.empty(E, np.int32)
        cap = C.c_uint32()
        ng, tg = group if group else (0, 0)
        self.L.oracle_topkgating_full(_ptr(logits, _fp), T, E, K, 1 if group else 0, ng, tg,
                                      0 if drop is None else 1, 1.0 if drop is None else drop,
                                      min_capacity, 1 if norm_topk_prob else 0, scale, _ptr(probs, _fp),
                                      _ptr(idx, _i32p), _ptr(w, _fp), _ptr(keep, _u8p), _ptr(cnt, _i32p),
                                      C.byref(cap))
        return dict(probs=probs, idx=idx, w=w, keep=keep.astype(bool), exp_counts=cnt, capacity=cap.value)

    def swiglu_ffn(self, x, gu, dn, I: int) -> np.ndarray:
        n, H = x.shape
        out = np.empty((n, H), dtype=np.float32)
        self.L.oracle_swiglu_ffn(_ptr(x, _fp), _ptr(gu, _fp), _ptr(dn, _fp), _ptr(out, _fp),
                                 n, H, I, self.nthreads)
        return out

    def router(self, x, router_w, K: int, bias=None):
        T, H = x.shape
        E = router_w.shape[0]
        logits = np.empty((T, E), np.float32)
        probs = np.empty((T, E), np.float32)
        tw = np.empty((T, K), np.float32)
        ti = np.empty((T, K), np.int32)
        self.L.oracle_router(_ptr(x, _fp), T, H, E, K, _ptr(router_w, _fp), _ptr(bias, _fp),
                             _ptr(logits, _fp), _ptr(probs, _fp), _ptr(tw, _fp),
                             _ptr(ti, _i32p), self.nthreads)
        return logits, probs, tw, ti

    def moe_forward(self, x, router_w, shared_gu, shared_dn, experts_gu, experts_dn, K: int,
                    I: int, bias=None, resid=None):
        """experts_gu/dn: lists of E arrays (or None for experts no token selects)."""
        T, H = x.shape
        E = router_w.shape[0]
        gu_arr = (_fp * E)(*[_ptr(a, _fp) for a in experts_gu])
        dn_arr = (_fp * E)(*[_ptr(a, _fp) for a in experts_dn])
        out = np.empty((T, H), np.float32)
        logits = np.empty((T, E), np.float32)
        probs = np.empty((T, E), np.float32)
        tw = np.empty((T, K), np.float32)
        ti = np.empty((T, K), np.int32)
        rc = self.L.oracle_moe_forward(_ptr(x, _fp), _ptr(resid, _fp), T, H, I, E, K,
                                       _ptr(router_w, _fp), _ptr(bias, _fp),
                                       _ptr(shared_gu, _fp), _ptr(shared_dn, _fp), gu_arr, dn_arr,
                                       _ptr(out, _fp), _ptr(logits, _fp), _ptr(probs, _fp),
                                       _ptr(tw, _fp), _ptr(ti, _i32p), self.nthreads)
        if rc != 0:
            raise RuntimeError("oracle_moe_forward: a selected expert has no weights")
        return dict(out=out, logits=logits, probs=probs, w=tw, idx=ti)


class RefMoE:
    """The reference's own moe_forward_cpu (src/attention.cpp:191-313), single-threaded
    as written."""

    def __init__(self):
        if not os.path.exists(LIB_REF):
            build(ref=True)
        L = C.CDLL(LIB_REF)
        self.L = L
        u32 = C.c_uint32
        L.hyref_weights_create.argtypes = [u32, u32, u32, _fp, _fp, _fp, C.POINTER(_fp),
                                           C.POINTER(_fp)]
        L.hyref_weights_create.restype = C.c_void_p
        L.hyref_weights_destroy.argtypes = [C.c_void_p]
        L.hyref_moe_forward.argtypes = [_fp, C.c_void_p, u32, u32, u32, u32, _fp, _fp, _fp,
                                        _i32p]
        L.hyref_swiglu_ffn.argtypes = [_fp, _fp, _fp, _fp, u32, u32, u32]
        L.hyref_rms_norm.argtypes = [_fp, _fp, _fp, u32, u32, C.c_float]
        L.hyref_full_capacity_bound.argtypes = [u32, u32, u32, C.c_int, C.c_float, u32]
        L.hyref_full_capacity_bound.restype = u32
        L.hyref_topkgating_full.argtypes = [_fp, u32, u32, u32, C.c_int, u32, u32, C.c_int, C.c_float, u32,
                                            C.c_int, C.c_float, _fp, _u8p, _fp, _i32p, C.POINTER(u32),
                                            C.POINTER(C.c_float)]
        L.hyref_topkgating_full.restype = C.c_int

    @staticmethod
    def available() -> bool:
        return os.path.exists(LIB_REF)

    def weights(self, H, I, router_w, shared_gu, shared_dn, experts_gu, experts_dn):
        E = router_w.shape[0]
        gu_arr = (_fp * E)(*[_ptr(a, _fp) for a in experts_gu])
        dn_arr = (_fp * E)(*[_ptr(a, _fp) for a in experts_dn])
        h = self.L.hyref_weights_create(H, I, E, _ptr(router_w, _fp), _ptr(shared_gu, _fp),
                                        _ptr(shared_dn, _fp), gu_arr, dn_arr)
        return h

    def free(self, h) -> None:
        self.L.hyref_weights_destroy(h)

    def moe_forward(self, x, handle, E: int, H: int, I: int, K: int):
        T = x.shape[0]
        out = np.empty((T, H), np.float32)
        probs = np.empty((T, E), np.float32)
        tw = np.empty((T, K), np.float32)
        ti = np.empty((T, K), np.int32)
        self.L.hyref_moe_forward(_ptr(x, _fp), handle, T, H, I, K, _ptr(out, _fp),
                                 _ptr(probs, _fp), _ptr(tw, _fp), _ptr(ti, _i32p))
        return dict(out=out, probs=probs, w=tw, idx=ti)

    def topkgating_full(self, logits: np.ndarray, K: int, group=None, drop=None, min_capacity: int = 8,
                        norm_topk_prob: bool = True, scale: float = 1.0) -> dict:
        """The reference's topkgating_full (src/hunyuan_moe_full.cpp:119-350): probs, the
        dispatch mask and combine weights [T, E, capacity], expert counts, capacity, rate."""
        logits = np.ascontiguousarray(logits, np.float32)
        T, E = logits.shape
        dt = 0 if drop is None else 1
        cf = 1.0 if drop is None else drop
        bound = self.L.hyref_full_capacity_bound(T, E, K, dt, cf, min_capacity)
        probs = np.empty((T, E), np.float32)
        mask = np.zeros(T * E * bound, np.uint8)
        comb = np.zeros(T * E * bound, np.float32)
        cnt = np.empty(E, np.int32)
        cap = C.c_uint32()
        rate = C.c_float()
        ng, tg = group if group else (0, 0)
        rc = self.L.hyref_topkgating_full(_ptr(logits, _fp), T, E, K, 1 if group else 0, ng, tg, dt, cf,
                                          min_capacity, 1 if norm_topk_prob else 0, scale, _ptr(probs, _fp),
                                          _ptr(mask, _u8p), _ptr(comb, _fp), _ptr(cnt, _i32p), C.byref(cap),
                                          C.byref(rate))
        if rc != 0:
            raise RuntimeError("topkgating_full computed a capacity above the bound")
        c = cap.value
        return dict(probs=probs, mask=mask[:T * E * c].reshape(T, E, c).astype(bool),
                    combine=comb[:T * E * c].reshape(T, E, c), exp_counts=cnt, capacity=c,
                    rate=rate.value)

    def rms_norm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        """The reference's rms_norm_f32 (src/rms_norm.cpp:9-33)."""
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        out = np.empty_like(x)
        self.L.hyref_rms_norm(_ptr(x, _fp), _ptr(w, _fp), _ptr(out, _fp), x.shape[0], x.shape[1], eps)
        return out


def synth_layer_f32(orc: Oracle, seed: int, layer: int, H: int, I: int, E: int, wtype: int,
                    std: float = 0.02, experts=None):
    """F32 weights of one synthetic layer as the oracle consumes them (quantised to
    `wtype` and dequantised with the standard GGUF rule).  The router stays F32.
    `experts` limits generation to a subset (others are None)."""
    rw = orc.fill_normal(E * H, seed, stream_id(layer, KIND_ROUTER), std).reshape(E, H)
    sgu = orc.synth_tensor_f32(wtype, 2 * I * H, seed,
                               stream_id(layer, KIND_GATE_UP, SHARED_INDEX), std)
    sdn = orc.synth_tensor_f32(wtype, H * I, seed, stream_id(layer, KIND_DOWN, SHARED_INDEX), std)
    want = set(range(E)) if experts is None else set(int(e) for e in experts)
    egu, edn = [], []
    for e in range(E):
        if e in want:
            egu.append(orc.synth_tensor_f32(wtype, 2 * I * H, seed,
                                            stream_id(layer, KIND_GATE_UP, e), std))
            edn.append(orc.synth_tensor_f32(wtype, H * I, seed, stream_id(layer, KIND_DOWN, e),
                                            std))
        else:
            egu.append(None)
            edn.append(None)
    return rw, sgu, sdn, egu, edn


def synth_x(orc: Oracle, seed: int, T: int, H: int, layer: int = 0) -> np.ndarray:
    return orc.fill_normal(T * H, seed, stream_id(layer, KIND_X), 1.0).reshape(T, H)


def synth_bias(orc: Oracle, seed: int, E: int, std: float = 0.5, layer: int = 0) -> np.ndarray:
    return orc.fill_normal(E, seed, stream_id(layer, KIND_BIAS), std)


def zipf_bias(seed: int, E: int, s: float = 1.1) -> np.ndarray:
    """Router bias that skews expected load by a Zipf(s) law over a seeded permutation
    of the experts: p_r ∝ r^-s, bias_e = ln(E * p_rank(e))."""
    rng = np.random.Generator(np.random.Philox(seed))
    perm = rng.permutation(E)
    r = np.arange(1, E + 1, dtype=np.float64)
    p = r ** (-s)
    p /= p.sum()
    bias = np.empty(E, np.float64)
    bias[perm] = np.log(E * p)
    return bias.astype(np.float32)
