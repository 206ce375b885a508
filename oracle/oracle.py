"""TEST INFRASTRUCTURE ONLY -- the parity checker, never the product.

ctypes wrappers around

* ``oracle/_build/libmoe_oracle.so`` -- the plain-C restatement of the
  reference algorithm (``oracle/moe_oracle.c``; each function there cites the
  reference lines it follows), and
* ``oracle/_ref/ref_bridge.so`` -- extern "C" entry points into the reference
  CPU engine compiled unmodified from its own sources (``oracle/Makefile``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline /
reference legs import this module.  The product package never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libmoe_oracle.so")
REF_BRIDGE_SO = os.path.join(HERE, "_ref", "ref_bridge.so")
REF_EXT_SO = os.path.join(HERE, "_ref", "nanovllm_ext_ref.so")
# The reference's Int8-gemm source directory: the REF environment variable, else a checkout
# named `reference` beside this repository (absent on machines that only run the prebuilt files).
REF_SRC = os.environ.get("REF") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference", "Int8-gemm")

_P = C.c_void_p
_lib = None
_ref = None


def build(with_reference: bool = True) -> None:
    """Compile the C oracle, and the reference objects when the reference checkout exists."""
    targets = ["oracle"]
    if with_reference and os.path.isdir(REF_SRC):
        targets.append("ref")
    subprocess.check_call(["make", "-s", "-C", HERE, "-j4", "REF=" + REF_SRC] + targets)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build(with_reference=False)
        _lib = C.CDLL(ORACLE_SO)
        _lib.orc_route_preprocess.restype = C.c_int
        _lib.orc_quantize_block_q8_0.restype = C.c_float
    return _lib


def have_reference() -> bool:
    return os.path.exists(REF_BRIDGE_SO)


def ref() -> C.CDLL:
    """The reference engine bridge (tp = 1: NANOVLLM_TP_SIZE is set to 1 here)."""
    global _ref
    if _ref is None:
        os.environ["NANOVLLM_TP_SIZE"] = "1"
        import torch  # noqa: F401  (loads libtorch, the bridge's dependency)
        _ref = C.CDLL(REF_BRIDGE_SO)
        _ref.ref_last_error.restype = C.c_char_p
        _ref.ref_route_preprocess.restype = C.c_int
        _ref.ref_quantize_block.restype = C.c_float
        _ref.ref_engine_create.restype = _P
        _ref.ref_engine_create.argtypes = [C.c_int64, C.c_int64, C.c_int64, C.c_int]
        _ref.ref_engine_destroy.argtypes = [_P]
        _ref.ref_engine_store_repack.argtypes = [_P, C.c_int, C.c_int, _P, _P, _P, _P]
        _ref.ref_engine_quantize_store.argtypes = [_P, C.c_int64, C.c_char_p, _P, C.c_int64, C.c_int64]
        _ref.ref_engine_forward.argtypes = [_P, _P, _P, _P, _P, C.c_int64, C.c_int64, C.c_int]
        _ref.ref_engine_last_ms.restype = C.c_double
        _ref.ref_engine_last_ms.argtypes = [_P]
        _ref.ref_quantize_weight.argtypes = [_P, C.c_int64, C.c_int64, _P, _P]
    return _ref


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_P)


# ---------------------------------------------------------------- conversions
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_bf16(_ptr(x), _ptr(out), C.c_int64(x.size))
    return out


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_f16(_ptr(x), _ptr(out), C.c_int64(x.size))
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def f16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(b, dtype=np.uint16).view(np.float16).astype(np.float32)


# ---------------------------------------------------------------- routing
def _route(fn, ids, E):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, K = ids.shape
    counts = np.zeros(E, np.int32)
    starts = np.zeros(E + 1, np.int32)
    tmap = np.zeros((max(T * K, 1), 2), np.int32)
    smap = np.zeros(max(T * K, 1), np.int32)
    P = fn(E, K, T, _ptr(ids), _ptr(counts), _ptr(starts), _ptr(tmap), _ptr(smap))
    if P < 0:
        raise RuntimeError(ref().ref_last_error().decode())
    return counts, starts, tmap[:P].copy(), smap[: T * K].reshape(T, K).copy()


def route_preprocess(ids: np.ndarray, E: int):
    """Stable counting sort (moe_common.cpp:146-184): counts, starts, token_map[P,2], scatter_map[T,K]."""
    return _route(lib().orc_route_preprocess, ids, E)


def ref_route_preprocess(ids: np.ndarray, E: int):
    """The reference's own moe::preprocess_moe_routing (top_k in {1,8,10} only)."""
    return _route(ref().ref_route_preprocess, ids, E)


def topk_softmax(logits: np.ndarray, K: int, renormalize: bool = True):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    ids = np.zeros((T, K), np.int32)
    w = np.zeros((T, K), np.float32)
    lib().orc_topk_softmax(_ptr(logits), T, E, K, int(renormalize), _ptr(ids), _ptr(w))
    return ids, w


# ---------------------------------------------------------------- quantisation
def quantize_rows_q8_0(x: np.ndarray):
    """Activation rows -> (qs int8 [R,C], d fp32 [R,C/32])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    R, Cc = x.shape
    qs = np.empty((R, Cc), np.int8)
    d = np.empty((R, Cc // 32), np.float32)
    lib().orc_quantize_rows_q8_0_f32scale(_ptr(x), C.c_int64(R), C.c_int64(Cc), _ptr(qs), _ptr(d))
    return qs, d


def ref_quantize_rows_q8_0(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    R, Cc = x.shape
    qs = np.empty((R, Cc), np.int8)
    d = np.empty((R, Cc // 32), np.float32)
    r = ref()
    out = np.empty(32, np.int8)
    for i in range(R):
        for b in range(Cc // 32):
            blk = np.ascontiguousarray(x[i, b * 32:(b + 1) * 32])
            d[i, b] = r.ref_quantize_block(_ptr(blk), _ptr(out))
            qs[i, b * 32:(b + 1) * 32] = out
    return qs, d


def quantize_weight_q8_0(w: np.ndarray):
    """fp32 [..., N, K] -> (int8 [..., N, K], fp16 bits [..., N, K/32])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    shp = w.shape
    R, Kc = int(np.prod(shp[:-1])), shp[-1]
    qs = np.empty(shp, np.int8)
    d = np.empty(shp[:-1] + (Kc // 32,), np.uint16)
    lib().orc_quantize_weight_q8_0(_ptr(w), C.c_int64(R), C.c_int64(Kc), _ptr(qs), _ptr(d))
    return qs, d


def ref_quantize_weight_q8_0(w: np.ndarray):
    w = np.ascontiguousarray(w, dtype=np.float32)
    shp = w.shape
    R, Kc = int(np.prod(shp[:-1])), shp[-1]
    qs = np.empty(shp, np.int8)
    d = np.empty(shp[:-1] + (Kc // 32,), np.uint16)
    if ref().ref_quantize_weight(_ptr(w), R, Kc, _ptr(qs), _ptr(d)) != 0:
        raise RuntimeError(ref().ref_last_error().decode())
    return qs, d


def quantize_weight_q4_0(w: np.ndarray):
    """fp32 [..., N, K] -> (packed int32 [..., N, K/8], fp16 bits [..., N, K/32])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    shp = w.shape
    R, Kc = int(np.prod(shp[:-1])), shp[-1]
    qs = np.empty(shp[:-1] + (Kc // 8,), np.int32)
    d = np.empty(shp[:-1] + (Kc // 32,), np.uint16)
    lib().orc_quantize_weight_q4_0(_ptr(w), C.c_int64(R), C.c_int64(Kc), _ptr(qs), _ptr(d))
    return qs, d


def decode_q(quant_type: int, qs: np.ndarray, rows: int, cols: int) -> np.ndarray:
    qs = np.ascontiguousarray(qs)
    out = np.empty((rows, cols), np.int8)
    lib().orc_decode_q(quant_type, _ptr(qs), C.c_int64(rows), C.c_int64(cols), _ptr(out))
    return out


# ---------------------------------------------------------------- forward
def moe_forward_q(quant_type, scale_is_bf16, x_f32, ids, topk_w, gu_qs, gu_d, dn_qs, dn_d, want_h=False):
    """C restatement of the Q8_0/Q4_0 fused forward (fp32 output before the final cast)."""
    x_f32 = np.ascontiguousarray(x_f32, np.float32)
    ids = np.ascontiguousarray(ids, np.int32)
    topk_w = np.ascontiguousarray(topk_w, np.float32)
    T, H = x_f32.shape
    K = ids.shape[1]
    E = gu_d.shape[0]
    I = gu_d.shape[1] // 2
    y = np.zeros((T, H), np.float32)
    h = np.zeros((max(T * K, 1), I), np.float32) if want_h else None
    arrs = [np.ascontiguousarray(a) for a in (gu_qs, gu_d, dn_qs, dn_d)]
    lib().orc_moe_forward_q(quant_type, int(scale_is_bf16), E, H, I, T, K, _ptr(x_f32), _ptr(ids),
                            _ptr(topk_w), *[_ptr(a) for a in arrs], _ptr(y), _ptr(h) if want_h else None)
    return (y, h) if want_h else y


def moe_forward_awq(x_f32, ids, topk_w, w13_qw, w13_sc, w13_qz, w2_qw, w2_sc, w2_qz, group=128):
    x_f32 = np.ascontiguousarray(x_f32, np.float32)
    ids = np.ascontiguousarray(ids, np.int32)
    topk_w = np.ascontiguousarray(topk_w, np.float32)
    T, H = x_f32.shape
    K = ids.shape[1]
    E = w13_qw.shape[0]
    I = w2_qw.shape[1]
    y = np.zeros((T, H), np.float32)
    a = [np.ascontiguousarray(v) for v in (w13_qw, w13_sc, w13_qz, w2_qw, w2_sc, w2_qz)]
    lib().orc_moe_forward_awq(E, H, I, group, T, K, _ptr(x_f32), _ptr(ids), _ptr(topk_w),
                              *[_ptr(v) for v in a], _ptr(y))
    return y


def awq_dequant(qw, sc, qz, group=128):
    """One expert's [K, N] AWQ matrix -> fp32 W[N, K]."""
    qw, sc, qz = (np.ascontiguousarray(v) for v in (qw, sc, qz))
    Kd, N = qw.shape[0], qw.shape[1] * 8
    W = np.empty((N, Kd), np.float32)
    lib().orc_awq_dequant(_ptr(qw), _ptr(sc), _ptr(qz), C.c_int64(Kd), C.c_int64(N), group, _ptr(W))
    return W


class RefEngine:
    """The reference MoEInfer engine (tp = 1) driven through the extern "C" bridge."""

    def __init__(self, E, H, I, quant_type):
        self.r = ref()
        self.h = self.r.ref_engine_create(E, H, I, quant_type)
        if not self.h:
            raise RuntimeError(self.r.ref_last_error().decode())
        self.qt = quant_type

    def store_repack(self, scale_is_bf16, gu_qs, gu_d, dn_qs, dn_d):
        arrs = [np.ascontiguousarray(a) for a in (gu_qs, gu_d, dn_qs, dn_d)]
        if self.r.ref_engine_store_repack(self.h, self.qt, int(scale_is_bf16), *[_ptr(a) for a in arrs]):
            raise RuntimeError(self.r.ref_last_error().decode())

    def quantize_store(self, e, proj, w):
        w = np.ascontiguousarray(w, np.float32)
        if self.r.ref_engine_quantize_store(self.h, e, proj.encode(), _ptr(w), w.shape[0], w.shape[1]):
            raise RuntimeError(self.r.ref_last_error().decode())

    def forward(self, x_bits: np.ndarray, ids, topk_w, act_is_bf16=True) -> np.ndarray:
        """x_bits: uint16 [T,H] bf16/fp16 bits.  Returns the uint16 output bits."""
        x_bits = np.ascontiguousarray(x_bits, np.uint16)
        ids = np.ascontiguousarray(ids, np.int32)
        topk_w = np.ascontiguousarray(topk_w, np.float32)
        T, K = ids.shape
        y = np.zeros_like(x_bits)
        if self.r.ref_engine_forward(self.h, _ptr(x_bits), _ptr(y), _ptr(ids), _ptr(topk_w), T, K,
                                     int(act_is_bf16)):
            raise RuntimeError(self.r.ref_last_error().decode())
        return y

    def last_ms(self) -> float:
        return self.r.ref_engine_last_ms(self.h)

    def close(self):
        if self.h:
            self.r.ref_engine_destroy(self.h)
            self.h = None
