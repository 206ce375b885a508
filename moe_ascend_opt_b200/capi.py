"""ctypes view of the C ABI (include/moe_b200.h).

Device buffers are passed as raw addresses (``tensor.data_ptr()``); streams as
``torch.cuda.current_stream().cuda_stream``.  Every call checks the status and
raises :class:`MoeError` with ``moe_last_error()`` on failure.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmoe_b200.so")

MOE_OK, MOE_ERR_INVALID, MOE_ERR_CUDA, MOE_ERR_STATE, MOE_ERR_DEVICE = 0, -1, -2, -3, -4
Q8_0, Q4_0, AWQ = 0, 1, 2
REPLICATED = 1 << 30
F16, BF16, F32 = 0, 1, 2

# every symbol include/moe_b200.h declares
SYMBOLS = [
    "moe_engine_create", "moe_engine_destroy", "moe_engine_load_quantized", "moe_engine_quantize_store_expert",
    "moe_engine_load_awq", "moe_engine_forward", "moe_engine_reserve", "moe_engine_last_time_ms",
    "moe_engine_device_error", "moe_engine_export_expert", "moe_route_topk", "moe_route_permute",
    "moe_quantize_rows_q8_0", "moe_engine_debug_timeline", "moe_engine_forward_noalloc", "moe_last_error",
    "moe_engine_p2p_mailbox", "moe_engine_p2p_connect", "moe_engine_p2p_enable", "moe_engine_p2p_covers",
    "moe_engine_set_expert_map", "moe_route_gemm_topk", "moe_engine_save", "moe_engine_load_file",
    "moe_engine_set_replica_split", "moe_engine_forward_dense",
]


class MoeConfig(C.Structure):
    _fields_ = [("num_experts", C.c_int64), ("hidden_size", C.c_int64), ("intermediate_size", C.c_int64),
                ("quant_type", C.c_int32), ("group_size", C.c_int32), ("device", C.c_int32),
                ("expert_offset", C.c_int32)]


class MoeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


_lib = None
_P = C.c_void_p
_I64 = C.c_int64
_I32 = C.c_int32


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build with `python moe_ascend_opt_b200/build.py`")
        L = C.CDLL(LIB_PATH)
        L.moe_last_error.restype = C.c_char_p
        sig = {
            "moe_engine_create": [C.POINTER(MoeConfig), C.POINTER(_P)],
            "moe_engine_destroy": [_P],
            "moe_engine_load_quantized": [_P, _P, _P, _P, _P, _I32, _I32, _P],
            "moe_engine_quantize_store_expert": [_P, _I64, _I32, _P, _I32, _I32, _P],
            "moe_engine_load_awq": [_P, _P, _P, _P, _P, _P, _P, _I32, _P],
            "moe_engine_forward": [_P, _P, _P, _P, _P, _I64, _I64, _I32, _I32, _P],
            "moe_engine_reserve": [_P, _I64, _I64],
            "moe_engine_last_time_ms": [_P, C.POINTER(C.c_double)],
            "moe_engine_device_error": [_P, C.POINTER(_I32)],
            "moe_engine_export_expert": [_P, _I64, _I32, _P, _P],
            "moe_route_topk": [_P, _I64, _I64, _I64, _I32, _P, _P, _P],
            "moe_route_permute": [_P, _I64, _I64, _I64, _P, _P, _P, _P, _P],
            "moe_quantize_rows_q8_0": [_P, _I32, _I64, _I64, _P, _P, _P],
            "moe_engine_debug_timeline": [_P, _I32, _P, _I32, C.POINTER(_I32)],
            "moe_engine_forward_noalloc": [_P, _P, _P, _P, _P, _I64, _I64, _I32, _I32, _P],
            "moe_engine_p2p_mailbox": [_P, _I32, _I64, _P],
            "moe_engine_p2p_connect": [_P, _I32, _I32, _P],
            "moe_engine_p2p_enable": [_P, _I32],
            "moe_engine_p2p_covers": [_P, _I64],
            "moe_engine_set_expert_map": [_P, _P, _I64],
            "moe_route_gemm_topk": [_P, _I32, _P, _I32, _I64, _I64, _I64, _I64, _I32, _P, _P, _P, _P],
            "moe_engine_save": [_P, C.c_char_p],
            "moe_engine_set_replica_split": [_P, _I32, _I32],
            "moe_engine_forward_dense": [_P, _I64, _P, _P, _I64, _I32, _I32, _P],
            "moe_engine_load_file": [_P, C.c_char_p],
        }
        for name, args in sig.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = C.c_int
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != MOE_OK:
        raise MoeError(rc, lib().moe_last_error().decode())


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))


def stream_handle(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def route_gemm_topk(hidden, router_w, top_k, renormalize=True, logits=None, stream=None):
    """moe_route_gemm_topk on CUDA tensors: (ids int32 [T,K], weights fp32 [T,K])."""
    import torch
    T, H = hidden.shape
    E = router_w.shape[0]
    ids = torch.empty((T, top_k), dtype=torch.int32, device=hidden.device)
    w = torch.empty((T, top_k), dtype=torch.float32, device=hidden.device)
    code = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}
    call("moe_route_gemm_topk", hidden.data_ptr(), code[hidden.dtype], router_w.data_ptr(), code[router_w.dtype], T, H, E,
         top_k, int(renormalize), ids.data_ptr(), w.data_ptr(), logits.data_ptr() if logits is not None else None,
         stream_handle(stream))
    return ids, w


class Engine:
    """Thin owner of a moe_engine*; the methods mirror the C entry points."""

    def __init__(self, E, H, I, quant_type, device=0, group_size=128, expert_offset=0):
        cfg = MoeConfig(E, H, I, quant_type, group_size, device, expert_offset)
        h = C.c_void_p()
        call("moe_engine_create", C.byref(cfg), C.byref(h))
        self.h = h
        self.E, self.H, self.I, self.qt, self.device = E, H, I, quant_type, device

    def load_quantized(self, gu_qs, gu_d, dn_qs, dn_d, scale_dtype, stream=None):
        on_dev = int(gu_qs.is_cuda)
        call("moe_engine_load_quantized", self.h, gu_qs.data_ptr(), gu_d.data_ptr(), dn_qs.data_ptr(),
             dn_d.data_ptr(), scale_dtype, on_dev, stream_handle(stream))

    def quantize_store_expert(self, e, proj, w, w_dtype, stream=None):
        call("moe_engine_quantize_store_expert", self.h, e, proj, w.data_ptr(), w_dtype, int(w.is_cuda),
             stream_handle(stream))

    def load_awq(self, w13_qw, w13_sc, w13_qz, w2_qw, w2_sc, w2_qz, stream=None):
        call("moe_engine_load_awq", self.h, w13_qw.data_ptr(), w13_sc.data_ptr(), w13_qz.data_ptr(),
             w2_qw.data_ptr(), w2_sc.data_ptr(), w2_qz.data_ptr(), int(w13_qw.is_cuda), stream_handle(stream))

    def forward(self, x, y, ids, w, act_dtype, out_dtype, stream=None):
        call("moe_engine_forward", self.h, x.data_ptr(), y.data_ptr(), ids.data_ptr(), w.data_ptr(),
             x.shape[0], ids.shape[1], act_dtype, out_dtype, stream_handle(stream))

    def forward_noalloc(self, x, y, ids, w, act_dtype, out_dtype, stream=None):
        call("moe_engine_forward_noalloc", self.h, x.data_ptr(), y.data_ptr(), ids.data_ptr(), w.data_ptr(),
             x.shape[0], ids.shape[1], act_dtype, out_dtype, stream_handle(stream))

    def set_expert_map(self, local_of_global):
        import numpy as np
        m = np.ascontiguousarray(local_of_global, np.int32)
        call("moe_engine_set_expert_map", self.h, m.ctypes.data, m.size)

    def set_replica_split(self, rank, world):
        call("moe_engine_set_replica_split", self.h, rank, world)

    def forward_dense(self, expert, x, y, act_dtype, out_dtype, stream=None):
        call("moe_engine_forward_dense", self.h, expert, x.data_ptr(), y.data_ptr(), x.shape[0], act_dtype, out_dtype,
             stream_handle(stream))

    def save(self, path):
        call("moe_engine_save", self.h, os.fsencode(path))

    def load_file(self, path):
        call("moe_engine_load_file", self.h, os.fsencode(path))

    def reserve(self, T, K):
        call("moe_engine_reserve", self.h, T, K)

    def last_time_ms(self) -> float:
        v = C.c_double()
        call("moe_engine_last_time_ms", self.h, C.byref(v))
        return v.value

    def device_error(self) -> int:
        v = C.c_int32()
        call("moe_engine_device_error", self.h, C.byref(v))
        return v.value

    def export_expert(self, e, which, qs_out, d_out):
        call("moe_engine_export_expert", self.h, e, which, qs_out.ctypes.data, d_out.ctypes.data)

    def timeline(self, enable=None):
        """Enable/disable per-CTA phase stamps, or (enable=None) fetch the last launch's [CTAs, 20] stamps."""
        import numpy as np
        n = C.c_int32()
        if enable is not None:
            call("moe_engine_debug_timeline", self.h, int(enable), None, 0, C.byref(n))
            return None
        call("moe_engine_debug_timeline", self.h, 1, None, 0, C.byref(n))
        out = np.zeros(n.value, np.uint64)
        call("moe_engine_debug_timeline", self.h, 1, out.ctypes.data, n.value, C.byref(n))
        return out.reshape(-1, 20)

    def close(self):
        if self.h:
            lib().moe_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
