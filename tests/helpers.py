"""Seeded synthetic inputs and parity metrics shared by the tests."""
from __future__ import annotations

import hashlib

import numpy as np

from oracle import oracle as O

# North-star tolerance for the FFN output (bf16 in / fp32 accumulate).
MAX_REL = 1e-2
MIN_COS = 0.9999


def parity(y: np.ndarray, y_ref: np.ndarray):
    """(normwise max rel err, cosine) of y against y_ref."""
    y = np.asarray(y, np.float64).ravel()
    r = np.asarray(y_ref, np.float64).ravel()
    den = np.abs(r).max()
    rel = float(np.abs(y - r).max() / den) if den > 0 else float(np.abs(y).max())
    nr, ny = np.linalg.norm(r), np.linalg.norm(y)
    cos = float(np.dot(y, r) / (nr * ny)) if nr > 0 and ny > 0 else (1.0 if nr == ny else 0.0)
    return rel, cos


def q_weights(qt: int, E: int, H: int, I: int, seed: int, scale_bf16: bool = False, std: float = 0.02):
    """Row-major quantised weights: fp32 N(0, std^2) -> Q8_0 (reference rule) or Q4_0 (harness rule)."""
    rng = np.random.default_rng(seed)
    wg = (rng.standard_normal((E, 2 * I, H), dtype=np.float32) * std).astype(np.float32)
    wd = (rng.standard_normal((E, H, I), dtype=np.float32) * std).astype(np.float32)
    if qt == 0:
        gq, gd = O.quantize_weight_q8_0(wg)
        dq, dd = O.quantize_weight_q8_0(wd)
    else:
        gq, gd = O.quantize_weight_q4_0(wg)
        dq, dd = O.quantize_weight_q4_0(wd)
    if scale_bf16:
        gd = O.f32_to_bf16_bits(O.f16_bits_to_f32(gd))
        dd = O.f32_to_bf16_bits(O.f16_bits_to_f32(dd))
    return gq, gd, dq, dd


def tokens(T: int, H: int, E: int, K: int, seed: int, bf16: bool = True):
    """(x bits uint16 [T,H], x as fp32, topk ids [T,K], topk weights [T,K]) with softmax-top-K routing."""
    rng = np.random.default_rng(seed + 7919)
    xf = rng.standard_normal((T, H), dtype=np.float32)
    bits = O.f32_to_bf16_bits(xf) if bf16 else O.f32_to_f16_bits(xf)
    xf = O.bf16_bits_to_f32(bits) if bf16 else O.f16_bits_to_f32(bits)
    logits = rng.standard_normal((T, E), dtype=np.float32)
    ids, w = O.topk_softmax(logits, K, True)
    return bits, xf, ids, w


def awq_weights(E: int, H: int, I: int, G: int, seed: int):
    """AWQ GEMM-packed weights with the BASELINE configs[2] distributions: q, z uniform in [0,15]
    (8 per int32), bf16 scales U(0.001, 0.01)."""
    rng = np.random.default_rng(seed)

    def words(shape):
        return rng.integers(0, 2 ** 32, size=shape, dtype=np.uint64).astype(np.uint32).view(np.int32)

    def scales(shape):
        return O.f32_to_bf16_bits(rng.uniform(0.001, 0.01, size=shape).astype(np.float32))

    w13_qw = words((E, H, 2 * I // 8))
    w13_sc = scales((E, H // G, 2 * I))
    w13_qz = words((E, H // G, 2 * I // 8))
    w2_qw = words((E, I, H // 8))
    w2_sc = scales((E, I // G, H))
    w2_qz = words((E, I // G, H // 8))
    return w13_qw, w13_sc, w13_qz, w2_qw, w2_sc, w2_qz


def expert_weights_fp32(e, seed, H, I):
    """fp32 N(0, 0.02^2) weights of expert e (independent stream per expert)."""
    rng = np.random.default_rng(seed * 100003 + e)
    wg = (rng.standard_normal((I, H), dtype=np.float32) * 0.02).astype(np.float32)
    wu = (rng.standard_normal((I, H), dtype=np.float32) * 0.02).astype(np.float32)
    wd = (rng.standard_normal((H, I), dtype=np.float32) * 0.02).astype(np.float32)
    return wg, wu, wd


def big_case_inputs(T, seed, H=2048, E=128, K=8):
    """Tokens of the full-size configs: bf16 N(0,1) hidden, softmax-top-K routing of N(0,1) logits."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H), dtype=np.float32)
    xb = O.f32_to_bf16_bits(x)
    logits = rng.standard_normal((T, E), dtype=np.float32)
    ids, w = O.topk_softmax(logits, K, True)
    return xb, ids, w


def digest_inputs(*arrays) -> str:
    """SHA-256 over the raw bytes of the generated inputs (checks generator stability)."""
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def random_q_weights(qt: int, E: int, H: int, I: int, seed: int):
    """Directly quantised random weights in the style of the reference's Q4_0 harness
    (test/fused_moe_cpu_int4.py:74-115): uniform quant words (Q4_0: 8 nibbles per uint32;
    Q8_0: int8 in [-127, 127]) and fp16 scales U(0,1) * s / sqrt(cols), s = 1/8 for Q4_0 and
    2/127 for Q8_0.  Cheap to regenerate at full E, unlike fp32 weights quantised per expert."""
    rng = np.random.default_rng(seed)

    def q(rows, cols):
        if qt == 1:
            return rng.integers(0, 2 ** 32, size=(E, rows, cols // 8), dtype=np.uint64).astype(np.uint32).view(np.int32)
        return rng.integers(-127, 128, size=(E, rows, cols), dtype=np.int8)

    def d(rows, cols):
        s = (1.0 / 8.0) if qt == 1 else (2.0 / 127.0)
        return O.f32_to_f16_bits((rng.random((E, rows, cols // 32), dtype=np.float32) * s / np.sqrt(cols)).astype(np.float32))

    gq = q(2 * I, H)
    gd = d(2 * I, H)
    dq = q(H, I)
    dd = d(H, I)
    return gq, gd, dq, dd


def golden_rows(T: int, n: int = 32) -> np.ndarray:
    """Token rows whose outputs a large-T golden fixture keeps: n rows spread over [0, T)."""
    if T <= n:
        return np.arange(T)
    return np.unique(np.linspace(0, T - 1, n).round().astype(np.int64))
