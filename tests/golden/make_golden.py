"""Generate the golden fixtures of tests/golden/ from the REFERENCE implementation.

Runs the reference CPU engine compiled unmodified from its own sources
(oracle/_ref/ref_bridge.so, built by `make -C oracle ref` where the reference
checkout exists) on seeded inputs and stores its outputs.  The inputs are NOT
stored: tests regenerate them from the seeds with tests/helpers.py and check a
SHA-256 of the regenerated arrays against the one recorded here.

    python tests/golden/make_golden.py

Fixtures:
  route_k{1,8,10}.npz      preprocess_moe_routing (moe_common.cpp:146-216)
  xquant.npz               quantize_block_q8_0 on activations (gemm_kernels.cpp:25-58)
  wquant.npz               quantize_weight_only (q8_gemm.cpp:219-260)
  fwd_*.npz                MoEInfer forward, small shapes, Q8_0/Q4_0, f16/bf16 scales
  fwd_c1_q8.npz            BASELINE configs[0]: H2048 I768 E128 top8 T=1, Q8_0 from fp32 N(0,.02^2)
  fwd_c2_q4_T{1,4,8,32}    BASELINE configs[1]: same shape, Q4_0, token sweep
  big_*.npz                large token counts at the sizes where the grouped GEMMs run by default
                           (Qwen Q4_0/Q8_0 T=128/512/1024/4096, MiniMax Q4_0 T=1024), weights drawn
                           directly in quantised form (tests/helpers.py random_q_weights); only the
                           output rows of tests/helpers.py golden_rows are kept

    python tests/golden/make_golden.py            # everything
    python tests/golden/make_golden.py big        # only the large-T fixtures
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
os.environ["NANOVLLM_TP_SIZE"] = "1"

from oracle import oracle as O  # noqa: E402
from tests.helpers import (big_case_inputs, expert_weights_fp32, golden_rows, q_weights,  # noqa: E402
                           random_q_weights, tokens)


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def route_cases():
    for K in (1, 8, 10):
        rng = np.random.default_rng(100 + K)
        cases = {}
        for ci, (T, E) in enumerate(((1, 16), (7, 16), (64, 128), (5, 8))):
            ids = rng.integers(-2, E + 2, size=(T, K)).astype(np.int32)
            c, s, tm, sm = O.ref_route_preprocess(ids, E)
            cases.update({f"ids{ci}": ids, f"E{ci}": np.int32(E), f"counts{ci}": c, f"starts{ci}": s,
                          f"tmap{ci}": tm, f"smap{ci}": sm})
        np.savez_compressed(os.path.join(HERE, f"route_k{K}.npz"), **cases)


def quant_cases():
    rng = np.random.default_rng(7)
    x = (rng.standard_normal((16, 512), dtype=np.float32) * 3.0).astype(np.float32)
    x[0, :32] = 0.0
    x[1, :32] = 1e-30
    x[2, 5] = 300.0
    qs, d = O.ref_quantize_rows_q8_0(x)
    np.savez_compressed(os.path.join(HERE, "xquant.npz"), x=x, qs=qs, d=d)
    w = (rng.standard_normal((24, 256), dtype=np.float32) * 0.02).astype(np.float32)
    qs, d = O.ref_quantize_weight_q8_0(w)
    np.savez_compressed(os.path.join(HERE, "wquant.npz"), w=w, qs=qs, d=d)


def fwd_case(name, qt, E, H, I, T, K, seed, scale_bf16, act_bf16=True, bad_ids=False):
    gq, gd, dq, dd = q_weights(qt, E, H, I, seed, scale_bf16)
    xb, _, ids, w = tokens(T, H, E, K, seed, act_bf16)
    if bad_ids:
        ids[0, -1] = -1
        ids[T - 1, 0] = E + 3
    eng = O.RefEngine(E, H, I, qt)
    eng.store_repack(scale_bf16, gq, gd, dq, dd)
    y = eng.forward(xb, ids, w, act_bf16)
    eng.close()
    np.savez_compressed(os.path.join(HERE, f"fwd_{name}.npz"), y=y, ids=ids, w=w,
                        meta=np.array([qt, E, H, I, T, K, seed, int(scale_bf16), int(act_bf16)], np.int64),
                        sha=np.array(digest(gq, gd, dq, dd, xb)))


def fwd_c1():
    """Q8_0 by the reference's own online quantiser (quantize_and_store_expert)."""
    H, I, E, K, T, seed = 2048, 768, 128, 8, 1, 11
    xb, ids, w = big_case_inputs(T, seed)
    eng = O.RefEngine(E, H, I, 0)
    for e in np.unique(ids):
        wg, wu, wd = expert_weights_fp32(int(e), seed, H, I)
        eng.quantize_store(int(e), "gate_proj", wg)
        eng.quantize_store(int(e), "up_proj", wu)
        eng.quantize_store(int(e), "down_proj", wd)
    y = eng.forward(xb, ids, w)
    eng.close()
    np.savez_compressed(os.path.join(HERE, "fwd_c1_q8.npz"), y=y, ids=ids, w=w, xb=xb, seed=np.int64(seed))


def fwd_c2():
    """Q4_0 (harness quantiser), token sweep 1/4/8/32."""
    H, I, E, K = 2048, 768, 128, 8
    for T in (1, 4, 8, 32):
        seed = 20 + T
        xb, ids, w = big_case_inputs(T, seed)
        gq = np.zeros((E, 2 * I, H // 8), np.int32)
        gd = np.zeros((E, 2 * I, H // 32), np.uint16)
        dq = np.zeros((E, H, I // 8), np.int32)
        dd = np.zeros((E, H, I // 32), np.uint16)
        for e in np.unique(ids):
            wg, wu, wd = expert_weights_fp32(int(e), seed, H, I)
            gq[e], gd[e] = O.quantize_weight_q4_0(np.concatenate([wg, wu], 0))
            dq[e], dd[e] = O.quantize_weight_q4_0(wd)
        eng = O.RefEngine(E, H, I, 1)
        eng.store_repack(False, gq, gd, dq, dd)
        y = eng.forward(xb, ids, w)
        eng.close()
        np.savez_compressed(os.path.join(HERE, f"fwd_c2_q4_T{T}.npz"), y=y, ids=ids, w=w, xb=xb,
                            seed=np.int64(seed))


BIG_CASES = [  # name, quant, H, I, E, T, seed
    ("big_q4_T128", 1, 2048, 768, 128, 128, 501),
    ("big_q4_T512", 1, 2048, 768, 128, 512, 502),
    ("big_q4_T1024", 1, 2048, 768, 128, 1024, 503),
    ("big_q4_T4096", 1, 2048, 768, 128, 4096, 504),
    ("big_q8_T1024", 0, 2048, 768, 128, 1024, 505),
    ("big_q8_T4096", 0, 2048, 768, 128, 4096, 506),
    ("big_mm_q4_T1024", 1, 3072, 1536, 256, 1024, 507),
]


def fwd_big():
    """Large-T cases through the reference engine; the kept rows and an input digest are stored."""
    K = 8
    for name, qt, H, I, E, T, seed in BIG_CASES:
        gq, gd, dq, dd = random_q_weights(qt, E, H, I, seed)
        xb, ids, w = big_case_inputs(T, seed, H=H, E=E)
        eng = O.RefEngine(E, H, I, qt)
        eng.store_repack(False, gq, gd, dq, dd)
        y = eng.forward(xb, ids, w)
        eng.close()
        rows = golden_rows(T)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), y_rows=y[rows], rows=rows,
                            meta=np.array([qt, E, H, I, T, K, seed], np.int64),
                            sha=np.array(digest(gq, gd, dq, dd, xb, ids, w)))
        print("wrote", name, flush=True)


def write_manifest():
    files = sorted(f for f in os.listdir(HERE) if f.endswith(".npz"))
    with open(os.path.join(HERE, "MANIFEST.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py",
                   "reference": "Int8-gemm (MoEInfer, preprocess_moe_routing, quantize_block_q8_0, "
                                "quantize_weight_only) built unmodified by oracle/Makefile with the scalar "
                                "NEON and single-node NUMA shims, NANOVLLM_TP_SIZE=1",
                   "files": files}, f, indent=1)
    return files


def main():
    if not O.have_reference():
        sys.exit("oracle/_ref/ref_bridge.so missing: run `make -C oracle ref` with the reference checkout")
    if sys.argv[1:] == ["big"]:
        fwd_big()
        write_manifest()
        sys.stdout.flush()
        os._exit(0)
    route_cases()
    quant_cases()
    small = [
        ("q8_f16_T1", 0, 16, 256, 128, 1, 8, 1, False),
        ("q8_bf16_T5", 0, 16, 256, 128, 5, 8, 2, True),
        ("q4_f16_T5", 1, 16, 256, 128, 5, 8, 3, False),
        ("q4_bf16_T3_k10", 1, 32, 512, 256, 3, 10, 4, True),
        ("q8_f16_T4_k1", 0, 8, 512, 256, 4, 1, 5, False),
    ]
    for args in small:
        fwd_case(*args)
    fwd_case("q4_f16_T4_bad", 1, 16, 256, 128, 4, 8, 6, False, True, True)
    fwd_case("q8_f16_T2_act16", 0, 16, 256, 128, 2, 8, 7, False, False)
    fwd_c1()
    fwd_c2()
    fwd_big()
    files = write_manifest()
    print("wrote", len(files), "fixtures")
    sys.stdout.flush()
    os._exit(0)  # skip the reference thread pool's teardown


if __name__ == "__main__":
    main()
