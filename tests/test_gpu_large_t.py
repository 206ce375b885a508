"""Large token counts at the sizes where the grouped GEMMs run by default, against the
reference's own outputs (Q4_0 / Q8_0) or the C oracle (AWQ), through the C ABI.

* big_q4_T{128,512}: the int8 mma grouped GEMMs (weights-on-M / tokens-on-M tiles);
* big_q4_T{1024,4096}, big_q8_T{1024,4096}: the tcgen05 GEMMs (>= 48 tokens per expert);
* big_mm_q4_T1024: BASELINE configs[3]'s MiniMax-M2 shape (H3072 I1536 E256) on tcgen05;
* AWQ Qwen T=64 and T=1024: the tcgen05 W4A16 GEMMs, oracle on a subset of token rows.

The fixtures keep the reference's outputs of 32 token rows (tests/helpers.py golden_rows);
the full layer runs on the GPU and those rows are compared.  Device errors raised by a
kernel surface as an exception at the next call (test_range_error_is_raised)."""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import (MAX_REL, MIN_COS, awq_weights, big_case_inputs, digest_inputs, golden_rows, parity,
                           q_weights, random_q_weights, tokens)

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import moe_ascend_opt_b200  # noqa: F401
    from moe_ascend_opt_b200 import capi

GOLD = os.path.join(os.path.dirname(__file__), "golden")
BIG = ["big_q4_T128", "big_q4_T512", "big_q4_T1024", "big_q4_T4096", "big_q8_T1024", "big_q8_T4096",
       "big_mm_q4_T1024"]


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("name", BIG)
def test_large_t_matches_reference(name):
    f = np.load(os.path.join(GOLD, name + ".npz"))
    qt, E, H, I, T, K, seed = (int(v) for v in f["meta"])
    gq, gd, dq, dd = random_q_weights(qt, E, H, I, seed)
    xb, ids, w = big_case_inputs(T, seed, H=H, E=E)
    assert digest_inputs(gq, gd, dq, dd, xb, ids, w) == str(f["sha"]), "input generator drifted"
    eng = capi.Engine(E, H, I, qt)
    eng.load_quantized(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)), torch.from_numpy(dq),
                       torch.from_numpy(dd.view(np.int16)), capi.F16)
    del gq, gd, dq, dd
    x = dev(xb.view(np.int16)).view(torch.bfloat16)
    y = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    eng.forward(x, y, dev(ids), dev(w), capi.BF16, capi.BF16)
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    rows = f["rows"]
    assert np.array_equal(rows, golden_rows(T))
    rel, cos = parity(y.float().cpu().numpy()[rows], O.bf16_bits_to_f32(f["y_rows"]))
    assert rel <= MAX_REL and cos >= MIN_COS, (name, rel, cos)
    assert np.isfinite(y.float().cpu().numpy()).all()


@pytest.mark.parametrize("T", [64, 1024])
def test_awq_large_t_matches_oracle(T):
    E, H, I, K, G = 128, 2048, 768, 8, 128
    seed = 600 + T
    wts = awq_weights(E, H, I, G, seed)
    xb, ids, w = big_case_inputs(T, seed, H=H, E=E)
    eng = capi.Engine(E, H, I, capi.AWQ, group_size=G)
    eng.load_awq(*[torch.from_numpy(a) for a in wts])
    x = dev(xb.view(np.int16)).view(torch.bfloat16)
    y = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    eng.forward(x, y, dev(ids), dev(w), capi.BF16, capi.BF16)
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    rows = golden_rows(T, 16)
    y_ref = O.moe_forward_awq(O.bf16_bits_to_f32(xb[rows]), ids[rows], w[rows], *wts, group=G)
    rel, cos = parity(y.float().cpu().numpy()[rows], y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (T, rel, cos)


def _small_q4_engine():
    E, H, I = 4, 512, 256
    gq, gd, dq, dd = q_weights(1, E, H, I, 5)
    eng = capi.Engine(E, H, I, 1)
    eng.load_quantized(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)), torch.from_numpy(dq),
                       torch.from_numpy(dd.view(np.int16)), capi.F16)
    return eng, (gq, gd, dq, dd), (E, H, I)


def test_range_error_is_raised():
    """An activation block beyond the fp16 range on the tcgen05 path (128 tokens per expert)
    sets device error 5; the next call on the engine raises it and resets the engine."""
    eng, _, (E, H, I) = _small_q4_engine()
    T, K = 128, 4
    xb, _, ids, w = tokens(T, H, E, K, 9)
    x = dev(xb.view(np.int16)).view(torch.bfloat16)
    x[5, 64:96] = 1.0e5
    y = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    eng.forward(x, y, dev(ids), dev(w), capi.BF16, capi.BF16)  # asynchronous: returns before the kernel ends
    torch.cuda.synchronize()
    with pytest.raises(capi.MoeError, match="float16 range"):
        eng.forward(x, y, dev(ids), dev(w), capi.BF16, capi.BF16)
    assert eng.device_error() == 0  # the failing call cleared the word
    x[5, 64:96] = 1.0
    eng.forward(x, y, dev(ids), dev(w), capi.BF16, capi.BF16)
    torch.cuda.synchronize()
    assert eng.device_error() == 0


def test_range_error_raises_through_torch_op():
    E, H, I = 4, 512, 256
    gq, gd, dq, dd = q_weights(1, E, H, I, 6)
    h = torch.classes.nanovllm.MoEInfer(E, H, I, 1)
    h.store_quantized_repack(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)).view(torch.float16),
                             torch.from_numpy(dq), torch.from_numpy(dd.view(np.int16)).view(torch.float16))
    T, K = 128, 4
    xb, _, ids, w = tokens(T, H, E, K, 10)
    x = dev(xb.view(np.int16)).view(torch.bfloat16)
    x[0, :32] = -2.0e5
    torch.ops.nanovllm.moe_forward(x, dev(ids), dev(w), h)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="device"):
        torch.ops.nanovllm.moe_forward(x, dev(ids), dev(w), h)


def test_timeline_off_then_gemm_forward():
    """Turning the phase timeline on and off leaves the grouped-GEMM workspace intact."""
    eng, (gq, gd, dq, dd), (E, H, I) = _small_q4_engine()
    K = 4
    for T in (1, 64):
        xb, xf, ids, w = tokens(T, H, E, K, 30 + T)
        x = dev(xb.view(np.int16)).view(torch.bfloat16)
        y = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
        eng.forward(x, y, dev(ids), dev(w), capi.BF16, capi.BF16)  # T=64 allocates the GEMM workspace
        eng.timeline(True)
        eng.forward(x, y, dev(ids), dev(w), capi.BF16, capi.BF16)
        eng.timeline(False)
        eng.forward(x, y, dev(ids), dev(w), capi.BF16, capi.BF16)
        torch.cuda.synchronize()
        assert eng.device_error() == 0
        rel, cos = parity(y.float().cpu().numpy(), O.moe_forward_q(1, False, xf, ids, w, gq, gd, dq, dd))
        assert rel <= MAX_REL and cos >= MIN_COS, (T, rel, cos)
    eng.close()
