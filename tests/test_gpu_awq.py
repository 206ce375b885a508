"""GPU parity of the AWQ W4A16 path (BASELINE configs[2]-[3] formats) against the C oracle.

The reference checkout has no AWQ implementation (its Ascend kernel lives in an
absent submodule), so the oracle's AWQ restatement is the specification here:
W = (q - z) * s per group of 128 along K, 16-bit activations, fp32 arithmetic.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import MAX_REL, MIN_COS, awq_weights, parity, tokens

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import moe_ascend_opt_b200  # noqa: F401
    from moe_ascend_opt_b200 import capi


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def awq_engine(E, H, I, G, seed):
    ws = awq_weights(E, H, I, G, seed)
    eng = capi.Engine(E, H, I, capi.AWQ, group_size=G)
    eng.load_awq(*[torch.from_numpy(np.ascontiguousarray(w)) for w in ws])
    return eng, ws


@pytest.mark.parametrize("E,H,I,G,T,K", [
    (16, 256, 128, 128, 1, 8),
    (16, 512, 256, 128, 3, 8),
    (32, 1024, 384, 128, 2, 8),
    (64, 2048, 768, 128, 1, 8),
    (64, 2048, 768, 128, 8, 8),
    (16, 512, 256, 64, 4, 10),
])
def test_awq_forward_matches_oracle(E, H, I, G, T, K):
    eng, ws = awq_engine(E, H, I, G, seed=E + T)
    xb, xf, ids, w = tokens(T, H, E, K, seed=T)
    x = dev(xb.view(np.int16)).view(torch.bfloat16)
    y = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    eng.forward(x, y, dev(ids), dev(w), capi.BF16, capi.BF16)
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    y_ref = O.moe_forward_awq(xf, ids, w, *ws, group=G)
    rel, cos = parity(y.float().cpu().numpy(), y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


def test_awq_fp16_activations_and_invalid_ids():
    E, H, I, G, T, K = 16, 512, 256, 128, 3, 8
    eng, ws = awq_engine(E, H, I, G, seed=5)
    xb, xf, ids, w = tokens(T, H, E, K, seed=5, bf16=False)
    ids[0, 2] = -1
    ids[2, 7] = E + 1
    x = dev(xb.view(np.int16)).view(torch.float16)
    y = torch.empty((T, H), dtype=torch.float16, device="cuda")
    eng.forward(x, y, dev(ids), dev(w), capi.F16, capi.F16)
    torch.cuda.synchronize()
    y_ref = O.moe_forward_awq(xf, ids, w, *ws, group=G)
    rel, cos = parity(y.float().cpu().numpy(), y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


def test_awq_export_decode_bit_exact():
    E, H, I, G = 4, 512, 256, 128
    eng, (w13_qw, w13_sc, w13_qz, w2_qw, w2_sc, w2_qz) = awq_engine(E, H, I, G, seed=2)
    for e in range(E):
        for which, (qw, sc, qz, Kd, N) in ((0, (w13_qw, w13_sc, w13_qz, H, 2 * I)), (1, (w2_qw, w2_sc, w2_qz, I, H))):
            ng = Kd // G
            q = np.empty((N, Kd // 2), np.uint8)
            d = np.empty((N, ng * 3), np.uint8)
            eng.export_expert(e, which, q, d)
            nib = np.stack([q & 0xF, q >> 4], -1).reshape(N, Kd)  # [n][k]
            # reference decode of the AWQ packing: dequantised W[n][k] = (q - z) * s
            W = O.awq_dequant(qw[e], sc[e], qz[e], G)
            s_dev = O.bf16_bits_to_f32(np.ascontiguousarray(d[:, : 2 * ng]).view(np.uint16))  # [N, ng]
            z_dev = d[:, 2 * ng:].astype(np.float32)
            W_dev = (nib.astype(np.float32) - np.repeat(z_dev, G, 1)) * np.repeat(s_dev, G, 1)
            assert np.array_equal(W_dev, W)


@pytest.mark.parametrize("bf16", [True, False])
@pytest.mark.parametrize("E,H,I,G,T,K", [(16, 512, 256, 128, 40, 8), (32, 1024, 384, 64, 100, 8)])
def test_awq_tcgen05_gemm_path_matches_oracle(E, H, I, G, T, K, bf16):
    # more than 24 tokens: the tcgen05 GEMMs on the 16-bit hidden rows (W4A16), bf16 / fp16 operands
    eng, ws = awq_engine(E, H, I, G, seed=E + T + G)
    xb, xf, ids, w = tokens(T, H, E, K, seed=T, bf16=bf16)
    ids[0, 1] = -1
    dt = torch.bfloat16 if bf16 else torch.float16
    x = dev(xb.view(np.int16)).view(dt)
    y = torch.empty((T, H), dtype=dt, device="cuda")
    eng.forward(x, y, dev(ids), dev(w), capi.BF16 if bf16 else capi.F16, capi.BF16 if bf16 else capi.F16)
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    y_ref = O.moe_forward_awq(xf, ids, w, *ws, group=G)
    rel, cos = parity(y.float().cpu().numpy(), y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)
