"""GPU parity of the CUDA path against the C oracle, through the C ABI.

Bit-exact: routing top-K ids, the stable permutation, Q8_0 activation
quantisation, online Q8_0 weight quantisation and the decoded device weights.
Tolerance (max rel <= 1e-2, cosine >= 0.9999): the fused FFN output.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import MAX_REL, MIN_COS, parity, q_weights, tokens

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import moe_ascend_opt_b200  # noqa: F401  (fails loudly without the CUDA build)
    from moe_ascend_opt_b200 import capi


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_engine(qt, E, H, I, T, K, seed, scale_bf16=False, act_bf16=True, bad_ids=False, out_dtype=None):
    gq, gd, dq, dd = q_weights(qt, E, H, I, seed, scale_bf16)
    xb, xf, ids, w = tokens(T, H, E, K, seed, act_bf16)
    if bad_ids and T > 0:
        ids[0, -1] = -1
        ids[T - 1, 0] = E + 3
    eng = capi.Engine(E, H, I, qt, device=0)
    sdt = capi.BF16 if scale_bf16 else capi.F16
    eng.load_quantized(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)), torch.from_numpy(dq),
                       torch.from_numpy(dd.view(np.int16)), sdt)
    x = dev(xb.view(np.int16)).view(torch.bfloat16 if act_bf16 else torch.float16)
    odt = out_dtype if out_dtype is not None else (capi.BF16 if act_bf16 else capi.F16)
    y = torch.empty((T, H), dtype={capi.F16: torch.float16, capi.BF16: torch.bfloat16, capi.F32: torch.float32}[odt],
                    device="cuda")
    eng.forward(x, y, dev(ids), dev(w), capi.BF16 if act_bf16 else capi.F16, odt)
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    y_ref = O.moe_forward_q(qt, scale_bf16, xf, ids, w, gq, gd, dq, dd)
    return y.float().cpu().numpy(), y_ref, eng


CASES = [
    # qt, E, H, I, T, K
    (0, 16, 256, 128, 1, 8),
    (1, 16, 256, 128, 1, 8),
    (0, 16, 256, 128, 5, 8),
    (1, 16, 256, 128, 5, 8),
    (1, 32, 1024, 384, 3, 10),
    (0, 8, 512, 256, 4, 1),
    (1, 64, 2048, 768, 8, 8),
    (0, 64, 2048, 768, 2, 8),
]


@pytest.mark.parametrize("qt,E,H,I,T,K", CASES)
def test_forward_matches_oracle(qt, E, H, I, T, K):
    y, y_ref, _ = run_engine(qt, E, H, I, T, K, seed=E + H + T)
    rel, cos = parity(y, y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


@pytest.mark.parametrize("scale_bf16,act_bf16", [(True, True), (False, False), (True, False)])
@pytest.mark.parametrize("qt", [0, 1])
def test_forward_dtypes(qt, scale_bf16, act_bf16):
    y, y_ref, _ = run_engine(qt, 16, 512, 256, 3, 8, seed=11, scale_bf16=scale_bf16, act_bf16=act_bf16)
    rel, cos = parity(y, y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


@pytest.mark.parametrize("qt", [0, 1])
def test_invalid_ids_are_skipped(qt):
    y, y_ref, _ = run_engine(qt, 16, 256, 128, 4, 8, seed=3, bad_ids=True)
    rel, cos = parity(y, y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


def test_fp32_partial_output():
    y, y_ref, _ = run_engine(1, 16, 256, 128, 2, 8, seed=5, out_dtype=capi.F32)
    rel, cos = parity(y, y_ref)
    assert rel <= 2e-3 and cos >= MIN_COS, (rel, cos)


def test_many_tokens_slices():
    # more tokens than one decode launch holds: the forward splits the tokens
    y, y_ref, _ = run_engine(1, 16, 512, 256, 70, 8, seed=9)
    rel, cos = parity(y, y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


def test_all_ids_invalid_gives_zero():
    E, H, I, T, K = 8, 256, 128, 3, 8
    gq, gd, dq, dd = q_weights(1, E, H, I, 1)
    xb, _, ids, w = tokens(T, H, E, K, 1)
    ids[:] = -1
    eng = capi.Engine(E, H, I, 1)
    eng.load_quantized(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)), torch.from_numpy(dq),
                       torch.from_numpy(dd.view(np.int16)), capi.F16)
    y = torch.full((T, H), 7.0, dtype=torch.bfloat16, device="cuda")
    eng.forward(dev(xb.view(np.int16)).view(torch.bfloat16), y, dev(ids), dev(w), capi.BF16, capi.BF16)
    torch.cuda.synchronize()
    assert torch.count_nonzero(y).item() == 0


def test_repeat_calls_identical():
    _, _, eng = run_engine(1, 16, 256, 128, 2, 8, seed=21)
    H = 256
    xb, _, ids, w = tokens(2, H, 16, 8, 21)
    x = dev(xb.view(np.int16)).view(torch.bfloat16)
    ys = []
    for _ in range(3):
        y = torch.empty((2, H), dtype=torch.bfloat16, device="cuda")
        eng.forward(x, y, dev(ids), dev(w), capi.BF16, capi.BF16)
        ys.append(y)
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[1], ys[2])


@pytest.mark.parametrize("qt", [0, 1])
def test_export_decode_bit_exact(qt):
    E, H, I = 8, 512, 256
    gq, gd, dq, dd = q_weights(qt, E, H, I, 4)
    eng = capi.Engine(E, H, I, qt)
    eng.load_quantized(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)), torch.from_numpy(dq),
                       torch.from_numpy(dd.view(np.int16)), capi.F16)
    for e in (0, 5, 7):
        q0 = np.empty_like(gq[e]); d0 = np.empty_like(gd[e])
        eng.export_expert(e, 0, q0, d0)
        assert np.array_equal(q0, gq[e]) and np.array_equal(d0, gd[e])
        q1 = np.empty_like(dq[e]); d1 = np.empty_like(dd[e])
        eng.export_expert(e, 1, q1, d1)
        assert np.array_equal(q1, dq[e]) and np.array_equal(d1, dd[e])
        assert np.array_equal(O.decode_q(qt, q0, 2 * I, H), O.decode_q(qt, gq[e], 2 * I, H))


@pytest.mark.parametrize("wdt", ["f32", "bf16"])
def test_online_quantize_bit_exact(wdt):
    E, H, I = 4, 256, 128
    rng = np.random.default_rng(2)
    wg = (rng.standard_normal((E, I, H), dtype=np.float32) * 0.02)
    wu = (rng.standard_normal((E, I, H), dtype=np.float32) * 0.02)
    wd = (rng.standard_normal((E, H, I), dtype=np.float32) * 0.02)
    if wdt == "bf16":
        wg, wu, wd = (O.bf16_bits_to_f32(O.f32_to_bf16_bits(a)) for a in (wg, wu, wd))
    eng = capi.Engine(E, H, I, 0)
    for e in range(E):
        for proj, a in ((0, wg[e]), (1, wu[e]), (2, wd[e])):
            t = torch.from_numpy(np.ascontiguousarray(a))
            if wdt == "bf16":
                eng.quantize_store_expert(e, proj, t.to(torch.bfloat16).cuda(), capi.BF16)
            else:
                eng.quantize_store_expert(e, proj, t, capi.F32)
    for e in range(E):
        q0 = np.empty((2 * I, H), np.int8); d0 = np.empty((2 * I, H // 32), np.uint16)
        eng.export_expert(e, 0, q0, d0)
        rq, rd = O.quantize_weight_q8_0(np.concatenate([wg[e], wu[e]], 0))
        assert np.array_equal(q0, rq) and np.array_equal(d0, rd)
        q1 = np.empty((H, I), np.int8); d1 = np.empty((H, I // 32), np.uint16)
        eng.export_expert(e, 1, q1, d1)
        rq, rd = O.quantize_weight_q8_0(wd[e])
        assert np.array_equal(q1, rq) and np.array_equal(d1, rd)


@pytest.mark.parametrize("T,K,E", [(1, 8, 128), (7, 8, 128), (64, 8, 128), (33, 10, 64), (5, 1, 16), (300, 8, 256)])
def test_route_permute_bit_exact(T, K, E):
    rng = np.random.default_rng(T * K + E)
    ids = rng.integers(-3, E + 3, size=(T, K)).astype(np.int32)
    counts = torch.empty(E, dtype=torch.int32, device="cuda")
    starts = torch.empty(E + 1, dtype=torch.int32, device="cuda")
    tmap = torch.full((T * K, 2), -1, dtype=torch.int32, device="cuda")
    smap = torch.empty((T, K), dtype=torch.int32, device="cuda")
    capi.call("moe_route_permute", dev(ids).data_ptr(), T, K, E, counts.data_ptr(), starts.data_ptr(),
              tmap.data_ptr(), smap.data_ptr(), capi.stream_handle())
    torch.cuda.synchronize()
    c, s, tm, sm = O.route_preprocess(ids, E)
    assert np.array_equal(counts.cpu().numpy(), c)
    assert np.array_equal(starts.cpu().numpy(), s)
    assert np.array_equal(tmap.cpu().numpy()[: len(tm)], tm)
    assert np.array_equal(smap.cpu().numpy(), sm)


@pytest.mark.parametrize("T,E,K,renorm", [(1, 128, 8, True), (37, 128, 8, True), (16, 256, 8, False), (9, 64, 10, True)])
def test_route_topk(T, E, K, renorm):
    rng = np.random.default_rng(T + E)
    logits = rng.standard_normal((T, E), dtype=np.float32)
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    w = torch.empty((T, K), dtype=torch.float32, device="cuda")
    capi.call("moe_route_topk", dev(logits).data_ptr(), T, E, K, int(renorm), ids.data_ptr(), w.data_ptr(),
              capi.stream_handle())
    torch.cuda.synchronize()
    rid, rw = O.topk_softmax(logits, K, renorm)
    assert np.array_equal(ids.cpu().numpy(), rid)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-6, atol=1e-7)
    tv, ti = torch.topk(torch.from_numpy(logits), K, sorted=True)
    assert np.array_equal(ti.numpy(), rid)


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_quantize_rows_bit_exact(dtype):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((13, 2048), dtype=np.float32) * 3
    x[0, :32] = 0.0
    x[1, 5] = 1e-30
    if dtype == "bf16":
        bits = O.f32_to_bf16_bits(x); xf = O.bf16_bits_to_f32(bits)
        xt = dev(bits.view(np.int16)).view(torch.bfloat16); code = capi.BF16
    elif dtype == "f16":
        bits = O.f32_to_f16_bits(x); xf = O.f16_bits_to_f32(bits)
        xt = dev(bits.view(np.int16)).view(torch.float16); code = capi.F16
    else:
        xf = x; xt = dev(x); code = capi.F32
    qs = torch.empty((13, 2048), dtype=torch.int8, device="cuda")
    d = torch.empty((13, 64), dtype=torch.float32, device="cuda")
    capi.call("moe_quantize_rows_q8_0", xt.data_ptr(), code, 13, 2048, qs.data_ptr(), d.data_ptr(),
              capi.stream_handle())
    torch.cuda.synchronize()
    rq, rd = O.quantize_rows_q8_0(xf)
    assert np.array_equal(qs.cpu().numpy(), rq)
    assert np.array_equal(d.cpu().numpy().view(np.uint32), rd.view(np.uint32))


@pytest.mark.parametrize("qt,E,H,I,T,K", [
    (1, 16, 512, 256, 33, 8),
    (0, 16, 512, 256, 100, 8),
    (1, 32, 1024, 384, 300, 10),
    (0, 64, 2048, 768, 64, 8),
    (1, 128, 2048, 768, 256, 8),
])
def test_grouped_gemm_path_matches_oracle(qt, E, H, I, T, K):
    """T above the decode threshold takes the grouped int8-MMA GEMM path."""
    y, y_ref, _ = run_engine(qt, E, H, I, T, K, seed=T + E, bad_ids=True)
    rel, cos = parity(y, y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


def test_gemm_and_decode_paths_agree(monkeypatch):
    E, H, I, T, K = 32, 1024, 384, 40, 8
    outs = []
    for thr in ("1000", "0"):  # 1000: decode kernel in token slices; 0: grouped GEMM
        monkeypatch.setenv("MOE_GEMM_MIN_TOKENS", thr)
        y, y_ref, _ = run_engine(1, E, H, I, T, K, seed=4)
        outs.append(y)
    rel, cos = parity(outs[0], outs[1])
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


@pytest.mark.parametrize("qt,E,H,I,T,K", [(0, 16, 512, 256, 3, 8), (1, 64, 2048, 768, 8, 8), (1, 128, 2048, 768, 1, 8)])
def test_split_k_kernel_matches_barrier_kernel(qt, E, H, I, T, K, monkeypatch):
    # the split-K decode kernel (default for Q8_0/Q4_0) against the kernel with the grid
    # barrier between gate_up and down: both within fp32 rounding of each other
    monkeypatch.setenv("MOE_SK_MIN_CHUNKS", "0")  # split-K even where the default picks the barrier kernel
    y_sk, y_ref, _ = run_engine(qt, E, H, I, T, K, seed=31, out_dtype=capi.F32)
    monkeypatch.setenv("MOE_DECODE_SK", "0")
    y_bar, _, _ = run_engine(qt, E, H, I, T, K, seed=31, out_dtype=capi.F32)
    rel, cos = parity(y_sk, y_bar)
    assert rel <= 1e-5 and cos >= 0.999999, (rel, cos)
    rel, cos = parity(y_sk, y_ref)
    assert rel <= 2e-3 and cos >= MIN_COS, (rel, cos)


@pytest.mark.parametrize("bm", ["w8", "w16", "16", "32", "64", "128"])
@pytest.mark.parametrize("qt", [0, 1])
def test_gemm_tile_rows_variants(qt, bm, monkeypatch):
    # every token-tile height of the grouped GEMM, on ragged per-expert counts
    monkeypatch.setenv("MOE_GEMM_BM", bm)
    y, y_ref, _ = run_engine(qt, 32, 1024, 384, 90, 8, seed=7, bad_ids=True)
    rel, cos = parity(y, y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


@pytest.mark.parametrize("scale_bf16,act_bf16", [(True, True), (False, False)])
@pytest.mark.parametrize("qt", [0, 1])
def test_tcgen05_gemm_dtypes(qt, scale_bf16, act_bf16, monkeypatch):
    # the tcgen05 path with bf16 / fp16 block scales and bf16 / fp16 activations
    monkeypatch.setenv("MOE_GEMM_BM", "128")
    y, y_ref, _ = run_engine(qt, 16, 1024, 384, 150, 8, seed=13, scale_bf16=scale_bf16, act_bf16=act_bf16)
    rel, cos = parity(y, y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)
