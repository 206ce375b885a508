"""The two-pass decode kernels (AWQ: tp_gate_up_kernel + tp_down_kernel; Q8_0 / Q4_0:
tp_gate_up_q_kernel + tp_down_q_kernel: one CTA per row tile and piece, weights bulk-copied at
CTA start, h between the passes in global memory, last-arriver combine per 32-row block) against
the C oracle, the cluster kernel and the grid-barrier kernel, through the C ABI.  Covers T = 1..8,
bf16 and fp16 activations, fp32 output, invalid ids, duplicate ids inside a token (more pieces
than experts), calls with no valid id, repeated calls (the arrival counters reset), an explicit
expert map with replicated experts split over ranks, and determinism."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import MAX_REL, MIN_COS, awq_weights, parity, tokens

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import moe_ascend_opt_b200  # noqa: F401
    from moe_ascend_opt_b200 import capi
    from tests.test_gpu_cluster import dev, make_engine, oracle, run

AWQ = 2
SHAPES = [(128, 2048, 768), (32, 1024, 512), (16, 512, 256)]


@pytest.mark.parametrize("qt", [AWQ, 1, 0])
@pytest.mark.parametrize("E,H,I", SHAPES)
@pytest.mark.parametrize("T", [1, 2, 3, 5, 8])
def test_two_pass_matches_oracle(qt, E, H, I, T):
    seed = 2000 + 11 * T + E + qt
    eng, wts = make_engine(qt, E, H, I, seed, two_pass=True)
    xb, xf, ids, w = tokens(T, H, E, 8, seed)
    y = run(eng, xb, ids, w, H)
    rel, cos = parity(y, oracle(qt, xf, ids, w, wts))
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


@pytest.mark.parametrize("qt", [AWQ, 1, 0])
@pytest.mark.parametrize("T", [1, 4])
def test_two_pass_fp16_activations(qt, T):
    E, H, I = 32, 1024, 512
    eng, wts = make_engine(qt, E, H, I, 78, two_pass=True)
    xb, xf, ids, w = tokens(T, H, E, 8, 78, bf16=False)
    y = run(eng, xb, ids, w, H, act_bf16=False)
    rel, cos = parity(y, oracle(qt, xf, ids, w, wts))
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


@pytest.mark.parametrize("qt", [AWQ, 1])
def test_two_pass_matches_other_kernels(qt):
    E, H, I = 128, 2048, 768
    tp, _ = make_engine(qt, E, H, I, 5, two_pass=True)
    cl, _ = make_engine(qt, E, H, I, 5)
    leg, _ = make_engine(qt, E, H, I, 5, legacy=True)
    for T in (1, 4, 8):
        xb, _, ids, w = tokens(T, H, E, 8, 60 + T)
        y = run(tp, xb, ids, w, H)
        for other in (cl, leg):
            rel, cos = parity(y, run(other, xb, ids, w, H))
            assert rel <= MAX_REL and cos >= MIN_COS, (T, rel, cos)


@pytest.mark.parametrize("qt", [AWQ, 1, 0])
def test_two_pass_odd_routing(qt):
    """Invalid ids, one expert five times in a token (two pieces at T=3: ncol = 3), a token
    with no valid id, then a call with no valid id at all (zero output), then the first call
    again (counters reset)."""
    E, H, I, T, K = 32, 1024, 512, 3, 8
    eng, wts = make_engine(qt, E, H, I, 9, two_pass=True)
    xb, xf, ids, w = tokens(T, H, E, K, 9)
    ids[0, :5] = 7
    ids[1, 2] = 7
    ids[1, 3] = -1
    ids[2, :] = E + 5
    y = run(eng, xb, ids, w, H)
    rel, cos = parity(y, oracle(qt, xf, ids, w, wts))
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)
    assert np.all(y[2] == 0.0)
    y0 = run(eng, xb, np.full_like(ids, -3), w, H)
    assert np.all(y0 == 0.0)
    y2 = run(eng, xb, ids, w, H)
    assert np.array_equal(y2, y)


def test_two_pass_fp32_output_and_replicas():
    """Three engines on one GPU hold disjoint cold experts plus two replicated hot experts
    (explicit map with MOE_REPLICATED, pairs split by (t + id) % 3): the fp32 partial outputs
    sum to the full layer."""
    from moe_ascend_opt_b200.ep import replicated_placement
    E, H, I, T, K, W = 32, 1024, 512, 6, 8, 3
    wts = awq_weights(E, H, I, 128, 31)
    xb, xf, ids, w = tokens(T, H, E, K, 31)
    pl, hot = replicated_placement(np.bincount(ids.ravel(), minlength=E), W, 2)
    x = dev(xb.view(np.int16)).view(torch.bfloat16)
    total = np.zeros((T, H), np.float64)
    for r in range(W):
        experts = pl[r]
        eng, _ = make_engine(AWQ, len(experts), H, I, 0, two_pass=True)
        m = np.full(E, -1, np.int32)
        for l, g in enumerate(experts):
            m[g] = l | (capi.REPLICATED if g in hot else 0)
        eng.set_expert_map(m)
        eng.set_replica_split(r, W)
        sel = np.asarray(experts)
        eng.load_awq(*[torch.from_numpy(np.ascontiguousarray(a[sel])) for a in wts])
        y = torch.empty((T, H), dtype=torch.float32, device="cuda")
        eng.forward(x, y, dev(ids), dev(w), capi.BF16, capi.F32)
        torch.cuda.synchronize()
        assert eng.device_error() == 0
        total += y.cpu().numpy()
    rel, cos = parity(total.astype(np.float32), O.moe_forward_awq(xf, ids, w, *wts, group=128))
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


def test_two_pass_deterministic_and_graph():
    E, H, I, T = 128, 2048, 768, 2
    eng, _ = make_engine(AWQ, E, H, I, 3, two_pass=True)
    xb, _, ids, w = tokens(T, H, E, 8, 3)
    outs = [run(eng, xb, ids, w, H) for _ in range(3)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])
    # captured in a CUDA graph and replayed: same output
    x = dev(xb.view(np.int16)).view(torch.bfloat16)
    y = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    di, dw = dev(ids), dev(w)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        eng.forward(x, y, di, dw, capi.BF16, capi.BF16, stream=s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        eng.forward(x, y, di, dw, capi.BF16, capi.BF16, stream=s)
    for _ in range(5):
        g.replay()
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    assert np.array_equal(y.float().cpu().numpy(), outs[0])


@pytest.mark.parametrize("T", [12, 20, 32])
def test_two_pass_token_slices_awq(T):
    """AWQ calls of 9-32 tokens run the two-pass kernels in slices of 8 tokens (each slice's
    pass 1 waits for the previous slice's pass 2 through the stream)."""
    E, H, I = 32, 1024, 512
    eng, wts = make_engine(AWQ, E, H, I, 300 + T, two_pass=True)
    xb, xf, ids, w = tokens(T, H, E, 8, 300 + T)
    y = run(eng, xb, ids, w, H)
    rel, cos = parity(y, oracle(AWQ, xf, ids, w, wts))
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)
