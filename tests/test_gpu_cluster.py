"""The cluster decode kernel (moe_decode_cl_kernel: one 16-CTA cluster per routed expert,
h exchanged through distributed shared memory, last-arriver combine) against the C oracle
and against the grid-barrier / split-K decode kernels it replaces for decode sizes, through
the C ABI.  Covers Q8_0 / Q4_0 / AWQ (bf16 and fp16 activations), T = 1..8, invalid ids,
duplicate ids within a token (an expert with more routed pairs than tokens), calls with no
valid id, expert offsets, and repeated calls on one engine (the combine counters reset)."""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import MAX_REL, MIN_COS, awq_weights, parity, q_weights, tokens

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import moe_ascend_opt_b200  # noqa: F401
    from moe_ascend_opt_b200 import capi


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def make_engine(qt, E, H, I, seed, legacy=False, G=128, expert_offset=0, two_pass=False):
    """Engine with Q weights (or AWQ) that takes the cluster kernel for up to 8 tokens, or
    (legacy=True) never; two_pass=True: the two-pass kernels (AWQ) for up to 8 tokens."""
    env = {"MOE_CL_MAX_TOKENS": "0" if legacy else "8", "MOE_TP_MAX_TOKENS": "8" if two_pass else "0"}
    old = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        eng = capi.Engine(E, H, I, qt, group_size=G, expert_offset=expert_offset)
    finally:
        for k, v in old.items():
            if v is None:
                del os.environ[k]
            else:
                os.environ[k] = v
    if qt == capi.AWQ:
        wts = awq_weights(E, H, I, G, seed)
        eng.load_awq(*[torch.from_numpy(a) for a in wts])
    else:
        wts = q_weights(qt, E, H, I, seed)
        gq, gd, dq, dd = wts
        eng.load_quantized(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)), torch.from_numpy(dq),
                           torch.from_numpy(dd.view(np.int16)), capi.F16)
    return eng, wts


def oracle(qt, xf, ids, w, wts, G=128):
    if qt == capi.AWQ:
        return O.moe_forward_awq(xf, ids, w, *wts, group=G)
    return O.moe_forward_q(qt, False, xf, ids, w, *wts)


def run(eng, xb, ids, w, H, act_bf16=True):
    T = ids.shape[0]
    x = dev(xb.view(np.int16)).view(torch.bfloat16 if act_bf16 else torch.float16)
    y = torch.empty((T, H), dtype=torch.bfloat16 if act_bf16 else torch.float16, device="cuda")
    a = capi.BF16 if act_bf16 else capi.F16
    eng.forward(x, y, dev(ids), dev(w), a, a)
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    return y.float().cpu().numpy()


SHAPES = [  # qt, E, H, I
    (1, 128, 2048, 768),
    (0, 128, 2048, 768),
    (2, 128, 2048, 768),
    (1, 16, 512, 256),
    (0, 32, 1024, 512),
    (2, 32, 1024, 512),
]


@pytest.mark.parametrize("qt,E,H,I", SHAPES)
@pytest.mark.parametrize("T", [1, 2, 5, 8])
def test_cluster_kernel_matches_oracle(qt, E, H, I, T):
    seed = 1000 + 7 * T + qt
    eng, wts = make_engine(qt, E, H, I, seed)
    xb, xf, ids, w = tokens(T, H, E, 8, seed)
    y = run(eng, xb, ids, w, H)
    rel, cos = parity(y, oracle(qt, xf, ids, w, wts))
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


@pytest.mark.parametrize("qt", [0, 1, 2])
def test_cluster_kernel_fp16_activations(qt):
    E, H, I, T = 32, 1024, 512, 3
    eng, wts = make_engine(qt, E, H, I, 77)
    xb, xf, ids, w = tokens(T, H, E, 8, 77, bf16=False)
    y = run(eng, xb, ids, w, H, act_bf16=False)
    rel, cos = parity(y, oracle(qt, xf, ids, w, wts))
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


@pytest.mark.parametrize("qt", [1, 2])
def test_cluster_kernel_matches_legacy_kernels(qt):
    E, H, I = 128, 2048, 768
    eng, wts = make_engine(qt, E, H, I, 5)
    leg, _ = make_engine(qt, E, H, I, 5, legacy=True)
    for T in (1, 4, 8):
        xb, xf, ids, w = tokens(T, H, E, 8, 50 + T)
        y = run(eng, xb, ids, w, H)
        y_leg = run(leg, xb, ids, w, H)
        rel, cos = parity(y, y_leg)
        assert rel <= MAX_REL and cos >= MIN_COS, (T, rel, cos)


@pytest.mark.parametrize("qt", [0, 1, 2])
def test_cluster_kernel_odd_routing(qt):
    """Invalid ids, duplicates inside a token (one expert holding more pairs than tokens, so
    its positions are split into several work units), a token with no valid id, and calls
    where no id is valid at all (zero output)."""
    E, H, I, T, K = 32, 1024, 512, 3, 8
    eng, wts = make_engine(qt, E, H, I, 9)
    xb, xf, ids, w = tokens(T, H, E, K, 9)
    ids[0, :5] = 7          # expert 7 five times in token 0
    ids[1, 2] = 7
    ids[1, 3] = -1
    ids[2, :] = E + 5       # token 2: nothing valid
    y = run(eng, xb, ids, w, H)
    y_ref = oracle(qt, xf, ids, w, wts)
    rel, cos = parity(y, y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)
    assert np.all(y[2] == 0.0)
    bad = np.full_like(ids, -3)
    y0 = run(eng, xb, bad, w, H)
    assert np.all(y0 == 0.0)
    y2 = run(eng, xb, ids, w, H)  # the counters were reset by the previous calls
    assert np.array_equal(y2, y)


def test_cluster_kernel_expert_offset_partial():
    """An engine holding experts [16, 32) of 32 (expert parallel): fp32 partial output."""
    E, H, I, T = 32, 1024, 512, 4
    gq, gd, dq, dd = q_weights(1, E, H, I, 12)
    xb, xf, ids, w = tokens(T, H, E, 8, 12)
    eng, _ = make_engine(1, 16, H, I, 0, expert_offset=16)  # weights replaced below
    eng.load_quantized(torch.from_numpy(gq[16:]), torch.from_numpy(gd[16:].view(np.int16)),
                       torch.from_numpy(dq[16:]), torch.from_numpy(dd[16:].view(np.int16)), capi.F16)
    x = dev(xb.view(np.int16)).view(torch.bfloat16)
    y = torch.empty((T, H), dtype=torch.float32, device="cuda")
    eng.forward(x, y, dev(ids), dev(w), capi.BF16, capi.F32)
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    ids_l = np.where(ids >= 16, ids - 16, -1).astype(np.int32)
    y_ref = O.moe_forward_q(1, False, xf, ids_l, w, gq[16:], gd[16:], dq[16:], dd[16:])
    rel, cos = parity(y.cpu().numpy(), y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


def test_cluster_kernel_deterministic():
    E, H, I, T = 128, 2048, 768, 2
    eng, _ = make_engine(2, E, H, I, 3)
    xb, _, ids, w = tokens(T, H, E, 8, 3)
    outs = [run(eng, xb, ids, w, H) for _ in range(3)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])
