"""BASELINE configs beyond the Qwen shape: the MiniMax-M2-shaped layer (H=3072, I=1536,
E=256, top-8) in Q4_0 and AWQ, and Zipf(1.2)-skewed routing (configs[2] run B), against
the C oracle.  Only the routed experts carry weights (the others stay zero), so the
oracle runs on the active experts with remapped ids."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import MAX_REL, MIN_COS, awq_weights, parity, q_weights, tokens

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import moe_ascend_opt_b200  # noqa: F401
    from moe_ascend_opt_b200 import capi


def zipf_ids(T, E, K, seed, s=1.2):
    rng = np.random.default_rng(seed)
    perm = rng.permutation(E)
    p = np.arange(1, E + 1, dtype=np.float64) ** -s
    p /= p.sum()
    ids = np.stack([perm[rng.choice(E, K, replace=False, p=p)] for _ in range(T)]).astype(np.int32)
    return ids, np.full((T, K), 1.0 / K, np.float32)


def run_subset(qt, E, H, I, T, K, seed, routing="softmax", G=128):
    xb, xf, ids, w = tokens(T, H, E, K, seed)
    if routing == "zipf":
        ids, w = zipf_ids(T, E, K, seed)
    act = np.unique(ids)
    A = len(act)
    rid = np.searchsorted(act, ids).astype(np.int32)
    if qt == capi.AWQ:
        sub = awq_weights(A, H, I, G, seed)  # active experts' weights
        full = []
        for a, shp in zip(sub, [(E, H, 2 * I // 8), (E, H // G, 2 * I), (E, H // G, 2 * I // 8),
                                (E, I, H // 8), (E, I // G, H), (E, I // G, H // 8)]):
            f = np.zeros(shp, a.dtype)
            f[act] = a
            full.append(torch.from_numpy(f))
        eng = capi.Engine(E, H, I, qt, group_size=G)
        eng.load_awq(*full)
        y_ref = O.moe_forward_awq(xf, rid, w, *sub, group=G)
    else:
        gq, gd, dq, dd = q_weights(qt, A, H, I, seed)
        full = [np.zeros((E,) + a.shape[1:], a.dtype) for a in (gq, gd, dq, dd)]
        for f, a in zip(full, (gq, gd, dq, dd)):
            f[act] = a
        eng = capi.Engine(E, H, I, qt)
        eng.load_quantized(torch.from_numpy(full[0]), torch.from_numpy(full[1].view(np.int16)),
                           torch.from_numpy(full[2]), torch.from_numpy(full[3].view(np.int16)), capi.F16)
        y_ref = O.moe_forward_q(qt, False, xf, rid, w, gq, gd, dq, dd)
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    y = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    eng.forward(x, y, torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), capi.BF16, capi.BF16)
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    return y.float().cpu().numpy(), y_ref


@pytest.mark.parametrize("qt,T", [(1, 1), (1, 8), (1, 128), (2, 1), (2, 8)])
def test_minimax_shape(qt, T):
    y, y_ref = run_subset(qt, 256, 3072, 1536, T, 8, seed=T + qt)
    rel, cos = parity(y, y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


@pytest.mark.parametrize("qt,T", [(1, 4), (2, 4), (0, 64)])
def test_zipf_routing(qt, T):
    y, y_ref = run_subset(qt, 128, 2048, 768, T, 8, seed=40 + T, routing="zipf")
    rel, cos = parity(y, y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)
