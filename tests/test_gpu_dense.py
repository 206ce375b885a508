"""Dense MLP / shared expert through the fused kernels: moe_engine_forward_dense (and
torch.ops.nanovllm.moe_dense_forward) against the oracle with one expert at weight 1, and a
shared expert fused into the routed layer as an extra top-k column equal to the routed layer
plus the dense call."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import MAX_REL, MIN_COS, parity, q_weights, tokens

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import moe_ascend_opt_b200  # noqa: F401
    from moe_ascend_opt_b200 import capi


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("qt,T", [(0, 1), (1, 1), (1, 6), (1, 100), (0, 40)])
def test_dense_forward_matches_oracle(qt, T):
    E, H, I = 4, 1024, 512
    gq, gd, dq, dd = q_weights(qt, E, H, I, 70 + T)
    eng = capi.Engine(E, H, I, qt)
    eng.load_quantized(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)), torch.from_numpy(dq),
                       torch.from_numpy(dd.view(np.int16)), capi.F16)
    xb, xf, _, _ = tokens(T, H, E, 1, 70 + T)
    x = dev(xb.view(np.int16)).view(torch.bfloat16)
    for expert in (2, 0):
        y = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
        eng.forward_dense(expert, x, y, capi.BF16, capi.BF16)
        torch.cuda.synchronize()
        assert eng.device_error() == 0
        ids = np.full((T, 1), expert, np.int32)
        w = np.ones((T, 1), np.float32)
        rel, cos = parity(y.float().cpu().numpy(), O.moe_forward_q(qt, False, xf, ids, w, gq, gd, dq, dd))
        assert rel <= MAX_REL and cos >= MIN_COS, (expert, rel, cos)


def test_shared_expert_as_extra_column():
    """Routed top-8 over experts 0..15 plus shared expert 16 with a per-token gate, in one
    call, equals the routed call plus the gated dense call."""
    E, H, I, T, K = 17, 1024, 512, 5, 8
    gq, gd, dq, dd = q_weights(1, E, H, I, 81)
    h = torch.classes.nanovllm.MoEInfer(E, H, I, 1)
    h.store_quantized_repack(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)).view(torch.float16),
                             torch.from_numpy(dq), torch.from_numpy(dd.view(np.int16)).view(torch.float16))
    xb, xf, ids, w = tokens(T, H, 16, K, 81)
    gate = np.random.default_rng(1).uniform(0.2, 0.9, size=(T, 1)).astype(np.float32)
    ids9 = np.concatenate([ids, np.full((T, 1), 16, np.int32)], 1)
    w9 = np.concatenate([w, gate], 1)
    x = dev(xb.view(np.int16)).view(torch.bfloat16)
    y_fused = torch.ops.nanovllm.moe_forward(x, dev(ids9), dev(w9), h).float()
    y_routed = torch.ops.nanovllm.moe_forward_partial(x, dev(ids), dev(w), h)
    y_shared = torch.ops.nanovllm.moe_dense_forward(x, 16, h).float()
    torch.cuda.synchronize()
    rel, cos = parity(y_fused.cpu().numpy(), (y_routed + torch.from_numpy(gate).cuda() * y_shared).cpu().numpy())
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)
    y_ref = O.moe_forward_q(1, False, xf, ids9, w9, gq, gd, dq, dd)
    rel, cos = parity(y_fused.cpu().numpy(), y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)
