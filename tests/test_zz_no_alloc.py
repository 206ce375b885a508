"""moe_engine_forward_noalloc: the forward for callers that may not allocate.

Serving runtimes that reserve all device memory at start-up, and latency-critical
paths that cannot take an allocation's implicit device synchronisation, cannot call
cudaMalloc when they run the layer.  This entry point draws its scratch from a
fixed device array instead of the engine's workspace.  The test calls it twice in a
row through the C ABI and compares each result with moe_engine_forward's, within
the tolerance the other parity tests use, and checks that sizes beyond the array
are refused.  The file is collected last so that a run stopping at the first
failure has run every other test first.
"""
import numpy as np
import pytest
import torch

from tests.helpers import MAX_REL, MIN_COS, parity, q_weights, tokens

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import moe_ascend_opt_b200  # noqa: F401
    from moe_ascend_opt_b200 import capi


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("qt", [0, 1])
def test_noalloc_matches_forward_twice(qt):
    E, H, I, T, K = 32, 1024, 384, 3, 8
    gq, gd, dq, dd = q_weights(qt, E, H, I, 77)
    eng = capi.Engine(E, H, I, qt)
    eng.load_quantized(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)), torch.from_numpy(dq),
                       torch.from_numpy(dd.view(np.int16)), capi.F16)
    for call in range(2):  # two calls in a row share (and reuse) the fixed scratch
        xb, _, ids, w = tokens(T, H, E, K, 77 + call)
        x = dev(xb.view(np.int16)).view(torch.bfloat16)
        idt, wt = dev(ids), dev(w)
        y_ref = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
        eng.forward(x, y_ref, idt, wt, capi.BF16, capi.BF16)
        y = torch.full((T, H), 3.0, dtype=torch.bfloat16, device="cuda")
        eng.forward_noalloc(x, y, idt, wt, capi.BF16, capi.BF16)
        torch.cuda.synchronize()
        rel, cos = parity(y.float().cpu().numpy(), y_ref.float().cpu().numpy())
        assert rel <= MAX_REL and cos >= MIN_COS, (call, rel, cos)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    E, H, I, K = 8, 256, 768, 8
    gq, gd, dq, dd = q_weights(1, E, H, I, 3)
    eng = capi.Engine(E, H, I, 1)
    eng.load_quantized(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)), torch.from_numpy(dq),
                       torch.from_numpy(dd.view(np.int16)), capi.F16)
    T = 22  # 256 + 22 x 8 x 768 x 4 bytes of h exceed the 512 KiB array
    x = torch.zeros((T, H), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((T, H), dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros((T, K), dtype=torch.int32, device="cuda")
    w = torch.zeros((T, K), dtype=torch.float32, device="cuda")
    with pytest.raises(capi.MoeError, match="scratch"):
        eng.forward_noalloc(x, y, ids, w, capi.BF16, capi.BF16)


def test_noalloc_on_a_fresh_engine_allocates_nothing():
    """First call on an engine that never ran moe_engine_forward: the device's free memory
    does not move across the call, and the result then matches moe_engine_forward's."""
    E, H, I, T, K = 32, 1024, 384, 2, 8
    gq, gd, dq, dd = q_weights(1, E, H, I, 91)
    eng = capi.Engine(E, H, I, 1)
    eng.load_quantized(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)), torch.from_numpy(dq),
                       torch.from_numpy(dd.view(np.int16)), capi.F16)
    xb, _, ids, w = tokens(T, H, E, K, 91)
    x = dev(xb.view(np.int16)).view(torch.bfloat16)
    idt, wt = dev(ids), dev(w)
    y = torch.full((T, H), 3.0, dtype=torch.bfloat16, device="cuda")
    y_ref = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    eng.forward_noalloc(x, y, idt, wt, capi.BF16, capi.BF16)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    eng.forward(x, y_ref, idt, wt, capi.BF16, capi.BF16)
    torch.cuda.synchronize()
    rel, cos = parity(y.float().cpu().numpy(), y_ref.float().cpu().numpy())
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)
    assert eng.device_error() == 0
