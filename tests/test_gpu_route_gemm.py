"""Router GEMM + top-k (moe_route_gemm_topk / torch.ops.nanovllm.moe_route_gemm): the
fp32 logits against a float64 product, the selection bit-exact against the oracle's top-k
of the kernel's own logits (Int8-gemm/test/fused_moe_cpu.py:20-37), and the selected ids
against the float64 ranking wherever the top-K boundary is not a near tie."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import moe_ascend_opt_b200  # noqa: F401
    from moe_ascend_opt_b200 import capi


@pytest.mark.parametrize("T,H,E,K,wdt,renorm", [(1, 2048, 128, 8, torch.float32, True),
                                                 (7, 2048, 128, 8, torch.bfloat16, True),
                                                 (33, 3072, 256, 8, torch.float32, False),
                                                 (5, 1024, 64, 10, torch.float16, True)])
def test_route_gemm_matches_reference(T, H, E, K, wdt, renorm):
    g = torch.Generator().manual_seed(T * 1000 + E)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16)
    w = (torch.randn((E, H), generator=g) * 0.02).to(wdt)
    logits = torch.empty((T, E), dtype=torch.float32, device="cuda")
    ids, tw = capi.route_gemm_topk(x.cuda(), w.cuda(), K, renorm, logits=logits)
    torch.cuda.synchronize()
    ref = x.double() @ w.double().t()
    lg = logits.cpu()
    assert torch.allclose(lg.double(), ref, rtol=1e-4, atol=1e-4), float((lg.double() - ref).abs().max())
    oi, ow = O.topk_softmax(lg.numpy(), K, renorm)
    assert np.array_equal(ids.cpu().numpy(), oi)
    np.testing.assert_allclose(tw.cpu().numpy(), ow, rtol=1e-5, atol=1e-7)
    srt = torch.sort(ref, dim=1, descending=True).values
    robust = (srt[:, K - 1] - srt[:, K]) > 1e-3
    want = torch.topk(ref, K, dim=1).indices
    got = ids.cpu().long()
    assert torch.equal(torch.sort(got[robust], 1).values, torch.sort(want[robust], 1).values)


def test_route_gemm_torch_op_feeds_forward():
    """The op's ids / weights drive moe_forward (the fused pre-step of a MoE layer)."""
    E, H, I, T, K = 16, 512, 256, 4, 8
    from tests.helpers import q_weights
    gq, gd, dq, dd = q_weights(1, E, H, I, 4)
    h = torch.classes.nanovllm.MoEInfer(E, H, I, 1)
    h.store_quantized_repack(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)).view(torch.float16),
                             torch.from_numpy(dq), torch.from_numpy(dd.view(np.int16)).view(torch.float16))
    g = torch.Generator().manual_seed(3)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16).cuda()
    wr = (torch.randn((E, H), generator=g) * 0.05).cuda()
    ids, tw = torch.ops.nanovllm.moe_route_gemm(x, wr, K, True)
    ids2, tw2 = torch.ops.nanovllm.moe_route((x.float() @ wr.t()).contiguous(), K, True)
    torch.cuda.synchronize()
    assert torch.equal(torch.sort(ids, 1).values, torch.sort(ids2, 1).values)
    y = torch.ops.nanovllm.moe_forward(x, ids, tw, h)
    y_ref = O.moe_forward_q(1, False, x.float().cpu().numpy(), ids.cpu().numpy(), tw.cpu().numpy(), gq, gd, dq, dd)
    from tests.helpers import MAX_REL, MIN_COS, parity
    rel, cos = parity(y.float().cpu().numpy(), y_ref)
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)
