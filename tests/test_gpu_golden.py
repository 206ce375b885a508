"""GPU path against the reference's own outputs at the BASELINE shapes
(H=2048, I=768, E=128, top-8), through the C ABI and through the torch ops.

fwd_c1_q8: configs[0], weights quantised online on the GPU by
quantize_and_store_expert (bit-exact with quantize_weight_only, checked in
test_gpu_parity) and the reference's own online quantiser for the fixture.
fwd_c2_q4_T*: configs[1], Q4_0 weights, token sweep 1/4/8/32."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import MAX_REL, MIN_COS, expert_weights_fp32, parity

pytestmark = pytest.mark.gpu

H, I, E, K = 2048, 768, 128, 8

if torch.cuda.is_available():
    import moe_ascend_opt_b200  # noqa: F401


def gold(name):
    import os
    return np.load(os.path.join(os.path.dirname(__file__), "golden", name))


def test_c1_q8_online_quantised_matches_reference():
    f = gold("fwd_c1_q8.npz")
    seed = int(f["seed"])
    h = torch.classes.nanovllm.MoEInfer(E, H, I, 0)
    for e in np.unique(f["ids"]):
        wg, wu, wd = expert_weights_fp32(int(e), seed, H, I)
        h.quantize_and_store_expert(int(e), "gate_proj", torch.from_numpy(wg).cuda())
        h.quantize_and_store_expert(int(e), "up_proj", torch.from_numpy(wu))
        h.quantize_and_store_expert(int(e), "down_proj", torch.from_numpy(wd).to(torch.float32))
    x = torch.from_numpy(f["xb"].view(np.int16)).cuda().view(torch.bfloat16)
    y = torch.ops.nanovllm.moe_forward(x, torch.from_numpy(f["ids"]).cuda(), torch.from_numpy(f["w"]).cuda(), h)
    torch.cuda.synchronize()
    rel, cos = parity(y.float().cpu().numpy(), O.bf16_bits_to_f32(f["y"]))
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)
    assert h.get_last_run_time_ms() > 0.0


@pytest.mark.parametrize("T", [1, 4, 8, 32])
def test_c2_q4_sweep_matches_reference(T):
    f = gold(f"fwd_c2_q4_T{T}.npz")
    seed = int(f["seed"])
    gq = np.zeros((E, 2 * I, H // 8), np.int32)
    gd = np.zeros((E, 2 * I, H // 32), np.uint16)
    dq = np.zeros((E, H, I // 8), np.int32)
    dd = np.zeros((E, H, I // 32), np.uint16)
    for e in np.unique(f["ids"]):
        wg, wu, wd = expert_weights_fp32(int(e), seed, H, I)
        gq[e], gd[e] = O.quantize_weight_q4_0(np.concatenate([wg, wu], 0))
        dq[e], dd[e] = O.quantize_weight_q4_0(wd)
    h = torch.classes.nanovllm.MoEInfer(E, H, I, 1)
    h.store_quantized_repack(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)).view(torch.float16),
                             torch.from_numpy(dq), torch.from_numpy(dd.view(np.int16)).view(torch.float16))
    x = torch.from_numpy(f["xb"].view(np.int16)).cuda().view(torch.bfloat16)
    y = torch.ops.nanovllm.moe_forward(x, torch.from_numpy(f["ids"]).cuda(), torch.from_numpy(f["w"]).cuda(), h)
    torch.cuda.synchronize()
    rel, cos = parity(y.float().cpu().numpy(), O.bf16_bits_to_f32(f["y"]))
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)


def test_graph_out_and_cuda_graph_replay():
    """MoEGraphContext + moe_forward_npu_graph_out inside a captured CUDA graph."""
    f = gold("fwd_c2_q4_T4.npz")
    seed = int(f["seed"])
    gq = np.zeros((E, 2 * I, H // 8), np.int32)
    gd = np.zeros((E, 2 * I, H // 32), np.uint16)
    dq = np.zeros((E, H, I // 8), np.int32)
    dd = np.zeros((E, H, I // 32), np.uint16)
    for e in np.unique(f["ids"]):
        wg, wu, wd = expert_weights_fp32(int(e), seed, H, I)
        gq[e], gd[e] = O.quantize_weight_q4_0(np.concatenate([wg, wu], 0))
        dq[e], dd[e] = O.quantize_weight_q4_0(wd)
    h = torch.classes.nanovllm.MoEInfer(E, H, I, 1)
    h.store_quantized_repack(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)).view(torch.float16),
                             torch.from_numpy(dq), torch.from_numpy(dd.view(np.int16)).view(torch.float16))
    T = f["ids"].shape[0]
    ctx = torch.classes.nanovllm.MoEGraphContext(h, T, K, 1)
    x = torch.from_numpy(f["xb"].view(np.int16)).cuda().view(torch.bfloat16)
    ids = torch.from_numpy(f["ids"]).cuda()
    w = torch.from_numpy(f["w"]).cuda()
    out = torch.empty_like(x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        torch.ops.nanovllm.moe_forward_npu_graph_out(x, ids, w, h, ctx, out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        torch.ops.nanovllm.moe_forward_npu_graph_out(x, ids, w, h, ctx, out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    rel, cos = parity(out.float().cpu().numpy(), O.bf16_bits_to_f32(f["y"]))
    assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)
    y2 = torch.ops.nanovllm.moe_forward_npu_stream(x, ids, w, h)
    torch.cuda.synchronize()
    assert torch.equal(y2, out)


def test_expert_parallel_partials_on_one_gpu():
    """Two engines holding expert halves (the EP layout) sum to the single engine."""
    from tests.helpers import q_weights, tokens
    E2, H2, I2, T = 16, 512, 256, 4
    gq, gd, dq, dd = q_weights(1, E2, H2, I2, 8)
    xb, xf, ids, w = tokens(T, H2, E2, K, 8)
    tens = [torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)).view(torch.float16),
            torch.from_numpy(dq), torch.from_numpy(dd.view(np.int16)).view(torch.float16)]
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    idt, wt = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
    parts = []
    for r in range(2):
        h = torch.classes.nanovllm.MoEInfer(E2, H2, I2, 1)
        h.set_expert_parallel(r, 2)
        h.store_quantized_repack(*tens)
        parts.append(torch.ops.nanovllm.moe_forward_partial(x, idt, wt, h))
    y = (parts[0] + parts[1]).cpu().numpy()
    rel, cos = parity(y, O.moe_forward_q(1, False, xf, ids, w, gq, gd, dq, dd))
    assert rel <= 2e-3 and cos >= MIN_COS, (rel, cos)


@pytest.mark.parametrize("T", [1, 40])  # decode kernel / grouped GEMMs
def test_expert_placement_partials_on_one_gpu(T):
    """Two engines with interleaved (non-contiguous) expert sets sum to the full layer."""
    import moe_ascend_opt_b200  # noqa: F401
    from oracle import oracle as O
    from tests.helpers import q_weights, tokens
    E, H, I, K = 32, 1024, 384, 8
    gq, gd, dq, dd = q_weights(1, E, H, I, 23)
    xb, xf, ids, w = tokens(T, H, E, K, 23)
    placement = [list(range(0, E, 2)), list(range(1, E, 2))]
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    total = None
    for r in range(2):
        h = torch.classes.nanovllm.MoEInfer(E, H, I, 1)
        h.set_expert_parallel(r, 2)
        h.set_expert_placement(placement[r])
        h.store_quantized_repack(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)).view(torch.float16),
                                 torch.from_numpy(dq), torch.from_numpy(dd.view(np.int16)).view(torch.float16))
        part = torch.ops.nanovllm.moe_forward_partial(x, torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), h)
        torch.cuda.synchronize()
        assert h.device_error() == 0
        total = part if total is None else total + part
    y_ref = O.moe_forward_q(1, False, xf, ids, w, gq, gd, dq, dd)
    rel = float(np.abs(total.cpu().numpy() - y_ref).max() / np.abs(y_ref).max())
    assert rel <= 1e-2, rel


@pytest.mark.parametrize("T,cl", [(1, "0"), (1, "8"), (5, "0"), (5, "8"), (64, "0")])
def test_replicated_hot_experts_on_one_gpu(T, cl):
    """Engines of 3 ranks on one GPU with 2 hot experts replicated on all of them: the fp32
    partials sum to the full layer (decode kernels, cluster kernel, grouped GEMMs)."""
    import os
    from moe_ascend_opt_b200.ep import replicated_placement
    from tests.helpers import q_weights, tokens
    E, H, I, K, W = 32, 1024, 512, 8, 3
    gq, gd, dq, dd = q_weights(1, E, H, I, 29)
    xb, xf, ids, w = tokens(T, H, E, K, 29)
    load = np.bincount(ids.ravel(), minlength=E)
    pl, hot = replicated_placement(load, W, 2)
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    old = os.environ.get("MOE_CL_MAX_TOKENS")
    os.environ["MOE_CL_MAX_TOKENS"] = cl
    total = None
    try:
        for r in range(W):
            h = torch.classes.nanovllm.MoEInfer(E, H, I, 1)
            h.set_expert_parallel(r, W)
            h.set_expert_placement(pl[r])
            h.set_expert_replicas(hot)
            h.store_quantized_repack(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)).view(torch.float16),
                                     torch.from_numpy(dq), torch.from_numpy(dd.view(np.int16)).view(torch.float16))
            part = torch.ops.nanovllm.moe_forward_partial(x, torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), h)
            torch.cuda.synchronize()
            assert h.device_error() == 0
            total = part if total is None else total + part
    finally:
        if old is None:
            del os.environ["MOE_CL_MAX_TOKENS"]
        else:
            os.environ["MOE_CL_MAX_TOKENS"] = old
    y_ref = O.moe_forward_q(1, False, xf, ids, w, gq, gd, dq, dd)
    rel = float(np.abs(total.cpu().numpy() - y_ref).max() / np.abs(y_ref).max())
    assert rel <= 1e-2, rel
