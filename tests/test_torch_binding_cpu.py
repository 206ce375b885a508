"""The torch.ops.nanovllm / torch.classes.nanovllm surface without a GPU:
registration, argument validation with the reference's messages
(Int8-gemm/nanovllm_ops.cpp:349-431, moe_infer.cpp:27-31,100-134), and no CPU
fallback: CPU tensors fail loudly."""
import pytest
import torch

import moe_ascend_opt_b200  # noqa: F401


def test_surface_registered():
    for op in ("moe_forward", "moe_forward_npu_stream", "moe_forward_npu_graph_out", "moe_forward_partial",
               "moe_route", "moe_route_permute", "quantize_rows_q8_0"):
        assert hasattr(torch.ops.nanovllm, op)
    h = torch.classes.nanovllm.MoEInfer(128, 2048, 768, 1)
    assert h.get_quant_type() == "Q4_0"
    assert (h.get_num_experts(), h.get_hidden_size(), h.get_intermediate_size()) == (128, 2048, 768)
    assert torch.classes.nanovllm.MoEInfer(8, 256, 128, 0).get_quant_type() == "Q8_0"
    assert torch.classes.nanovllm.MoEInfer(8, 256, 128, 2).get_quant_type() == "AWQ"
    torch.classes.nanovllm.NpuCallbackManager(0, 0)
    assert h.get_last_run_time_ms() == 0.0


def test_constructor_checks():
    with pytest.raises(RuntimeError, match="hidden_size must be multiple of 32"):
        torch.classes.nanovllm.MoEInfer(8, 100, 128, 0)
    with pytest.raises(RuntimeError, match="intermediate_size must be multiple of 32"):
        torch.classes.nanovllm.MoEInfer(8, 128, 100, 0)
    with pytest.raises(RuntimeError, match="quant_type"):
        torch.classes.nanovllm.MoEInfer(8, 128, 128, 5)


def test_q4_online_quantize_rejected():
    h = torch.classes.nanovllm.MoEInfer(8, 256, 128, 1)
    with pytest.raises(RuntimeError, match="Q4_0 does not support online quantization"):
        h.quantize_and_store_expert(0, "gate_proj", torch.zeros(128, 256))


def test_store_checks_before_device_work():
    h = torch.classes.nanovllm.MoEInfer(8, 256, 128, 0)
    qs = torch.zeros(8, 256, 256, dtype=torch.int8)
    d = torch.zeros(8, 256, 8, dtype=torch.float32)
    with pytest.raises(RuntimeError, match="gate_up_d must be float16 or bfloat16"):
        h.store_quantized_repack(qs, d, qs, d)
    d16 = torch.zeros(8, 256, 8, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="gate_up_d and down_proj_d must have the same dtype"):
        h.store_quantized_repack(qs, d16, qs, d16.to(torch.bfloat16))
    with pytest.raises(RuntimeError, match="Q8_0 gate_up_qs must be int8"):
        h.store_quantized_repack(qs.to(torch.int32), d16, qs, d16)
    with pytest.raises(RuntimeError, match="Unknown proj_name"):
        h.quantize_and_store_expert(0, "bogus", torch.zeros(128, 256))


def test_no_cpu_fallback():
    h = torch.classes.nanovllm.MoEInfer(8, 256, 128, 0)
    x = torch.zeros(1, 256, dtype=torch.bfloat16)
    ids = torch.zeros(1, 8, dtype=torch.int32)
    w = torch.zeros(1, 8, dtype=torch.float32)
    with pytest.raises(Exception):
        torch.ops.nanovllm.moe_forward(x, ids, w, h)


def test_expert_parallel_config_checks():
    h = torch.classes.nanovllm.MoEInfer(8, 256, 128, 0)
    with pytest.raises(RuntimeError, match="bad expert-parallel config"):
        h.set_expert_parallel(2, 2)
    # 8 experts in contiguous blocks do not split over 3 ranks (a placement with replicated
    # experts may); refused when the weights arrive
    h3 = torch.classes.nanovllm.MoEInfer(8, 256, 128, 0)
    h3.set_expert_parallel(0, 3)
    with pytest.raises(RuntimeError, match="bad expert-parallel config"):
        h3.store_quantized_repack(torch.zeros((8, 256, 256), dtype=torch.int8),
                                  torch.zeros((8, 256, 8), dtype=torch.float16),
                                  torch.zeros((8, 256, 128), dtype=torch.int8),
                                  torch.zeros((8, 256, 4), dtype=torch.float16))
    h.set_expert_parallel(1, 2)
