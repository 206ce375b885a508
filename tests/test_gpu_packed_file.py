"""Packed-layout files (moe_engine_save / moe_engine_load_file, MoEInfer.save / load_file):
an engine filled from a file computes the same bits as the engine that wrote it, at decode
and grouped-GEMM sizes, for Q8_0, Q4_0 and AWQ; corrupted or mismatched files are refused."""
import os

import numpy as np
import pytest
import torch

from tests.helpers import awq_weights, q_weights, tokens

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import moe_ascend_opt_b200  # noqa: F401
    from moe_ascend_opt_b200 import capi


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def build(qt, E, H, I, seed):
    eng = capi.Engine(E, H, I, qt, group_size=128)
    if qt == capi.AWQ:
        eng.load_awq(*[torch.from_numpy(a) for a in awq_weights(E, H, I, 128, seed)])
    else:
        gq, gd, dq, dd = q_weights(qt, E, H, I, seed)
        eng.load_quantized(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)), torch.from_numpy(dq),
                           torch.from_numpy(dd.view(np.int16)), capi.F16)
    return eng


def fwd(eng, E, H, T, seed):
    xb, _, ids, w = tokens(T, H, E, 8, seed)
    x = dev(xb.view(np.int16)).view(torch.bfloat16)
    y = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    eng.forward(x, y, dev(ids), dev(w), capi.BF16, capi.BF16)
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    return y.cpu()


@pytest.mark.parametrize("qt", [0, 1, 2])
def test_file_round_trip_is_bit_exact(qt, tmp_path):
    E, H, I = 32, 1024, 512
    src = build(qt, E, H, I, 60 + qt)
    path = str(tmp_path / f"layer{qt}.moeb")
    src.save(path)
    dst = capi.Engine(E, H, I, qt, group_size=128)
    dst.load_file(path)
    for T in (1, 3, 64):
        assert torch.equal(fwd(src, E, H, T, T), fwd(dst, E, H, T, T)), T
    assert os.path.getsize(path) > 0


def test_file_refuses_corruption_and_mismatch(tmp_path):
    E, H, I = 16, 512, 256
    src = build(1, E, H, I, 5)
    path = str(tmp_path / "a.moeb")
    src.save(path)
    with pytest.raises(capi.MoeError, match="differs"):
        capi.Engine(E, H, 2 * I, 1).load_file(path)
    with pytest.raises(capi.MoeError, match="differs"):
        capi.Engine(E, H, I, 0).load_file(path)
    data = bytearray(open(path, "rb").read())
    data[-100] ^= 0x40
    bad = str(tmp_path / "b.moeb")
    open(bad, "wb").write(bytes(data))
    with pytest.raises(capi.MoeError, match="checksum"):
        capi.Engine(E, H, I, 1).load_file(bad)
    with pytest.raises(capi.MoeError, match="magic"):
        open(bad, "wb").write(b"not a layout file at all")
        capi.Engine(E, H, I, 1).load_file(bad)


def test_torch_handle_save_load(tmp_path):
    E, H, I = 16, 512, 256
    gq, gd, dq, dd = q_weights(1, E, H, I, 8)
    h = torch.classes.nanovllm.MoEInfer(E, H, I, 1)
    h.store_quantized_repack(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)).view(torch.float16),
                             torch.from_numpy(dq), torch.from_numpy(dd.view(np.int16)).view(torch.float16))
    path = str(tmp_path / "t.moeb")
    h.save(path)
    h2 = torch.classes.nanovllm.MoEInfer(E, H, I, 1)
    h2.load_file(path)
    xb, _, ids, w = tokens(4, H, E, 8, 2)
    x = dev(xb.view(np.int16)).view(torch.bfloat16)
    y1 = torch.ops.nanovllm.moe_forward(x, dev(ids), dev(w), h)
    y2 = torch.ops.nanovllm.moe_forward(x, dev(ids), dev(w), h2)
    assert torch.equal(y1, y2)
