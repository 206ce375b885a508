"""Expert parallelism with the in-kernel combine over NVLink peer memory (2 GPUs).

Two processes, one per GPU, each holding half of the experts; decode-size calls sum
the ranks' partials inside the fused kernel (mailboxes mapped through CUDA IPC),
larger calls take the fp32 partial + NCCL all-reduce.  Every output is compared with
the C oracle over all experts.  Skipped with fewer than two GPUs.
"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch

from tests.helpers import MAX_REL, MIN_COS, parity, q_weights, tokens

pytestmark = pytest.mark.gpu

CASES = [(1, 1), (3, 2), (8, 3), (40, 4)]  # (T, seed): T <= 8 in-kernel combine, 40 partial + all-reduce


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, outdir, qt, E, H, I, K, sk_min):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if sk_min is not None:
        os.environ["MOE_SK_MIN_CHUNKS"] = sk_min  # read when the engine is created
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    import moe_ascend_opt_b200  # noqa: F401
    from moe_ascend_opt_b200.ep import ExpertParallelMoE

    gq, gd, dq, dd = q_weights(qt, E, H, I, 5)
    moe = ExpertParallelMoE(E, H, I, qt)
    moe.load_quantized(torch.from_numpy(gq), torch.from_numpy(gd.view(np.int16)).view(torch.float16),
                       torch.from_numpy(dq), torch.from_numpy(dd.view(np.int16)).view(torch.float16))
    moe.connect_peers(8)
    for T, seed in CASES:
        xb, _, ids, w = tokens(T, H, E, K, seed)
        x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
        ids_t, w_t = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
        ys = [moe.forward(x, ids_t, w_t).float().cpu().numpy() for _ in range(3)]  # repeated: epochs, parity
        torch.cuda.synchronize()
        assert moe.handle.device_error() == 0
        for r, y in enumerate(ys):
            np.save(os.path.join(outdir, f"y_{rank}_{T}_{r}.npy"), y)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("sk_min", [None, "0"])  # default kernel choice / split-K kernel at every T
@pytest.mark.parametrize("qt", [1])
def test_two_rank_peer_combine_matches_oracle(qt, sk_min):
    import torch.multiprocessing as mp

    from oracle import oracle as O

    E, H, I, K = 32, 1024, 384, 8
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, _free_port(), d, qt, E, H, I, K, sk_min), nprocs=2, join=True)
        gq, gd, dq, dd = q_weights(qt, E, H, I, 5)
        for T, seed in CASES:
            _, xf, ids, w = tokens(T, H, E, K, seed)
            y_ref = O.moe_forward_q(qt, False, xf, ids, w, gq, gd, dq, dd)
            y0 = [np.load(os.path.join(d, f"y_0_{T}_{r}.npy")) for r in range(3)]
            y1 = [np.load(os.path.join(d, f"y_1_{T}_{r}.npy")) for r in range(3)]
            for a in y0 + y1:
                assert np.array_equal(a, y0[0])  # both ranks, every repeat: the same bits
            rel, cos = parity(y0[0], y_ref)
            assert rel <= MAX_REL and cos >= MIN_COS, (T, rel, cos)


def _dispatch_worker(rank, world, port, outdir, E, H, I, K, T):
    import torch.distributed as dist

    from tests.helpers import awq_weights

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    import moe_ascend_opt_b200  # noqa: F401
    from moe_ascend_opt_b200.ep import ExpertParallelMoE

    wts = awq_weights(E, H, I, 128, 7)
    moe = ExpertParallelMoE(E, H, I, 2)
    t = [torch.from_numpy(np.ascontiguousarray(a)) for a in wts]
    t[1], t[4] = t[1].view(torch.int16).view(torch.bfloat16), t[4].view(torch.int16).view(torch.bfloat16)
    moe.load_awq(*t)  # the torch class takes the scales as bfloat16 tensors
    xb, _, ids, w = tokens(T, H, E, K, 7)
    lo, hi = rank * T // world, (rank + 1) * T // world  # this rank's own tokens
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)[lo:hi]
    y = moe.forward_dispatch(x, torch.from_numpy(ids[lo:hi]).cuda(), torch.from_numpy(w[lo:hi]).cuda())
    torch.cuda.synchronize()
    assert moe.handle.device_error() == 0
    np.save(os.path.join(outdir, f"d_{rank}.npy"), y.float().cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("T", [2, 37])
def test_two_rank_token_dispatch_awq_matches_oracle(T):
    """Token-sharded ranks, token all-to-all dispatch and combine over NCCL (AWQ, the MiniMax
    format): each rank's rows equal the oracle's rows for its own tokens."""
    import torch.multiprocessing as mp

    from oracle import oracle as O
    from tests.helpers import awq_weights

    E, H, I, K = 32, 1024, 512, 8
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_dispatch_worker, args=(2, _free_port(), d, E, H, I, K, T), nprocs=2, join=True)
        _, xf, ids, w = tokens(T, H, E, K, 7)
        y_ref = O.moe_forward_awq(xf, ids, w, *awq_weights(E, H, I, 128, 7), group=128)
        y = np.concatenate([np.load(os.path.join(d, f"d_{r}.npy")) for r in range(2)])
        rel, cos = parity(y, y_ref)
        assert rel <= MAX_REL and cos >= MIN_COS, (rel, cos)
