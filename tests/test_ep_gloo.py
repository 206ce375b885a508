"""Expert-parallel decomposition on CPU ranks (gloo, world size 2).

Each rank evaluates the oracle over its block of experts with the ids remapped
the way the kernel remaps them (others -> -1), the fp32 partials are summed by
an all-reduce, and the result must equal the single-rank forward.  This is the
host-side contract the GPU path follows with NCCL.  A second test checks that a
rank that fails before the collective makes its peer's collective fail instead
of hanging (short process-group timeout)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from moe_ascend_opt_b200.ep import expert_partition, local_ids


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, qt, result_q):
    from oracle import oracle as O
    from tests.helpers import q_weights, tokens
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    E, H, I, T, K = 16, 256, 128, 5, 8
    gq, gd, dq, dd = q_weights(qt, E, H, I, 31)
    _, xf, ids, w = tokens(T, H, E, K, 31)
    lo, hi = expert_partition(E, world)[rank]
    part = O.moe_forward_q(qt, False, xf, local_ids(ids, lo, hi), w, gq[lo:hi], gd[lo:hi], dq[lo:hi], dd[lo:hi])
    t = torch.from_numpy(part)
    dist.all_reduce(t)
    if rank == 0:
        full = O.moe_forward_q(qt, False, xf, ids, w, gq, gd, dq, dd)
        result_q.put(float(np.abs(t.numpy() - full).max() / np.abs(full).max()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("qt", [0, 1])
def test_ep_partials_sum_to_full_forward(qt):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, qt, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=5) < 1e-5


def _failing_worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # this rank dies between steps, before the combine
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        result_q.put("completed")
    except Exception as ex:  # the survivor learns of it from the collective, it does not hang
        result_q.put("error:" + type(ex).__name__)


def test_dead_rank_fails_collective_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert procs[1].exitcode == 3
    assert q.get(timeout=5).startswith("error:")


def test_partition_and_remap():
    assert expert_partition(128, 8)[3] == (48, 64)
    with pytest.raises(ValueError):
        expert_partition(10, 4)
    ids = np.array([[0, 5, 9, -1, 16]], np.int32)
    assert local_ids(ids, 4, 12).tolist() == [[-1, 1, 5, -1, -1]]


def test_balanced_placement_evens_zipf_load():
    from moe_ascend_opt_b200.ep import balanced_placement, placement_imbalance
    E, W = 128, 8
    load = 1.0 / np.arange(1, E + 1) ** 1.2  # Zipf(s=1.2) tokens per expert
    rng = np.random.default_rng(3)
    load = load[rng.permutation(E)]
    pl = balanced_placement(load, W)
    assert sorted(e for r in pl for e in r) == list(range(E))
    assert all(len(r) == E // W for r in pl)
    contiguous = [list(range(r * E // W, (r + 1) * E // W)) for r in range(W)]
    assert placement_imbalance(load, pl) < placement_imbalance(load, contiguous)
    # the hottest expert alone bounds the balance from below; the rest is dealt evenly
    assert placement_imbalance(load, pl) <= (load.max() + load.sum() / W) / (load.sum() / W)


@pytest.mark.parametrize("qt", [0, 1])
def test_placed_partials_sum_to_full_forward(qt):
    # non-contiguous expert sets per rank, ids remapped through the per-rank table
    from oracle import oracle as O
    from moe_ascend_opt_b200.ep import balanced_placement, local_ids_map
    from tests.helpers import q_weights, tokens
    E, H, I, T, K, W = 16, 256, 128, 6, 8, 2
    gq, gd, dq, dd = q_weights(qt, E, H, I, 17)
    _, xf, ids, w = tokens(T, H, E, K, 17)
    load = np.bincount(ids.ravel(), minlength=E)
    pl = balanced_placement(load, W)
    total = sum(O.moe_forward_q(qt, False, xf, local_ids_map(ids, ex), w, gq[ex], gd[ex], dq[ex], dd[ex]) for ex in pl)
    full = O.moe_forward_q(qt, False, xf, ids, w, gq, gd, dq, dd)
    assert float(np.abs(total - full).max() / np.abs(full).max()) < 1e-5


def test_replicated_placement_evens_zipf_load():
    """Replicating the hottest experts on every rank removes the floor that one hot expert
    puts under the balanced placement's imbalance."""
    from moe_ascend_opt_b200.ep import balanced_placement, placement_imbalance, replicated_placement
    E, W = 128, 8
    load = 1.0 / np.arange(1, E + 1) ** 1.2
    load = load[np.random.default_rng(3).permutation(E)]
    pl, hot = replicated_placement(load, W, 8)
    assert len(hot) == 8 and all(set(hot) <= set(r) for r in pl)
    own = [e for r in pl for e in r if e not in hot]
    assert sorted(own + hot) == list(range(E))
    assert placement_imbalance(load, pl, hot) < 1.1 < placement_imbalance(load, balanced_placement(load, W))


def replica_local_ids(ids, experts, hot, rank, world):
    """The kernels' rule for a rank holding `experts` (local order) with replicated `hot`:
    a pair of a hot expert g is this rank's when (t + g) % world == rank."""
    from moe_ascend_opt_b200.ep import local_ids_map
    loc = local_ids_map(ids, experts)
    t = np.arange(ids.shape[0])[:, None]
    mine = ((t + ids) % world) == rank
    is_hot = np.isin(ids, hot)
    return np.where(is_hot & ~mine, -1, loc).astype(np.int32)


@pytest.mark.parametrize("qt", [0, 1])
def test_replicated_partials_sum_to_full_forward(qt):
    from oracle import oracle as O
    from moe_ascend_opt_b200.ep import replicated_placement
    from tests.helpers import q_weights, tokens
    E, H, I, T, K, W = 16, 256, 128, 9, 4, 2
    gq, gd, dq, dd = q_weights(qt, E, H, I, 19)
    _, xf, ids, w = tokens(T, H, E, K, 19)
    load = np.bincount(ids.ravel(), minlength=E)
    pl, hot = replicated_placement(load, W, 2)
    total = sum(O.moe_forward_q(qt, False, xf, replica_local_ids(ids, ex, hot, r, W), w, gq[ex], gd[ex], dq[ex],
                                dd[ex]) for r, ex in enumerate(pl))
    full = O.moe_forward_q(qt, False, xf, ids, w, gq, gd, dq, dd)
    assert float(np.abs(total - full).max() / np.abs(full).max()) < 1e-5


def _dispatch_worker(rank, world, port, placed, result_q):
    from oracle import oracle as O
    from tests.helpers import q_weights, tokens
    from moe_ascend_opt_b200.ep import balanced_placement, dispatch_forward, expert_owner, local_ids_map
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    E, H, I, K = 16, 256, 128, 8
    counts = [5, 3, 0, 2][:world]  # token-sharded: each rank its own tokens (one rank none at 4)
    T = counts[rank]
    gq, gd, dq, dd = q_weights(1, E, H, I, 41)
    _, xf_all, ids_all, w_all = tokens(sum(counts), H, E, K, 41)
    off = sum(counts[:rank])
    xf, ids, w = xf_all[off:off + T].copy(), ids_all[off:off + T].copy(), w_all[off:off + T].copy()
    if rank == 0 and T:
        ids[0, :3] = 9      # an expert three times in a token
        ids[1, 2] = -1      # invalid ids travel as -1
    placement = balanced_placement(np.bincount(ids_all.ravel(), minlength=E), world) if placed else None
    owner = expert_owner(E, world, placement)
    mine = placement[rank] if placed else list(range(rank * E // world, (rank + 1) * E // world))
    sel = np.asarray(mine)

    def compute(x, i, wt):  # this rank's experts over the received rows (the engine's role)
        li = local_ids_map(i.numpy(), mine)
        return torch.from_numpy(O.moe_forward_q(1, False, x.numpy(), li, wt.numpy(),
                                                gq[sel], gd[sel], dq[sel], dd[sel]))

    y = dispatch_forward(torch.from_numpy(xf), torch.from_numpy(ids), torch.from_numpy(w), owner, world, compute)
    full = O.moe_forward_q(1, False, xf, ids, w, gq, gd, dq, dd) if T else np.zeros((0, H), np.float32)
    err = float(np.abs(y.numpy() - full).max() / max(np.abs(full).max(), 1e-30)) if T else 0.0
    result_q.put((rank, err, tuple(y.shape)))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,placed", [(2, False), (2, True), (4, True)])
def test_token_all_to_all_dispatch(world, placed):
    """Token-sharded ranks (5, 3 and 0 tokens): every routed row goes to the ranks owning its
    experts, the partials come back and each rank's output equals the single-rank forward of
    its own tokens (contiguous blocks, load-balanced placement, a rank with no tokens)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dispatch_worker, args=(r, world, port, placed, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    assert all(p.exitcode == 0 for p in procs)
    res = sorted(q.get(timeout=5) for _ in range(world))
    for rank, err, shape in res:
        assert err <= 1e-5, (rank, err)
