"""Expert parallelism across the GPUs of one node (one process per GPU).

Experts are placed in contiguous blocks by default: rank r of W holds global experts
[r*E/W, (r+1)*E/W); `balanced_placement` deals them by routing load instead (skewed,
e.g. Zipf, routing), and the kernels then map ids through a per-rank table.  Every rank receives the full hidden states and routing
(as in the reference's caller, which hands the same [T,H] to the engine), runs
the fused layer over its local experts only -- ids outside the block are
skipped exactly like invalid ids in the reference (moe_common.cpp:158,175-181)
-- and produces an fp32 partial sum; one all-reduce over NCCL (NVLink /
NVSwitch) adds the partials, then the result is cast to the hidden dtype.
After `connect_peers()`, decode-size calls instead sum the partials inside the fused
kernel: each CTA stores its output rows into every rank's mailbox over NVLink and waits
(bounded) for the same CTA of the other ranks.
This replaces the reference's NUMA "TP" split (moe_infer.cpp:143-205,
q8_gemm.cpp:621-641), whose node-0 reduction becomes the all-reduce.

Token-sharded callers (data-parallel attention: each rank holds its own tokens) use
`forward_dispatch` instead: every token row is sent once to each rank that owns one of its
experts (NCCL all-to-all), each rank runs the fused layer on the rows it received (fp32
partial), and a second all-to-all returns the partials, which the token's rank adds in
rank order.  The traffic per layer is the routed rows (2 x T x fan-out x H values) instead
of an all-reduce of the whole [T, H] output.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import numpy as np


def expert_partition(num_experts: int, world: int) -> List[Tuple[int, int]]:
    """[lo, hi) of global expert ids held by each rank."""
    if world < 1 or num_experts % world != 0:
        raise ValueError(f"num_experts={num_experts} must be divisible by the world size {world}")
    per = num_experts // world
    return [(r * per, (r + 1) * per) for r in range(world)]


def balanced_placement(load, world: int) -> List[List[int]]:
    """Experts -> ranks from routing statistics (tokens per expert, e.g. counted over a
    calibration batch): every rank keeps E/W experts (equal weight memory), and the
    experts are dealt heaviest first to the rank with the least load that still has room,
    so Zipf-skewed routing no longer piles the hot experts onto one rank."""
    load = np.asarray(load, np.float64)
    E = load.shape[0]
    if world < 1 or E % world != 0:
        raise ValueError(f"num_experts={E} must be divisible by the world size {world}")
    per = E // world
    ranks: List[List[int]] = [[] for _ in range(world)]
    tot = np.zeros(world)
    for e in np.argsort(-load, kind="stable"):
        open_r = [r for r in range(world) if len(ranks[r]) < per]
        r = min(open_r, key=lambda q: (tot[q], q))
        ranks[r].append(int(e))
        tot[r] += load[e]
    return [sorted(r) for r in ranks]


def replicated_placement(load, world: int, n_hot: int) -> Tuple[List[List[int]], List[int]]:
    """Hot-expert replication: the n_hot most loaded experts are held by every rank (their
    routed pairs are split between the ranks by token: (t + e) % world), the others are dealt
    by balanced_placement.  Returns (per-rank expert lists, replicated experts); each rank's
    list holds its own experts followed by the replicated ones.  The rest (E - n_hot) must
    divide by the world size."""
    load = np.asarray(load, np.float64)
    E = load.shape[0]
    if n_hot <= 0:
        return balanced_placement(load, world), []
    hot = [int(e) for e in np.argsort(-load, kind="stable")[:n_hot]]
    rest = [e for e in range(E) if e not in set(hot)]
    if len(rest) % world != 0:
        raise ValueError(f"{len(rest)} experts outside the replicated set do not divide by {world} ranks")
    sub = balanced_placement(load[rest], world)
    ranks = [sorted(rest[i] for i in r) + sorted(hot) for r in sub]
    return ranks, sorted(hot)


def placement_imbalance(load, placement: List[List[int]], replicas: Optional[List[int]] = None) -> float:
    """max / mean of the per-rank load (1.0 = perfectly balanced); a replicated expert's load
    is split evenly over the ranks."""
    load = np.asarray(load, np.float64)
    rep = set(replicas or [])
    W = len(placement)
    per_rank = np.array([sum(load[e] / W if e in rep else load[e] for e in r) for r in placement])
    return float(per_rank.max() / max(per_rank.mean(), 1e-12))


def local_ids_map(ids: np.ndarray, experts: List[int]) -> np.ndarray:
    """Global ids -> local ids of a rank holding `experts` (in local order), -1 elsewhere."""
    m = np.full(max(experts) + 1, -1, np.int32)
    for l, e in enumerate(experts):
        m[e] = l
    ids = np.asarray(ids, np.int64)
    ok = (ids >= 0) & (ids < m.size)
    return np.where(ok, m[np.clip(ids, 0, m.size - 1)], -1).astype(np.int32)


def local_ids(ids: np.ndarray, lo: int, hi: int) -> np.ndarray:
    """Global ids -> this rank's local ids, -1 for experts held elsewhere (the kernel's remap)."""
    ids = np.asarray(ids, np.int32)
    return np.where((ids >= lo) & (ids < hi), ids - lo, -1).astype(np.int32)


def expert_owner(num_experts: int, world: int, placement: Optional[List[List[int]]] = None) -> np.ndarray:
    """[E] rank holding each global expert: the placement's lists, else contiguous blocks."""
    own = np.full(num_experts, -1, np.int64)
    if placement is None:
        for r, (lo, hi) in enumerate(expert_partition(num_experts, world)):
            own[lo:hi] = r
    else:
        for r, experts in enumerate(placement):
            for e in experts:
                if own[e] < 0:  # a replicated expert goes to its first holder
                    own[e] = r
    return own


def dispatch_plan(topk_ids, owner: np.ndarray, world: int) -> dict:
    """Rows each rank sends in the token all-to-all: for destination d, the rows (tokens) with
    at least one expert on d, in token order, and a [rows, K] mask of the pairs d computes
    (the other ids are sent as -1, which the kernels skip like invalid ids)."""
    ids = np.asarray(topk_ids.cpu() if hasattr(topk_ids, "cpu") else topk_ids, np.int64)
    E = owner.shape[0]
    ok = (ids >= 0) & (ids < E)
    dest = np.where(ok, owner[np.clip(ids, 0, E - 1)], -1)
    rows, masks = [], []
    for d in range(world):
        m = dest == d
        r = np.nonzero(m.any(axis=1))[0]
        rows.append(r)
        masks.append(m[r])
    return {"rows": rows, "masks": masks, "dest": dest}


def dispatch_forward(hidden, topk_ids, topk_w, owner: np.ndarray, world: int, compute, group=None):
    """Token all-to-all dispatch and combine over `group` (see ExpertParallelMoE.forward_dispatch):
    the rows of `dispatch_plan` go out in one all-to-all (hidden, ids with the other ranks' pairs
    set to -1, weights), `compute(rows, ids, w)` returns the received rows' fp32 partials, a
    second all-to-all brings them back and they are added per token in rank order."""
    import torch
    import torch.distributed as dist

    plan = dispatch_plan(topk_ids, owner, world)
    dev = hidden.device
    rows = [torch.as_tensor(r, dtype=torch.long, device=dev) for r in plan["rows"]]
    ids_t = torch.as_tensor(topk_ids, device=dev)
    w_t = torch.as_tensor(topk_w, device=dev)
    send_x = torch.cat([hidden[r] for r in rows])
    send_i = torch.cat([torch.where(torch.as_tensor(m, device=dev), ids_t[r], torch.full_like(ids_t[r], -1))
                        for r, m in zip(rows, plan["masks"])])
    send_w = torch.cat([w_t[r] for r in rows])
    scount = [len(r) for r in plan["rows"]]
    sc = torch.tensor(scount, dtype=torch.long, device=dev)
    rc = torch.empty_like(sc)
    dist.all_to_all_single(rc, sc, group=group)
    rcount = [int(v) for v in rc.tolist()]
    nrecv = sum(rcount)
    H = hidden.shape[1]
    recv_x = hidden.new_empty((nrecv, H))
    recv_i = send_i.new_empty((nrecv, send_i.shape[1]))
    recv_w = send_w.new_empty((nrecv, send_w.shape[1]))
    dist.all_to_all_single(recv_x, send_x.contiguous(), rcount, scount, group=group)
    dist.all_to_all_single(recv_i, send_i.contiguous(), rcount, scount, group=group)
    dist.all_to_all_single(recv_w, send_w.contiguous(), rcount, scount, group=group)
    part = compute(recv_x, recv_i, recv_w) if nrecv else torch.zeros((0, H), dtype=torch.float32, device=dev)
    back = part.new_empty((send_x.shape[0], H))
    dist.all_to_all_single(back, part.contiguous(), scount, rcount, group=group)
    y = torch.zeros((hidden.shape[0], H), dtype=torch.float32, device=dev)
    off = 0
    for r, n in zip(rows, scount):  # rank order: deterministic sums
        if n:
            y[r] += back[off:off + n]
        off += n
    return y.to(hidden.dtype)


class ExpertParallelMoE:
    """Fused MoE layer with experts sharded over a process group.

    `forward` returns the full [T, H] output on every rank.  Weight loaders take
    the full [E, ...] tensors (host or device); each rank keeps its block.
    """

    def __init__(self, num_experts: int, hidden: int, inter: int, quant_type: int, group=None,
                 group_size: int = 128, placement: Optional[List[List[int]]] = None,
                 replicas: Optional[List[int]] = None):
        import torch
        import torch.distributed as dist

        import moe_ascend_opt_b200  # noqa: F401  (registers torch.classes.nanovllm)

        self.group = group
        self.num_experts = num_experts
        self.placement = placement
        self.replicas = list(replicas or [])
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.lo, self.hi = expert_partition(num_experts, self.world)[self.rank]
        self.handle = torch.classes.nanovllm.MoEInfer(num_experts, hidden, inter, quant_type)
        if quant_type == 2:
            self.handle.set_group_size(group_size)
        self.handle.set_expert_parallel(self.rank, self.world)
        if placement is not None:  # e.g. balanced_placement(tokens per expert, world)
            if len(placement) != self.world:
                raise ValueError("placement needs one expert list per rank")
            self.handle.set_expert_placement(list(placement[self.rank]))
            if replicas:  # hot experts on every rank, e.g. from replicated_placement
                self.handle.set_expert_replicas(list(replicas))

    def load_quantized(self, gate_up_qs, gate_up_d, down_qs, down_d):
        self.handle.store_quantized_repack(gate_up_qs, gate_up_d, down_qs, down_d)

    def load_awq(self, *tensors):
        self.handle.store_awq(*tensors)

    def quantize_and_store_expert(self, e: int, proj: str, w):
        self.handle.quantize_and_store_expert(e, proj, w)

    def connect_peers(self, max_tokens: int = 8) -> None:
        """Set up the in-kernel combine over peer memory (NVLink): every rank creates its
        mailbox, the CUDA IPC handles are all-gathered over the process group, and each
        rank maps the others'.  Afterwards decode-size forwards sum the ranks' partials
        inside the fused kernel; larger ones still use the partial + all-reduce path."""
        import torch
        import torch.distributed as dist

        if self.world == 1:
            return
        h = self.handle.p2p_mailbox(self.world, max_tokens)
        dev = torch.device("cuda", torch.cuda.current_device())
        mine = h.to(dev)
        allh = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(allh, mine, group=self.group)
        self.handle.p2p_connect(torch.stack(allh).cpu())
        self.peers = True

    peers = False

    def expert_owner(self) -> np.ndarray:
        """[E] rank holding each global expert (from the placement, else the contiguous blocks)."""
        return expert_owner(self.num_experts, self.world, self.placement)

    def forward_dispatch(self, hidden, topk_ids, topk_w, compute=None):
        """Token all-to-all dispatch and combine: `hidden` [T_r, H], `topk_ids` / `topk_w`
        [T_r, K] are this rank's own tokens (global expert ids); returns this rank's [T_r, H]
        output.  `compute(rows, ids, w) -> fp32 [N, H]` runs the layer over this rank's experts
        (default: moe_forward_partial on this rank's engine)."""
        import torch

        if self.replicas:
            raise ValueError("forward_dispatch sends each pair to one rank; build the layer without replicas")
        if compute is None:
            compute = lambda x, i, w: torch.ops.nanovllm.moe_forward_partial(x, i, w, self.handle)  # noqa: E731
        return dispatch_forward(hidden, topk_ids, topk_w, self.expert_owner(), self.world, compute, self.group)

    def forward(self, hidden, topk_ids, topk_w, out: Optional[object] = None):
        import torch
        import torch.distributed as dist

        T = hidden.shape[0]
        if self.world == 1:
            y = torch.ops.nanovllm.moe_forward(hidden, topk_ids, topk_w, self.handle)
        elif self.peers and self.handle.p2p_covers(T):
            y = torch.ops.nanovllm.moe_forward(hidden, topk_ids, topk_w, self.handle)  # summed in the kernel
        else:
            if self.peers:
                self.handle.p2p_enable(False)
            try:
                part = torch.ops.nanovllm.moe_forward_partial(hidden, topk_ids, topk_w, self.handle)
            finally:
                if self.peers:
                    self.handle.p2p_enable(True)
            dist.all_reduce(part, group=self.group)
            y = part.to(hidden.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
