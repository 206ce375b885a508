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
