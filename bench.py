"""Benchmark of the fused MoE expert layer (one JSON line on stdout, rank 0).

Workload (N=1): BASELINE configs[1] -- Q4_0 fused MoE layer, H=2048, I=768,
E=128, top-8, T=1 token, weights fp32 N(0, 0.02^2) quantised to Q4_0 (fp16
block scales, 8 nibbles per uint32), bf16 N(0,1) activations, routing from
N(0,1) logits through the engine's softmax-top-8 router.  A step is one
fused-MoE layer forward.  The steps cycle over `--sets` independent weight
sets (layers) and per-step routings, so the bytes streamed between two uses
of a weight set exceed 2x the 126 MB L2 (inputs larger than L2).

metric: effective weight bandwidth = unique active experts x bytes/expert
        / time (test/benchmark_fused_moe_cpu.py:78-99,198 of the reference).

Arms:
  default            this engine (CUDA graphs of the torch.ops.nanovllm.moe_forward op)
  --impl reference   the reference CPU engine (oracle/_ref, built unmodified from the
                     reference sources) through its own torch.ops.nanovllm.moe_forward
Multi-GPU (torchrun): experts are partitioned across ranks (expert parallel);
each rank computes its experts' partial sum and one NCCL all-reduce combines.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, I, E, K = 2048, 768, 128, 8
Q4_BYTES_PER_EXPERT = (2 * I * H // 2) + (2 * I * (H // 32) * 2) + (H * I // 2) + (H * (I // 32) * 2)  # 2,654,208
Q8_BYTES_PER_EXPERT = (2 * I * H) + (2 * I * (H // 32) * 2) + (H * I) + (H * (I // 32) * 2)  # 5,013,504
METRIC = "fused MoE layer µs & effective weight GB/s vs HBM peak, tokens 1–4096, 1/2/4/8 GPU"
HBM_FALLBACK = 6650.0


def tflops_peaks():
    """Sustained dense bf16 TFLOP/s of this pool's B200s (MEASURED_PEAKS.json), else the fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops_sustained"])
    except Exception:
        return 1400.0


# DRAM bytes per layer step measured by ncu for the workloads that were captured (mean over 10
# launches each): (format, shape, tokens) -> tp_gate_up + tp_down read + write bytes (Q4_0
# 14,203,443 + 7,154,739; AWQ 13,817,651 + 6,936,243); algorithmic 21,233,664 and 19,611,648.
NCU_TRAFFIC = {("q4", "qwen", 1): 21358182, ("awq", "qwen", 1): 20753894}


def path_kernels(quant, T, K, E, peer_combine=False):
    """(kernel(s) of the layer's path, launches per layer step) under the engine's default
    dispatch: AWQ up to 32 tokens the two-pass kernels (in slices of 8 tokens), beyond that the
    tcgen05 grouped GEMMs; Q8_0 / Q4_0 up to 4 tokens the two-pass kernels, up to
    8 the split-K decode kernel, beyond that the grouped GEMMs (route, quantise, two GEMMs,
    combine)."""
    if peer_combine:
        return "moe_decode_kernel (peer combine)", 1
    if quant == "awq":
        if T <= 32:  # slices of 8 tokens
            return "tp_gate_up_kernel + tp_down_kernel", 2 * ((T + 7) // 8)
        return "grouped_gemm_tc_kernel", 7
    if T <= 4:
        return "tp_gate_up_q_kernel + tp_down_q_kernel", 2
    if T <= 8:
        return "moe_decode_sk_kernel", 1
    return ("grouped_gemm_wm_kernel" if T * K <= 24 * E else "grouped_gemm_kernel"), 7


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK, "fallback"


# ----------------------------------------------------------------- weights
def q4_quantize_torch(w):
    """fp32 [..., N, Kd] -> (int32 packed [..., N, Kd/8], fp16 [..., N, Kd/32]); d = amax/7, RNE, clamp [-8,7]."""
    import torch
    shp = w.shape
    b = w.reshape(*shp[:-1], shp[-1] // 32, 32)
    d32 = b.abs().amax(-1) / 7.0
    idv = torch.where(d32 != 0, 1.0 / d32, torch.zeros_like(d32))
    q = torch.clamp(torch.round(b * idv.unsqueeze(-1)), -8, 7).to(torch.int64) + 8
    q = q.reshape(*shp[:-1], shp[-1] // 8, 8)
    shifts = torch.arange(0, 32, 4, device=w.device, dtype=torch.int64)
    words = (q << shifts).sum(-1)
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)
    return words, d32.to(torch.float16)


def make_q4_layer(seed, device, e_lo=0, e_hi=E):
    """One layer's Q4_0 weights for experts [e_lo, e_hi) (full-E tensors, other experts zero)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    gu_qs = torch.zeros((E, 2 * I, H // 8), dtype=torch.int32, device=device)
    gu_d = torch.zeros((E, 2 * I, H // 32), dtype=torch.float16, device=device)
    dn_qs = torch.zeros((E, H, I // 8), dtype=torch.int32, device=device)
    dn_d = torch.zeros((E, H, I // 32), dtype=torch.float16, device=device)
    for e0 in range(0, E, 16):
        e1 = min(E, e0 + 16)
        wg = torch.randn((e1 - e0, 2 * I, H), generator=g, device=device) * 0.02
        wd = torch.randn((e1 - e0, H, I), generator=g, device=device) * 0.02
        if e1 <= e_lo or e0 >= e_hi:
            continue
        a, b = q4_quantize_torch(wg)
        gu_qs[e0:e1], gu_d[e0:e1] = a, b
        a, b = q4_quantize_torch(wd)
        dn_qs[e0:e1], dn_d[e0:e1] = a, b
        del wg, wd
    return gu_qs, gu_d, dn_qs, dn_d


SHAPES = {"qwen": (2048, 768, 128), "minimax": (3072, 1536, 256)}  # H, I, E (top-8 both)


def bytes_per_expert(quant, H_, I_, G=128):
    """Algorithmic weight bytes of one expert (gate_up + down, quants + scales (+ zeros))."""
    if quant == "q4":
        return (2 * I_ * H_ // 2) + (2 * I_ * (H_ // 32) * 2) + (H_ * I_ // 2) + (H_ * (I_ // 32) * 2)
    if quant == "q8":
        return (2 * I_ * H_) + (2 * I_ * (H_ // 32) * 2) + (H_ * I_) + (H_ * (I_ // 32) * 2)
    # AWQ: int4 weights, bf16 scales and int4 zeros per group of G along K
    return (2 * I_ * H_ // 2) + (2 * I_ * (H_ // G) * 2) + (2 * I_ * (H_ // G) // 2) + \
           (H_ * I_ // 2) + (H_ * (I_ // G) * 2) + (H_ * (I_ // G) // 2)


def q8_quantize_torch(w):
    """fp32 [..., N, Kd] -> (int8 [..., N, Kd], fp16 [..., N, Kd/32]): d = amax/127, RNE."""
    import torch
    shp = w.shape
    b = w.reshape(*shp[:-1], shp[-1] // 32, 32)
    d32 = b.abs().amax(-1) / 127.0
    idv = torch.where(d32 != 0, 1.0 / d32, torch.zeros_like(d32))
    q = torch.clamp(torch.round(b * idv.unsqueeze(-1)), -128, 127).to(torch.int8)
    return q.reshape(shp), d32.to(torch.float16)


def make_layer(quant, shape, seed, device, e_lo, e_hi, world, rank, placement=None):
    """A loaded MoEInfer handle with one synthetic layer (BASELINE configs value distributions)."""
    import torch
    H_, I_, E_ = SHAPES[shape]
    qt = {"q8": 0, "q4": 1, "awq": 2}[quant]
    h = torch.classes.nanovllm.MoEInfer(E_, H_, I_, qt)
    if quant == "awq":
        h.set_group_size(128)
    if world > 1:
        h.set_expert_parallel(rank, world)
        if placement is not None:
            h.set_expert_placement(placement[rank])
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    if quant == "awq":  # q, z uniform [0,15] (random words), bf16 scales U(0.001, 0.01)
        G = 128
        def words(*shp):
            return torch.randint(-2 ** 31, 2 ** 31 - 1, shp, generator=g, device=device, dtype=torch.int64).to(torch.int32)
        def scales(*shp):
            return (torch.rand(shp, generator=g, device=device) * 0.009 + 0.001).to(torch.bfloat16)
        h.store_awq(words(E_, H_, 2 * I_ // 8), scales(E_, H_ // G, 2 * I_), words(E_, H_ // G, 2 * I_ // 8),
                    words(E_, I_, H_ // 8), scales(E_, I_ // G, H_), words(E_, I_ // G, H_ // 8))
        return h
    qfn = q4_quantize_torch if quant == "q4" else q8_quantize_torch
    kq = 8 if quant == "q4" else 1
    qdt = torch.int32 if quant == "q4" else torch.int8
    gu_qs = torch.zeros((E_, 2 * I_, H_ // kq), dtype=qdt, device=device)
    gu_d = torch.zeros((E_, 2 * I_, H_ // 32), dtype=torch.float16, device=device)
    dn_qs = torch.zeros((E_, H_, I_ // kq), dtype=qdt, device=device)
    dn_d = torch.zeros((E_, H_, I_ // 32), dtype=torch.float16, device=device)
    step = 8
    for e0 in range(0, E_, step):
        e1 = min(E_, e0 + step)
        wg = torch.randn((e1 - e0, 2 * I_, H_), generator=g, device=device) * 0.02
        wd = torch.randn((e1 - e0, H_, I_), generator=g, device=device) * 0.02
        if e1 <= e_lo or e0 >= e_hi:
            continue
        gu_qs[e0:e1], gu_d[e0:e1] = qfn(wg)
        dn_qs[e0:e1], dn_d[e0:e1] = qfn(wd)
        del wg, wd
    h.store_quantized_repack(gu_qs, gu_d, dn_qs, dn_d)
    return h


def make_routing(kind, T, E_, K_, g, device):
    """softmax: top-K of N(0,1) logits with renormalised softmax weights (the engine's router);
    zipf: K distinct experts per token drawn with p(rank r) ~ r^-1.2 over a fixed random expert
    order, weights 1/K (BASELINE configs[2] run B)."""
    import torch
    if kind == "softmax":
        return torch.ops.nanovllm.moe_route(torch.randn((T, E_), generator=g, device=device), K_, True)
    perm = torch.randperm(E_, generator=g, device=device)
    p = (torch.arange(1, E_ + 1, device=device, dtype=torch.float32) ** -1.2)
    ranks = torch.multinomial(p.expand(T, E_), K_, replacement=False, generator=g)
    ids = perm[ranks].to(torch.int32).contiguous()
    w = torch.full((T, K_), 1.0 / K_, device=device, dtype=torch.float32)
    return ids, w


# ----------------------------------------------------------------- clocks
class ClockSampler:
    def __init__(self, out_path, gpu_index=0):
        self.path = out_path
        self.proc = None
        self.gpu = gpu_index

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        try:
            rows = [r.split(", ") for r in open(self.path).read().strip().splitlines() if r.strip()]
            sm = [float(r[1]) for r in rows]
            mx = float(rows[0][2])
            reasons = set()
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for r in rows:
                for n, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(n)
            loaded = [s for s in sm if s > 0.5 * mx] or sm
            return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                    "samples": len(sm)}
        except Exception as ex:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": str(ex)[:80]}


# ----------------------------------------------------------------- cpu baseline (reference)
def cpu_reference_worker(seconds: float, T: int):
    """Runs in a subprocess: the reference engine (oracle/_ref) at this workload on the host cores."""
    os.environ["NANOVLLM_TP_SIZE"] = "1"
    from oracle import oracle as O
    rng = np.random.default_rng(0)
    gq = rng.integers(0, 2 ** 32, size=(E, 2 * I, H // 8), dtype=np.uint32).view(np.int32)
    dq = rng.integers(0, 2 ** 32, size=(E, H, I // 8), dtype=np.uint32).view(np.int32)
    gd = O.f32_to_f16_bits((rng.random((E, 2 * I, H // 32), dtype=np.float32) * 0.004).astype(np.float32))
    dd = O.f32_to_f16_bits((rng.random((E, H, I // 32), dtype=np.float32) * 0.004).astype(np.float32))
    eng = O.RefEngine(E, H, I, 1)
    eng.store_repack(False, gq, gd, dq, dd)
    times, nbytes = [], []
    t_end = time.time() + seconds
    i = 0
    while time.time() < t_end or i < 3:
        xb = O.f32_to_bf16_bits(rng.standard_normal((T, H), dtype=np.float32))
        ids, w = O.topk_softmax(rng.standard_normal((T, E), dtype=np.float32), K, True)
        eng.forward(xb, ids, w)
        if i >= 2:
            times.append(eng.last_ms())
            nbytes.append(len(np.unique(ids)) * Q4_BYTES_PER_EXPERT)
        i += 1
    ms = statistics.mean(times)
    print(json.dumps({"ms": ms, "gbs": statistics.mean(nbytes) / (ms * 1e-3) / 1e9, "calls": len(times),
                      "cores": os.cpu_count()}))
    sys.stdout.flush()
    os._exit(0)


def cpu_baseline(T: int, seconds: float = 12.0):
    if not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "ref_bridge.so")):
        return None
    try:
        out = subprocess.run([sys.executable, os.path.abspath(__file__), "--cpu-worker", str(seconds), "--tokens", str(T)],
                             capture_output=True, text=True, timeout=seconds + 240,
                             env={**os.environ, "NANOVLLM_TP_SIZE": "1"})
        r = json.loads(out.stdout.strip().splitlines()[-1])
    except Exception as ex:
        return {"value": None, "unit": "GB/s", "cores": os.cpu_count(), "kind": "reference",
                "sample": f"failed: {str(ex)[:100]}"}
    return {"value": round(r["gbs"], 3), "unit": "GB/s", "cores": r["cores"], "kind": "reference",
            "ms_per_step": round(r["ms"], 4),
            "sample": f"{r['calls']} T={T} Q4_0 forwards of the reference engine (scalar-NEON-shim build, tp=1, "
                      f"NumaThreadPool on all {r['cores']} host threads), random routing, ~{seconds:.0f} s"}


# ----------------------------------------------------------------- reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    T = args.tokens
    os.environ["NANOVLLM_TP_SIZE"] = "1"
    os.environ.setdefault("NANOVLLM_TP_THREADS_PER_NODE", str(os.cpu_count()))
    so = os.path.join(ROOT, "oracle", "_ref", "nanovllm_ext_ref.so")
    if not os.path.exists(so):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/nanovllm_ext_ref.so not built "
                          "(needs the reference checkout; run oracle/Makefile ref)"}))
        return 0
    import ctypes
    import torch
    torch.ops.load_library(so)
    ctypes.CDLL(so).ref_pool_warmup()  # closes the reference pool's start-up race (oracle/ref_warmup.cpp)
    from oracle import oracle as O
    rng = np.random.default_rng(0)
    handles = []
    nsets = 2
    for s in range(nsets):
        h = torch.classes.nanovllm.MoEInfer(E, H, I, 1)
        gq = torch.from_numpy(rng.integers(0, 2 ** 32, size=(E, 2 * I, H // 8), dtype=np.uint32).view(np.int32))
        dq = torch.from_numpy(rng.integers(0, 2 ** 32, size=(E, H, I // 8), dtype=np.uint32).view(np.int32))
        gd = (torch.rand((E, 2 * I, H // 32)) * 0.004).to(torch.float16)
        dd = (torch.rand((E, H, I // 32)) * 0.004).to(torch.float16)
        h.store_quantized_repack(gq, gd, dq, dd)
        handles.append(h)
    steps = []
    for i in range(64):
        x = torch.randn(T, H).to(torch.bfloat16)
        ids, w = O.topk_softmax(rng.standard_normal((T, E), dtype=np.float32), K, True)
        steps.append((x, torch.from_numpy(ids), torch.from_numpy(w), len(np.unique(ids)) * Q4_BYTES_PER_EXPERT))
    for i in range(args.warmup):
        x, ids, w, _ = steps[i % len(steps)]
        torch.ops.nanovllm.moe_forward(x, ids, w, handles[i % nsets])
    t0 = time.perf_counter()
    tot_b = 0
    for i in range(args.steps):
        x, ids, w, nb = steps[i % len(steps)]
        torch.ops.nanovllm.moe_forward(x, ids, w, handles[i % nsets])
        tot_b += nb
    dt = time.perf_counter() - t0
    ms = dt / args.steps * 1e3
    val = tot_b / dt / 1e9
    line = {"metric": METRIC, "value": round(val, 3), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"Q4_0 fused MoE layer H{H} I{I} E{E} top{K} T={T} (BASELINE configs[1])",
                       "tokens": T},
            "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": os.cpu_count(), "kind": "reference",
                             "sample": f"{args.steps} T={T} forwards via torch.ops.nanovllm.moe_forward of the "
                                       f"reference built unmodified (scalar NEON shim, tp=1, {os.cpu_count()} threads)"},
            "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    sys.stdout.flush()
    os._exit(0)


# ----------------------------------------------------------------- our arm
def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    import moe_ascend_opt_b200  # noqa: F401

    T = args.tokens
    nsets = args.sets
    H, I, E = SHAPES[args.shape]
    bpe = bytes_per_expert(args.quant, H, I)
    el = E // world
    e_lo, e_hi = rank * el, (rank + 1) * el
    # per-step inputs: hidden + routing
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    nin = max(nsets, 16)
    xs, idss, wss, nbytes = [], [], [], []
    for i in range(nin):
        x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
        ids, w = make_routing(args.routing, T, E, K, g, dev)
        xs.append(x); idss.append(ids); wss.append(w)
        nbytes.append(int(torch.unique(ids).numel()) * bpe)
    placement = None
    if world > 1 and args.placement == "balanced":  # experts dealt to ranks by the routings' load
        from moe_ascend_opt_b200.ep import balanced_placement
        load = torch.bincount(torch.cat([i.flatten() for i in idss]).long(), minlength=E).cpu().numpy()
        placement = balanced_placement(load, world)

    imbalance = None
    if world > 1:  # max / mean over ranks of the active experts' bytes, averaged over the routings
        owner = np.zeros(E, np.int64)
        for r in range(world):
            owner[placement[r] if placement is not None else list(range(r * el, (r + 1) * el))] = r
        per_rank = np.zeros(world)
        for ids in idss:
            for e in torch.unique(ids).cpu().numpy():
                per_rank[owner[e]] += bpe
        imbalance = round(float(per_rank.max() / max(per_rank.mean(), 1e-9)), 3)

    handles = []
    for s in range(nsets):
        h = make_layer(args.quant, args.shape, 1000 + s, dev, e_lo, e_hi, world, rank, placement)
        h.reserve(max(T, 32), K)
        handles.append(h)
    torch.cuda.synchronize()
    combine_out = [torch.empty((T, H), dtype=torch.bfloat16, device=dev) for _ in range(nin)]

    # N>1, decode sizes: the partials are summed inside the fused kernel over NVLink peer
    # memory (every rank maps every other rank's mailbox); larger T: fp32 partial + NCCL.
    fused = world > 1 and not args.nccl_combine and not args.dispatch and handles[0].p2p_covers(T)
    if args.dispatch and world > 1:
        from moe_ascend_opt_b200.ep import dispatch_forward, expert_owner
        owner_d = expert_owner(E, world, placement)
        t_lo, t_hi = rank * T // world, (rank + 1) * T // world  # this rank's own tokens
    if fused:
        for h in handles:
            hnd = h.p2p_mailbox(world, max(T, 8)).to(dev)
            allh = [torch.empty_like(hnd) for _ in range(world)]
            dist.all_gather(allh, hnd)
            h.p2p_connect(torch.stack(allh).cpu())
        torch.cuda.synchronize()
        dist.barrier()

    def step(i):
        h = handles[i % nsets]
        j = i % nin
        if args.dispatch and world > 1:
            comp = lambda x, ii, ww: torch.ops.nanovllm.moe_forward_partial(x, ii, ww, h)  # noqa: E731
            return dispatch_forward(xs[j][t_lo:t_hi], idss[j][t_lo:t_hi], wss[j][t_lo:t_hi], owner_d, world, comp)
        if world == 1 or fused:
            return torch.ops.nanovllm.moe_forward(xs[j], idss[j], wss[j], h)
        part = torch.ops.nanovllm.moe_forward_partial(xs[j], idss[j], wss[j], h)
        dist.all_reduce(part)
        combine_out[j].copy_(part)
        return combine_out[j]

    # CUDA graphs (1 GPU): one graph holding a whole cycle of `ncycle` layer steps (a layer
    # stack, so the host launches once per cycle), plus one graph per step for remainders.
    graphs = None
    cycle_graph = None
    ncycle = int(np.lcm(nsets, nin))
    if (world == 1 or fused) and not args.no_graph:  # NCCL steps are not captured
        try:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for i in range(3):
                    step(i)
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            graphs = []
            for i in range(ncycle):
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr):
                    step(i)
                graphs.append(gr)
            cycle_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(cycle_graph):
                for i in range(ncycle):
                    step(i)
            torch.cuda.synchronize()
        except Exception as ex:  # eager launches are equally valid, just slower on the host
            print(f"[bench] graph capture unavailable ({str(ex)[:80]}); eager launches", file=sys.stderr)
            graphs = None
            cycle_graph = None

    def run(i):
        if graphs is not None:
            graphs[i % ncycle].replay()
        else:
            step(i)

    def run_steps(offset, nsteps):
        """Exactly `nsteps` layer steps starting at step `offset`."""
        i = offset
        end = offset + nsteps
        if cycle_graph is not None:
            while i < end and i % ncycle != 0:
                run(i); i += 1
            while end - i >= ncycle:
                cycle_graph.replay(); i += ncycle
        while i < end:
            run(i); i += 1

    for i in range(args.warmup):
        run(i)
    torch.cuda.synchronize()

    def timed(nsteps, offset=0):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        st = torch.cuda.current_stream()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(st)
        run_steps(offset, nsteps)
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    clk = ClockSampler(os.path.join(args.clock_dir or tempfile.gettempdir(), f"clocks_rank{rank}.csv"), local)
    with clk:
        # soak so the clock record covers a loaded GPU, then the timed region
        t_soak = time.time()
        while not args.no_soak and time.time() - t_soak < 1.0:
            timed(min(args.steps, 2000))
        total_ms = timed(args.steps)
    clocks = clk.summary()
    dev_errors = sorted({int(h.device_error()) for h in handles} - {0})

    avg_bytes = sum(nbytes[i % nin] for i in range(args.steps)) / args.steps
    qname = {"q4": "Q4_0", "q8": "Q8_0", "awq": "AWQ W4A16 g128"}[args.quant]
    default_wl = args.quant == "q4" and args.shape == "qwen" and args.routing == "softmax"
    ms_step = total_ms / args.steps
    value = avg_bytes / (ms_step * 1e-3) / 1e9
    peak, peak_kind = peaks()

    out = {"metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms_step, 6), "us_per_layer": round(ms_step * 1e3, 3),
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
           "dtype": "bf16" if args.quant == "awq" else "int8",
           "data": "synthetic",
           "config": {"workload": f"{qname} fused MoE layer H{H} I{I} E{E} top{K} T={T}"
                                  + (" (BASELINE configs[1])" if default_wl else f", {args.routing} routing"),
                      "tokens": T, "weight_sets": nsets,
                      "l2": f"inputs larger than L2: {nsets} rotating weight sets x {E} experts "
                            f"({nsets * E * bpe / 1e9:.1f} GB) and {nin} rotating routings",
                      "parallelism": f"ep{world}" if world > 1 else "single",
                      "placement": args.placement if world > 1 else "n/a",
                      "rank_load_imbalance": imbalance,
                      "combine": ("token all-to-all dispatch + combine (NCCL)" if args.dispatch else
                                  "in-kernel over NVLink peer memory" if fused else "fp32 partial + NCCL all-reduce")
                      if world > 1 else "in-kernel",
                      "launch": (f"cuda_graph ({ncycle} layer steps per graph replay)" if cycle_graph is not None
                                 else "eager"),
                      "avg_active_experts": round(avg_bytes / bpe, 2)},
           "gpu_launches": args.steps * path_kernels(args.quant, T, K, E, world > 1 and fused)[1],
           "clocks": clocks}
    if dev_errors:
        out["device_errors"] = dev_errors
    if True:
        out["roofline"] = {"bound": "hbm", "achieved": round(value, 2), "peak": peak, "unit": "GB/s",
                           "frac": round(value / peak, 4), "peak_source": peak_kind,
                           "traffic": NCU_TRAFFIC.get((args.quant, args.shape, T)) if world == 1 else None,
                           "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of both kernels, one "
                                              "capture of this workload (same command, --steps 50)")
                           if world == 1 and (args.quant, args.shape, T) in NCU_TRAFFIC else None,
                           "algorithmic_bytes_per_launch": round(avg_bytes),
                           "kernel": path_kernels(args.quant, T, K, E, world > 1 and fused)[0]}
    # end-to-end through the public op with host buffers and copies in the timed region
    if rank == 0 or world > 1:
        # one pinned host buffer per step holding hidden | topk_ids | topk_w (16-byte aligned
        # fields), one H2D copy into the matching device buffer, views as the op's inputs
        a16 = lambda n: (n + 15) // 16 * 16
        nbx, nbi = T * H * 2, T * K * 4
        off_i = a16(nbx)
        off_w = a16(off_i + nbi)
        tot = a16(off_w + nbi)
        hbuf = []
        for j in range(nin):
            b = torch.empty(tot, dtype=torch.uint8).pin_memory()
            b[:nbx].copy_(xs[j].cpu().contiguous().view(torch.uint8).flatten())
            b[off_i:off_i + nbi].copy_(idss[j].cpu().contiguous().view(torch.uint8).flatten())
            b[off_w:off_w + nbi].copy_(wss[j].cpu().contiguous().view(torch.uint8).flatten())
            hbuf.append(b)
        dbuf = torch.empty(tot, dtype=torch.uint8, device=dev)
        xd = dbuf[:nbx].view(torch.bfloat16).view(T, H)
        idd = dbuf[off_i:off_i + nbi].view(torch.int32).view(T, K)
        wd = dbuf[off_w:off_w + nbi].view(torch.float32).view(T, K)
        yh = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
        n_e2e = min(args.steps, 2000)

        def e2e_step(i):
            j = i % nin
            dbuf.copy_(hbuf[j], non_blocking=True)
            h = handles[i % nsets]
            if args.dispatch and world > 1:
                comp = lambda x, ii, ww: torch.ops.nanovllm.moe_forward_partial(x, ii, ww, h)  # noqa: E731
                y = dispatch_forward(xd[t_lo:t_hi], idd[t_lo:t_hi], wd[t_lo:t_hi], owner_d, world, comp)
                yh[t_lo:t_hi].copy_(y, non_blocking=True)
                return
            if world == 1 or fused:
                y = torch.ops.nanovllm.moe_forward(xd, idd, wd, h)
            else:
                y = torch.ops.nanovllm.moe_forward_partial(xd, idd, wd, h)
                dist.all_reduce(y)
                y = y.to(torch.bfloat16)
            yh.copy_(y, non_blocking=True)

        # graph mode, as a serving loop runs it: per step one CUDA graph holding the H2D copy
        # from that step's pinned buffer, the reference's graph-capture op
        # (moe_forward_npu_graph_out with a MoEGraphContext) and the D2H copy of the output
        # graph mode, as a serving loop runs it: one CUDA graph per cycle of steps; every step
        # copies its own pinned input buffer to the device, runs the reference's graph-capture
        # op (moe_forward_npu_graph_out with a MoEGraphContext) and copies its output back to
        # pinned host memory.  The copies run on a second stream (double-buffered device
        # inputs / outputs), so step i+1's input and step i's output cross the host link while
        # a layer computes.
        e2e_cycle = None
        if world == 1 and not args.no_graph:
            try:
                ctxs = [torch.classes.nanovllm.MoEGraphContext(h, T, K, 1) for h in handles]
                nstep_g = int(np.lcm(nsets, nin))
                dbufs = [torch.empty(tot, dtype=torch.uint8, device=dev) for _ in range(2)]
                views = [(b[:nbx].view(torch.bfloat16).view(T, H), b[off_i:off_i + nbi].view(torch.int32).view(T, K),
                          b[off_w:off_w + nbi].view(torch.float32).view(T, K)) for b in dbufs]
                ydevs = [torch.empty((T, H), dtype=torch.bfloat16, device=dev) for _ in range(2)]
                side = torch.cuda.Stream()

                def cycle():
                    main = torch.cuda.current_stream()
                    side.wait_stream(main)
                    ev_in = [torch.cuda.Event() for _ in range(nstep_g)]
                    ev_k = [torch.cuda.Event() for _ in range(nstep_g)]
                    ev_d = [torch.cuda.Event() for _ in range(nstep_g)]
                    dbufs[0].copy_(hbuf[0], non_blocking=True)
                    ev_in[0].record(main)
                    for i in range(nstep_g):
                        main.wait_event(ev_in[i])
                        if i >= 2:
                            main.wait_event(ev_d[i - 2])  # the output buffer has been copied out
                        xv, iv, wv = views[i % 2]
                        torch.ops.nanovllm.moe_forward_npu_graph_out(xv, iv, wv, handles[i % nsets], ctxs[i % nsets],
                                                                     ydevs[i % 2])
                        ev_k[i].record(main)
                        with torch.cuda.stream(side):
                            if i + 1 < nstep_g:
                                if i >= 1:
                                    side.wait_event(ev_k[i - 1])  # the input buffer has been read
                                dbufs[(i + 1) % 2].copy_(hbuf[(i + 1) % nin], non_blocking=True)
                                ev_in[i + 1].record(side)
                            side.wait_event(ev_k[i])
                            yh.copy_(ydevs[i % 2], non_blocking=True)
                            ev_d[i].record(side)
                    main.wait_stream(side)

                sg = torch.cuda.Stream()
                sg.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(sg):
                    cycle()
                torch.cuda.current_stream().wait_stream(sg)
                torch.cuda.synchronize()
                e2e_cycle = torch.cuda.CUDAGraph()
                with torch.cuda.graph(e2e_cycle):
                    cycle()
                torch.cuda.synchronize()
            except Exception as ex:
                print(f"[bench] e2e graph capture unavailable ({str(ex)[:80]})", file=sys.stderr)
                e2e_cycle = None

        def time_e2e(fn):
            for i in range(3):
                fn(i)
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(n_e2e):
                fn(i)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            if world > 1:
                t = torch.tensor([ms], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
            return ms

        def time_e2e_cycles(graph, n_cyc):
            for _ in range(2):
                graph.replay()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(n_cyc):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1)

        eb = sum(nbytes[i % nin] for i in range(n_e2e)) / n_e2e
        ems_eager = time_e2e(e2e_step)
        eager = {"value": round(eb / (ems_eager / n_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
                 "ms_per_step": round(ems_eager / n_e2e, 6), "steps": n_e2e,
                 "h2d_bytes_per_step": tot, "d2h_bytes_per_step": T * H * 2,
                 "api": "torch.ops.nanovllm.moe_forward (eager; one pinned H2D copy of hidden, "
                        "ids and weights, one D2H copy of the output)"}
        if e2e_cycle is not None:
            # whole cycles of the graph: at least one, and at least the main run's step count
            n_cyc = max(1, -(-n_e2e // nstep_g))
            n_g = n_cyc * nstep_g
            eb_g = sum(nbytes[i % nin] for i in range(n_g)) / n_g
            ems = time_e2e_cycles(e2e_cycle, n_cyc)
            out["e2e"] = {"value": round(eb_g / (ems / n_g * 1e-3) / 1e9, 2), "unit": "GB/s",
                          "ms_per_step": round(ems / n_g, 6), "steps": n_g,
                          "h2d_bytes_per_step": tot, "d2h_bytes_per_step": T * H * 2,
                          "api": f"torch.ops.nanovllm.moe_forward_npu_graph_out + MoEGraphContext in a CUDA graph "
                                 f"of {nstep_g} steps; per step one pinned H2D copy of hidden/ids/weights and one "
                                 f"D2H copy of the output, on a second stream overlapping the neighbouring layers"}
            out["e2e_eager"] = eager
        else:
            out["e2e"] = eager
    if world == 1 and not args.no_north_star and default_wl:
        # AWQ W4A16 g128, Qwen shape, batch 1, softmax and Zipf(1.2) routing
        out["north_star"] = {r: extra_block("awq", "qwen", r, 1, min(args.steps, 4000), dev, peak)
                             for r in ("softmax", "zipf")}
    if world == 1 and args.stack:
        out["stack"] = stack_block(args.stack, "awq", "zipf", dev, peak, tflops_peaks())
    if world == 1 and not args.no_cpu and default_wl:
        out["cpu_baseline"] = cpu_baseline(T)
        if "stack" in out and (out["cpu_baseline"] or {}).get("ms_per_step"):
            # reference CPU engine per layer (Q4_0 T=1, the nearest format it has) x layers: a proxy
            out["stack"]["cpu_proxy_decode_T1_ms_per_step"] = round(out["cpu_baseline"]["ms_per_step"] * args.stack, 3)
    if args.sweep and world == 1:
        out["sweep"] = sweep(handles, dev, args, H, I, E, bpe)
    if rank == 0:
        print(json.dumps(out))
        sys.stdout.flush()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def extra_block(quant, shape, routing, T, steps, dev, peak, nsets=16):
    """One more measured workload in the same JSON line: a `nsets`-layer stack of random-init
    layers in one CUDA graph, rotating routings, `steps` timed steps (CUDA events)."""
    import torch
    H_, I_, E_ = SHAPES[shape]
    bpe = bytes_per_expert(quant, H_, I_)
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    nin = 16
    xs, idss, wss, nb = [], [], [], []
    for i in range(nin):
        xs.append(torch.randn((T, H_), generator=g, device=dev).to(torch.bfloat16))
        ids, w = make_routing(routing, T, E_, K, g, dev)
        idss.append(ids); wss.append(w); nb.append(int(torch.unique(ids).numel()) * bpe)
    handles = [make_layer(quant, shape, 3000 + s, dev, 0, E_, 1, 0) for s in range(nsets)]
    for h in handles:
        h.reserve(max(T, 8), K)
    ncyc = int(np.lcm(nsets, nin))

    def step(i):
        return torch.ops.nanovllm.moe_forward(xs[i % nin], idss[i % nin], wss[i % nin], handles[i % nsets])

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(3):
            step(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for i in range(ncyc):
            step(i)
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    reps = max(1, steps // ncyc)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    n = reps * ncyc
    ms = e0.elapsed_time(e1) / n
    avg_b = sum(nb[i % nin] for i in range(n)) / n
    val = avg_b / (ms * 1e-3) / 1e9
    errs = sorted({int(h.device_error()) for h in handles} - {0})
    qname = {"q4": "Q4_0", "q8": "Q8_0", "awq": "AWQ W4A16 g128"}[quant]
    out = {"workload": f"{qname} fused MoE layer H{H_} I{I_} E{E_} top{K} T={T}, {routing} routing",
           "us_per_layer": round(ms * 1e3, 3), "value": round(val, 2), "unit": "GB/s", "steps": n,
           "avg_active_experts": round(avg_b / bpe, 2),
           "roofline": {"bound": "hbm", "achieved": round(val, 2), "peak": peak, "unit": "GB/s",
                        "frac": round(val / peak, 4), "algorithmic_bytes_per_launch": round(avg_b),
                        "traffic": NCU_TRAFFIC.get((quant, shape, T)),
                        "kernel": path_kernels(quant, T, K, E_)[0]},
           "launch": f"cuda_graph ({ncyc} layer steps per replay, {nsets} weight sets)"}
    if errs:
        out["device_errors"] = errs
    del handles
    torch.cuda.empty_cache()
    return out


def stack_block(nlayers, quant, routing, dev, peak, tflops_peak, decode_tokens=(1, 4, 8), prefill_tokens=4096,
                steps=20):
    """a stack of `nlayers` independent Qwen-shaped layers, one step = one
    forward through every layer (CUDA graph of the whole stack).  Decode steps at batch
    `decode_tokens`, one prefill-sized step; routing as given."""
    import torch
    H_, I_, E_ = SHAPES["qwen"]
    bpe = bytes_per_expert(quant, H_, I_)
    handles = [make_layer(quant, "qwen", 5000 + l, dev, 0, E_, 1, 0) for l in range(nlayers)]
    torch.cuda.synchronize()
    g = torch.Generator(device=dev)
    g.manual_seed(23)
    res = {"layers": nlayers, "quant": quant, "routing": routing}
    for T in list(decode_tokens) + [prefill_tokens]:
        for h in handles:
            h.reserve(T, K)
        xs, idss, wss, nb = [], [], [], []
        for l in range(nlayers):
            xs.append(torch.randn((T, H_), generator=g, device=dev).to(torch.bfloat16))
            ids, w = make_routing(routing, T, E_, K, g, dev)
            idss.append(ids); wss.append(w); nb.append(int(torch.unique(ids).numel()) * bpe)
        outs = [torch.empty((T, H_), dtype=torch.bfloat16, device=dev) for _ in range(nlayers)]
        ctxs = [torch.classes.nanovllm.MoEGraphContext(h, T, K, 1) for h in handles]

        def stack():
            for l in range(nlayers):
                torch.ops.nanovllm.moe_forward_npu_graph_out(xs[l], idss[l], wss[l], handles[l], ctxs[l], outs[l])

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            stack()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            stack()
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize()
        reps = steps if T <= 64 else max(3, steps // 4)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        byts = sum(nb)
        flops = 6.0 * T * K * H_ * I_ * nlayers
        key = f"decode_T{T}" if T in decode_tokens else f"prefill_T{T}"
        res[key] = {"ms_per_step": round(ms, 4), "us_per_layer": round(ms * 1e3 / nlayers, 3),
                    "weight_GBps": round(byts / (ms * 1e-3) / 1e9, 1),
                    "hbm_frac": round(byts / (ms * 1e-3) / 1e9 / peak, 4),
                    "TFLOPs": round(flops / (ms * 1e-3) / 1e12, 2),
                    "tensor_frac": round(flops / (ms * 1e-3) / 1e12 / tflops_peak, 4),
                    "active_weight_bytes": byts}
        errs = sorted({int(h.device_error()) for h in handles} - {0})
        if errs:
            res[key]["device_errors"] = errs
        del xs, idss, wss, outs, ctxs, gr
        torch.cuda.empty_cache()
    del handles
    torch.cuda.empty_cache()
    return res


def sweep(handles, dev, args, H, I, E, bpe):
    """Eager per-T timing (events) for the token sweep of BASELINE configs[1]."""
    import torch
    res = {}
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    for T in [int(v) for v in args.sweep_tokens.split(",")]:
        nrot = 16 if T <= 32 else 4
        xs, ids_l, w_l, nb = [], [], [], []
        for i in range(nrot):
            xs.append(torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16))
            ids, w = make_routing(args.routing, T, E, K, g, dev)
            ids_l.append(ids); w_l.append(w); nb.append(int(torch.unique(ids).numel()) * bpe)
        n = 200 if T <= 32 else (40 if T <= 1024 else 10)
        for h in handles:
            h.reserve(T, K)  # workspaces sized before timing (no allocation in the timed loop)
        for i in range(len(handles)):
            torch.ops.nanovllm.moe_forward(xs[i % nrot], ids_l[i % nrot], w_l[i % nrot], handles[i % len(handles)])
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(n):
            torch.ops.nanovllm.moe_forward(xs[i % nrot], ids_l[i % nrot], w_l[i % nrot], handles[i % len(handles)])
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / n
        b = sum(nb[i % nrot] for i in range(n)) / n
        res[f"T{T}"] = {"us": round(ms * 1e3, 2), "GB/s": round(b / (ms * 1e-3) / 1e9, 1),
                        "TFLOP/s": round(6.0 * T * K * H * I / (ms * 1e-3) / 1e12, 2),
                        "active_experts": round(b / bpe, 1)}
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--sets", type=int, default=16)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-north-star", action="store_true", help="skip the AWQ W4A16 T=1 blocks")
    ap.add_argument("--stack", type=int, default=0,
                    help="add a block for an N-layer AWQ stack (BASELINE configs[4]: decode 1/4/8, prefill 4096)")
    ap.add_argument("--sweep", action="store_true")
    ap.add_argument("--quant", default="q4", choices=["q4", "q8", "awq"])
    ap.add_argument("--shape", default="qwen", choices=["qwen", "minimax"])
    ap.add_argument("--routing", default="softmax", choices=["softmax", "zipf"])
    ap.add_argument("--sweep-tokens", default="1,4,8,32,128,1024,4096")
    ap.add_argument("--no-soak", action="store_true", help="skip the 1 s clock soak (profiling runs)")
    ap.add_argument("--nccl-combine", action="store_true", help="N>1: fp32 partial + NCCL all-reduce at every T")
    ap.add_argument("--dispatch", action="store_true",
                    help="N>1: token-sharded ranks (T/N tokens each), token all-to-all dispatch and combine (NCCL)")
    ap.add_argument("--placement", default="contiguous", choices=["contiguous", "balanced"],
                    help="N>1: experts per rank in contiguous blocks or dealt by routing load")
    ap.add_argument("--cpu-worker", type=float, default=None)
    ap.add_argument("--clock-dir", default=None, help="directory for the nvidia-smi clock samples (default: temp dir)")
    args = ap.parse_args()
    if args.cpu_worker is not None:
        return cpu_reference_worker(args.cpu_worker, args.tokens)
    if args.impl == "reference":
        args.steps = min(args.steps, 5000)  # each reference step is a ms-scale CPU forward
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
