// Fused MoE decode layer without a grid barrier (Q8_0 / Q4_0): split-K down projection.
//
// Same arithmetic as moe_decode_kernel (Int8-gemm/q8_gemm.cpp:426-650): per 32-block
// integer dots folded as (f32(isum) * d_w) * d_a, SiLU(gate) * up, h requantised per
// 32-block (pack_A_q8_0), routing-weighted sum over the top-k experts.  What changes is
// who computes the down projection:
//
//   phase 0  every CTA routes (counting sort in shared memory) and quantises the tokens;
//   phase 1  CTA c owns the 32-blocks [bb, be) of the (unique expert x I) unit space:
//            it computes those gate/up rows for the expert's tokens, keeps h in shared
//            memory and requantises its own 32-blocks (no other CTA needs them);
//   phase 2  the same CTA multiplies its h blocks by the matching 32-column chunk of the
//            down weights for ALL H output rows (a split-K slice of down), accumulating
//            w_k * partial into a per-CTA fp32 tile [T][H] in shared memory;
//   reduce   every CTA stores its tile to part[cta]; after the one grid barrier of the
//            launch, CTA c sums rows [H*c/G, H*(c+1)/G) of the partials of all CTAs in
//            CTA order (deterministic) and writes the output rows.
//
// h never leaves the SM, no CTA requantises another CTA's h, and the down-weight bytes
// stream concurrently with the gate_up bytes from the start.  The fp32 sum over experts
// and 32-blocks is formed in a different (fixed) order than the sequential loop of the
// reference, so the result matches it to fp32 rounding, not bit for bit, and is the
// same on every run.
//
// Down-weight layout for this kernel (built at load time from the row records):
//   dk [E][I/32 chunks][H/32 slices] slice = 32 rows x BB weight bytes | 32 x 2-byte scales
// so one CTA's chunk for a run of 32-row slices is one contiguous bulk copy.
#pragma once
#include "moe_decode.cuh"

namespace moe {

// Shared-memory layout of the split-K kernel (byte offsets), decided on the host.
struct SkLayout {
    int32_t off_tw;  // float [T*K] routing weights by pair, int [E+1] chunk-cost prefix,
                     // then per position: int token [T*K], float routing weight [T*K]
    int32_t off_a;   // union: quantised tokens (phase 1) | fp32 output tile [T][H] (phase 2)
    int32_t off_h;   // h slots x 128 B, one per (owned chunk, token): fp32 h, then q (32 B) | d | sum
    int32_t hslots;  // h slots per CTA (upper bound of sum over owned chunks of the token count)
    int32_t spw;     // 32-row slices of down handled per warp
};

template <bool Q4>
MOE_DEV void issue_sk_down(const DecodeParams& p, const RouteSmem& rt, int bb, int cl, int s0, int ns, int nb2,
                           int nsl, int sb, uint8_t* slot, uint64_t* bar, uint64_t pol) {
    const int gb = bb + cl, u = gb / nb2, jb = gb - u * nb2;
    const uint8_t* src = p.dk + (((size_t)rt.ue[u] * nb2 + jb) * nsl + s0) * (size_t)sb;
    issue_copy(slot, src, (uint32_t)(ns * sb), bar, pol);
}

// Cost-balanced ownership: a 32-block (chunk) of unique expert u costs A + cnt_u (A: the
// streaming share, cnt_u: one unit per token of compute); cpre[u] is the cost of all
// chunks before expert u.  Chunk b goes to CTA floor((cost before b + half its cost) *
// G / total), which is monotone in b, so every CTA owns one contiguous chunk range.
MOE_DEV int sk_assign(int b, const int32_t* cpre, const int32_t* ucnt, int nb2, int A, float scale, int G) {
    const int u = b / nb2;
    const int cu = A + ucnt[u];
    const int pb = cpre[u] + (b - u * nb2) * cu;
    return min(G - 1, (int)((float)(2 * pb + cu) * scale));  // monotone in b, same on every CTA
}

// (position, 32-block) pairs before chunk b = the h slot of chunk b's first token
// (P: all positions, for b = U*nb2).
MOE_DEV int sk_slot0(int b, const RouteSmem& rt, int U, int nb2, int P) {
    const int u = b / nb2;
    if (u >= U) return nb2 * P;
    return nb2 * rt.ups[u] + (b - u * nb2) * rt.ucnt[u];
}

// First chunk owned by CTA c or a later one (NB = U*nb2 when none), found by the whole
// warp: each round tests 32 evenly spaced chunks of the remaining interval.
MOE_DEV int sk_first_chunk(int c, const int32_t* cpre, const int32_t* ucnt, int U, int nb2, int A, int G,
                           int lane) {
    int lo = 0, hi = U * nb2;  // the answer lies in [lo, hi]
    if (c >= G) return hi;
    const float scale = (float)G / (2.0f * (float)cpre[U]);
    while (lo < hi) {
        const int step = (hi - lo + 30) / 31;  // 31 * step >= hi - lo: lane 31 tests b >= hi
        const int b = lo + lane * step;
        const bool ge = b >= hi || sk_assign(b, cpre, ucnt, nb2, A, scale, G) >= c;
        const int f = __ffs(__ballot_sync(0xffffffffu, ge)) - 1;
        if (f == 0) {
            hi = lo;
        } else {
            const int nlo = lo + (f - 1) * step + 1;
            hi = min(hi, lo + f * step);
            lo = nlo;
        }
    }
    return lo;
}

template <int FMT>
__global__ void __launch_bounds__(kThreads, 1) moe_decode_sk_kernel(const DecodeParams p, const SkLayout L) {
    constexpr bool Q4 = FMT == kQ4;
    constexpr int BB = Q4 ? 16 : 32;  // weight bytes per 32-block
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int T = p.T, K = p.K, TK = T * K, E = p.E, H = p.H, I = p.I;
    const int nb1 = H >> 5, nb2 = I >> 5, nsl = H >> 5;
    const int SB = 32 * BB + 64;  // bytes of one 32-row slice of a down chunk
    unsigned long long* dbg = p.dbg ? p.dbg + (size_t)cta * kStamps : nullptr;
    if (dbg && tid == 0) { dbg[0] = global_ns(); dbg[13] = clock64(); }

    RouteSmem rt = carve_route(reinterpret_cast<int32_t*>(smem), TK, E);
    float* tws = reinterpret_cast<float*>(smem + L.off_tw);
    int32_t* cpre = reinterpret_cast<int32_t*>(tws + TK);  // [E+1]
    int32_t* ptok = cpre + E + 1;                          // [TK] token of each position
    float* pw = reinterpret_cast<float*>(ptok + TK);       // [TK] routing weight of each position
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_ring - 8 * kWarps * p.slots);
    uint64_t* mybar = bars + warp * p.slots;
    uint8_t* myring = smem + p.off_ring + (size_t)warp * p.slots * p.slot_bytes;
    int8_t* xq = reinterpret_cast<int8_t*>(smem + L.off_a);
    float* xd = reinterpret_cast<float*>(xq + (size_t)T * H);  // T*H is a multiple of 32
    int32_t* xs = reinterpret_cast<int32_t*>(xd + (size_t)T * nb1);
    float* hsl = reinterpret_cast<float*>(smem + L.off_h);  // [slot][32]
    float* otile = reinterpret_cast<float*>(smem + L.off_a);  // [T][H], after phase 1
    __shared__ int s_ok, s_bb, s_be;
    __shared__ unsigned long long s_launch;

    // ---------------- phase 0 ----------------
    if (lane == 0)
        for (int s = 0; s < p.slots; ++s) mbar_init(&mybar[s], 1);
    if (warp == kWarps - 1) {
        // this launch's barrier target: the load is in flight while the warp routes
        const unsigned long long launch_idx = barrier_launch_index(p.bar, (uint32_t)G);
        route_warp(p.ids, TK, p.K, E, p.e_off, p.emap, p.emap_n, rt, lane);
        const int U = *rt.nuniq;
        int carry = 0;  // exclusive prefix of the chunk costs over the unique experts
        for (int u0 = 0; u0 < U; u0 += 32) {
            const int u = u0 + lane;
            const int c = u < U ? nb2 * (p.sk_cost_a + rt.ucnt[u]) : 0;
            int incl = c;
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            if (u < U) cpre[u] = carry + incl - c;
            carry += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) cpre[U] = carry;
        __syncwarp();
        const int f0 = sk_first_chunk(cta, cpre, rt.ucnt, U, nb2, p.sk_cost_a, G, lane);
        const int f1 = sk_first_chunk(cta + 1, cpre, rt.ucnt, U, nb2, p.sk_cost_a, G, lane);
        if (lane == 0) {
            s_bb = f0;
            s_be = f1;
            s_ok = 1;
            s_launch = launch_idx;
            if (dbg) dbg[1] = global_ns();
        }
    } else {
        for (int i = tid; i < TK; i += kThreads - 32) tws[i] = p.tw[i];
        quant_x_smem<Q4>(static_cast<const uint8_t*>(p.x), p.act_bf16, T, H, xq, xd, xs, tid, kThreads - 32);
        if (dbg && tid == 0) dbg[2] = global_ns();
    }
    fence_barrier_init();
    __syncthreads();
    if (dbg && tid == 0) dbg[3] = global_ns();

    const int bb = s_bb, be = s_be;  // this CTA's chunks (32-blocks of the unique-expert x I units)
    const int nc = be - bb;
    const int U = *rt.nuniq, P = rt.start[E];
    const int slot_b = sk_slot0(bb, rt, U, nb2, P);  // h slots of this CTA: [slot_b, slot_e)
    const int nslots = sk_slot0(be, rt, U, nb2, P) - slot_b;
    if (dbg && tid == 0) dbg[15] = ((unsigned long long)nslots << 32) | (unsigned)nc;
    const int64_t cb = (int64_t)bb * 32, ce = (int64_t)be * 32;
    P1Cursor c_issue{cb + (ce - cb) * warp / kWarps, cb + (ce - cb) * (warp + 1) / kWarps, I, p.units_per_item};
    P1Cursor c_use = c_issue;
    const int s0w = min(nsl, warp * L.spw), nsw = min(nsl, s0w + L.spw) - s0w;
    const int n2 = nsw > 0 ? nc : 0;  // down items of this warp: one per owned chunk
    int issued2 = 0, nissued = 0;
    const uint64_t pol = (p.flags & kFlagEvictFirst) ? l2_evict_first_policy() : 0ull;

    auto top_up = [&](int consumed) {
        __syncwarp();  // every lane's reads of the consumed slots are complete before reuse
        if (lane == 0) {
            while (nissued - consumed < p.slots) {
                const int s = nissued % p.slots;
                uint8_t* dst = myring + (size_t)s * p.slot_bytes;
                int u, j0, n;
                if (c_issue.next(u, j0, n)) {
                    issue_p1(p, rt, u, j0, n, dst, &mybar[s], pol);
                } else if (issued2 < n2) {
                    issue_sk_down<Q4>(p, rt, bb, issued2, s0w, nsw, nb2, nsl, SB, dst, &mybar[s], pol);
                    ++issued2;
                } else {
                    break;
                }
                ++nissued;
            }
        }
        c_issue.cur = __shfl_sync(0xffffffffu, c_issue.cur, 0);
        issued2 = __shfl_sync(0xffffffffu, issued2, 0);
        nissued = __shfl_sync(0xffffffffu, nissued, 0);
    };
    top_up(0);

    const bool sbf = p.scale_bf16 != 0;
    bool ok = true;
    int item = 0;

    // ---------------- phase 1: gate_up + SiLU*up into the CTA's h slots ----------------
    {
        const int LPU = 32 / p.units_per_item;
        const int usub = lane % LPU, uslot = lane / LPU;
        int u, j0, n;
        while (c_use.next(u, j0, n)) {
            const int s = item % p.slots;
            if (!mbar_wait(&mybar[s], (uint32_t)(item / p.slots) & 1u)) { set_err(p.err, kErrFullWait); ok = false; break; }
            if (dbg && tid == 0 && item == 0) dbg[4] = global_ns();
            const bool valid = uslot < n;
            const uint8_t* rec = myring + (size_t)s * p.slot_bytes + (size_t)(valid ? uslot : 0) * 2 * (p.rs1 + p.ss1);
            const uint8_t* qg = rec;
            const uint8_t* qu = rec + p.rs1;
            const uint16_t* sgate = reinterpret_cast<const uint16_t*>(rec + 2 * p.rs1);
            const uint16_t* sup = reinterpret_cast<const uint16_t*>(rec + 2 * p.rs1 + p.ss1);
            const int j = j0 + uslot;
            const int ps = rt.ups[u], cnt = rt.ucnt[u];
            float* hrow = hsl + (size_t)(sk_slot0(u * nb2 + (j >> 5), rt, U, nb2, P) - slot_b) * 32 + (j & 31);
            for (int m0 = 0; m0 < cnt; m0 += kTokTile) {
                const int nt = min(kTokTile, cnt - m0);
                int tk[kTokTile];
                float ag[kTokTile], au[kTokTile];
#pragma unroll
                for (int m = 0; m < kTokTile; ++m) {
                    tk[m] = m < nt ? rt.tok[ps + m0 + m] / K : 0;
                    ag[m] = 0.f;
                    au[m] = 0.f;
                }
                if (valid) {
#pragma unroll 4
                    for (int b = usub; b < nb1; b += LPU) {
                        const uint4* wg = reinterpret_cast<const uint4*>(qg + (size_t)b * BB);
                        const uint4* wu = reinterpret_cast<const uint4*>(qu + (size_t)b * BB);
                        const float dg = scale_to_f32(sgate[b], sbf), du = scale_to_f32(sup[b], sbf);
#pragma unroll
                        for (int m = 0; m < kTokTile; ++m) {
                            if (m >= nt) break;
                            const int t = tk[m];
                            const uint4* a = reinterpret_cast<const uint4*>(xq + (size_t)t * H + b * 32);
                            const float ad = xd[t * nb1 + b];
                            const int as = Q4 ? xs[t * nb1 + b] : 0;
                            ag[m] += ((float)block_dot<Q4>(wg, a, as) * dg) * ad;
                            au[m] += ((float)block_dot<Q4>(wu, a, as) * du) * ad;
                        }
                    }
                }
#pragma unroll
                for (int m = 0; m < kTokTile; ++m) {
                    if (m >= nt) break;
                    for (int o = LPU >> 1; o > 0; o >>= 1) {
                        ag[m] += __shfl_xor_sync(0xffffffffu, ag[m], o);
                        au[m] += __shfl_xor_sync(0xffffffffu, au[m], o);
                    }
                }
                if (valid && usub < nt) {
                    float g = ag[0], uu = au[0];
#pragma unroll
                    for (int m = 1; m < kTokTile; ++m)
                        if (usub == m) { g = ag[m]; uu = au[m]; }
                    hrow[(size_t)(m0 + usub) * 32] = silu_mul(g, uu);
                }
            }
            ++item;
            top_up(item);
        }
    }
    if (dbg && tid == 0) dbg[6] = global_ns();
    __syncthreads();

    // requantise the CTA's own h blocks in place (a quad of lanes per block and token),
    // and clear the output tile (the quantised tokens are no longer read)
    {
        const int sub = tid & 3;
        const uint32_t qm = quad_mask(lane);
        for (int t = tid >> 2; t < nslots; t += kThreads / 4) {
            float* slot = hsl + (size_t)t * 32;
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = slot[sub * 8 + e];
            float dd;
            int sum;
            uint2 o;
            quad_quant<Q4>(v, qm, dd, sum, o);  // every lane's loads precede the shuffles, hence the stores
            uint8_t* sbp = reinterpret_cast<uint8_t*>(slot);
            *reinterpret_cast<uint2*>(sbp + sub * 8) = o;
            if (sub == 0) *reinterpret_cast<float2*>(sbp + 32) = make_float2(dd, __int_as_float(sum));
        }
        float4* o4 = reinterpret_cast<float4*>(otile);
        for (int i = tid; i < T * H / 4; i += kThreads) o4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int pos = tid; pos < P; pos += kThreads) {
            const int pair = rt.tok[pos];
            ptok[pos] = pair / K;
            pw[pos] = tws[pair];
        }
    }
    __syncthreads();
    if (dbg && tid == 0) dbg[7] = global_ns();

    // ---------------- phase 2: split-K down for all H rows ----------------
    for (int k2 = 0; ok && k2 < n2; ++k2) {
        const int s = item % p.slots;
        if (!mbar_wait(&mybar[s], (uint32_t)(item / p.slots) & 1u)) { set_err(p.err, kErrFullWait); ok = false; break; }
        if (dbg && tid == 0 && k2 == 0) dbg[10] = global_ns();
        const uint8_t* st = myring + (size_t)s * p.slot_bytes;
        const int u = (bb + k2) / nb2;
        const int ps = rt.ups[u], cnt = rt.ucnt[u];
        const uint8_t* hq = reinterpret_cast<const uint8_t*>(hsl + (size_t)(sk_slot0(bb + k2, rt, U, nb2, P) - slot_b) * 32);
        for (int m = 0; m < cnt; ++m) {
            const uint8_t* hb = hq + (size_t)m * 128;
            const uint4* a = reinterpret_cast<const uint4*>(hb);
            const float2 ds = *reinterpret_cast<const float2*>(hb + 32);
            const int as = Q4 ? __float_as_int(ds.y) : 0;
            const float wk = pw[ps + m];
            float* orow = otile + (size_t)ptok[ps + m] * H + s0w * 32 + lane;
#pragma unroll 4
            for (int i = 0; i < nsw; ++i) {
                const uint8_t* sl = st + (size_t)i * SB;
                const uint4* w = reinterpret_cast<const uint4*>(sl + lane * BB);
                const float dw = scale_to_f32(reinterpret_cast<const uint16_t*>(sl + 32 * BB)[lane], sbf);
                const int is = block_dot<Q4>(w, a, as);
                orow[i * 32] += wk * (((float)is * dw) * ds.x);
            }
        }
        ++item;
        top_up(item);
    }
    if (!ok && lane == 0)  // a warp that stopped early still waits (bounded) for its copies in flight
        for (int i = item; i < nissued; ++i) mbar_wait(&mybar[i % p.slots], (uint32_t)(i / p.slots) & 1u);
    __syncthreads();
    if (dbg && tid == 0) dbg[11] = global_ns();

    // ---------------- partial tile -> global, grid barrier ----------------
    if (ok) {  // every CTA stores its tile (zero when it owns no chunk)
        const float4* o4 = reinterpret_cast<const float4*>(otile);
        float4* d4 = reinterpret_cast<float4*>(p.part + (size_t)cta * T * H);
        for (int i = tid; i < T * H / 4; i += kThreads) __stcg(d4 + i, o4[i]);
    }
    __syncthreads();
    if (tid == 1) {
        if (!grid_barrier(p.bar, (uint32_t)G, (s_launch + 1ull) * (uint32_t)G, p.err)) s_ok = 0;
    }
    __syncthreads();
    if (dbg && tid == 0) dbg[8] = global_ns();
    if (!s_ok) return;

    // ---------------- rows [n0, n0+R): sum the partials of all CTAs in a fixed order ----------------
    // ks threads per output: thread g adds CTAs g, g+ks, g+2ks, ... (loads in flight in
    // batches), then the ks sums are added in g order, so the result does not depend on timing.
    const int n0 = (int)((int64_t)H * cta / G), R = (int)((int64_t)H * (cta + 1) / G) - n0;
    const int O = T * R;
    if (O == 0) return;
    const int ks = max(1, min(kThreads / O, G));
    float* gsum = otile;  // ks*O <= max(kThreads, O) floats: the region holds both (the tile is stored already)
    for (int idx = tid; idx < ks * O; idx += kThreads) {
        const int g = idx / O, o = idx - g * O;
        const int t = o / R, r = o - t * R;
        const float* src = p.part + (size_t)t * H + n0 + r;
        const size_t kstride = (size_t)T * H;
        float acc = 0.f;
        constexpr int kBatch = 8;
        for (int k0 = g; k0 < G; k0 += ks * kBatch) {
            float v[kBatch];
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                const int k = k0 + j * ks;
                v[j] = k < G ? __ldcg(src + (size_t)k * kstride) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < kBatch; ++j) acc += v[j];
        }
        gsum[idx] = acc;
    }
    __syncthreads();
    for (int o = tid; o < O; o += kThreads) {
        float acc = 0.f;
        for (int g = 0; g < ks; ++g) acc += gsum[g * O + o];
        const int t = o / R, r = o - t * R;
        if (p.pc.world > 1) pc_put(p, s_launch + 1, t, n0 + r, acc);
        else st_out(p, (size_t)t * H + n0 + r, acc);
    }
    if (p.pc.world > 1) pc_finish(p, s_launch + 1, cta, G, n0, R, tid);
    if (dbg && tid == 0) { dbg[9] = global_ns(); dbg[14] = clock64(); }
}

}  // namespace moe
