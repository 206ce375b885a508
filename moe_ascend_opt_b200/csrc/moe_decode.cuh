// Persistent fused MoE layer kernel for decode-size token counts (Q8_0 / Q4_0).
//
// One CTA per SM (cooperative launch).  Per launch:
//   phase 0  every CTA routes the T*K pairs itself (stable counting sort of
//            moe_common.cpp:146-184, in shared memory) and quantises the T
//            token rows to Q8_0 (gemm_kernels.cpp:25-58) into shared memory;
//   phase 1  gate_up: the U*I "units" (gate row j + up row j of an active
//            expert) are split into equal contiguous ranges, one per CTA; each
//            unit's two rows are dotted with the expert's token rows and
//            SiLU(gate)*up goes to the fp32 workspace h[pos][j];
//   barrier  one grid barrier (bounded spin);
//   phase 2  down: each CTA owns an equal range of the H output rows for ALL
//            active experts, requantises h (pack_A_q8_0, gemm_kernels.cpp:394-425),
//            computes out[pos][n] and finally the k-ordered combine
//            y[t][n] = sum_k w[t,k] out[pos(t,k)][n] (q8_gemm.cpp:593-613).
// A producer warp streams every weight chunk of the CTA (phase 1, then phase 2)
// with cp.async.bulk into a ring of shared-memory stages guarded by mbarriers,
// so the down-projection weights are already arriving while the CTAs wait at
// the grid barrier.  Weights cross HBM exactly once per launch.
#pragma once
#include "common.cuh"

namespace moe {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kDecodeThreads = kConsumerThreads + 32;
constexpr int kTokTile = 4;  // token rows held in registers per pass

struct DecodeParams {
    const uint8_t* gu_qs;  // [E][I][2][rs1]   gate row j, up row j
    const uint8_t* gu_sc;  // [E][I][2][ss1]   16-bit scale bits
    const uint8_t* dn_qs;  // [E][H][rs2]
    const uint8_t* dn_sc;  // [E][H][ss2]
    int32_t rs1, ss1, rs2, ss2;
    int32_t E, e_off, H, I, T, K;
    int32_t scale_bf16, act_bf16, out_kind;  // out_kind: 0 f16, 1 bf16, 2 f32
    const void* x;
    void* y;
    const int32_t* ids;
    const float* tw;
    float* h_ws;     // [T*K][I]
    uint32_t* bar;   // grid barrier {count, generation}
    int32_t* err;    // device error word
    // shared-memory carve-up (bytes)
    int32_t off_x, off_out, off_stage, stage_bytes, nstages;
    int32_t units_per_chunk;   // phase-1 units per stage
    int32_t rows_max;          // phase-2 rows per CTA (upper bound)
    int32_t experts_per_chunk; // phase-2 experts per stage
    int32_t lanes_per_row;     // phase-2 lanes per down row (power of two)
};

// Shared routing tables, placed at the start of dynamic shared memory.
struct RouteSmem {
    int32_t* ids;    // [TK] local expert id or -1
    int32_t* smap;   // [TK] position or -1
    int32_t* tok;    // [TK] token of each position
    int32_t* cnt;    // [E] count per expert (then reused)
    int32_t* start;  // [E+1]
    int32_t* ue;     // [E] unique active experts (ascending)
    int32_t* ups;    // [E] first position of each unique expert
    int32_t* ucnt;   // [E]
    int32_t* nuniq;  // [1]
};

MOE_DEV int route_smem_ints(int TK, int E) { return 3 * TK + 5 * E + 4; }

MOE_DEV RouteSmem carve_route(int32_t* base, int TK, int E) {
    RouteSmem r;
    r.ids = base;
    r.smap = r.ids + TK;
    r.tok = r.smap + TK;
    r.cnt = r.tok + TK;
    r.start = r.cnt + E;
    r.ue = r.start + E + 1;
    r.ups = r.ue + E;
    r.ucnt = r.ups + E;
    r.nuniq = r.ucnt + E;
    return r;
}

// Stable counting sort by one warp (moe_common.cpp:146-184): pairs are taken in
// (t,k) order 32 at a time; lanes with the same expert rank themselves with
// __match_any_sync, so positions inside an expert follow pair order exactly.
MOE_DEV void route_warp(const int32_t* g_ids, int TK, int E, int e_off, RouteSmem r, int lane) {
    for (int e = lane; e < E; e += 32) r.cnt[e] = 0;
    __syncwarp();
    for (int i0 = 0; i0 < TK; i0 += 32) {
        const int i = i0 + lane;
        int e = -1;
        if (i < TK) {
            const int g = g_ids[i] - e_off;
            e = (g >= 0 && g < E) ? g : -1;
            r.ids[i] = e;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        int base = 0;
        if (e >= 0) base = r.cnt[e];
        __syncwarp();
        if (i < TK) r.smap[i] = (e >= 0) ? base + rank : -1;  // rank within expert for now
        if (e >= 0 && rank == 0) r.cnt[e] = base + __popc(peers);
        __syncwarp();
    }
    // exclusive scan of counts -> start, and the unique-expert list
    int carry = 0, ucarry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
        const int e = e0 + lane;
        const int c = (e < E) ? r.cnt[e] : 0;
        int incl = c;
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        const unsigned act = __ballot_sync(0xffffffffu, c > 0);
        if (e < E) {
            r.start[e] = carry + incl - c;
            if (c > 0) {
                const int u = ucarry + __popc(act & ((1u << lane) - 1u));
                r.ue[u] = e;
                r.ups[u] = carry + incl - c;
                r.ucnt[u] = c;
            }
        }
        carry += __shfl_sync(0xffffffffu, incl, 31);
        ucarry += __popc(act);
    }
    if (lane == 0) {
        r.start[E] = carry;
        *r.nuniq = ucarry;
    }
    __syncwarp();
    for (int i = lane; i < TK; i += 32) {
        const int e = r.ids[i];
        if (e >= 0) {
            const int pos = r.start[e] + r.smap[i];
            r.smap[i] = pos;
            r.tok[pos] = i;  // pair index; token = i / K
        }
    }
    __syncwarp();
}

// Q4_0 activation byte order inside a 32-block: the weight word w holds
// elements 8w..8w+7 in nibbles 0..7, so its low nibbles are elements
// 8w+{0,2,4,6} and its high nibbles 8w+{1,3,5,7}.
MOE_DEV int q4_perm(int e) {
    const int w = e >> 3, r = e & 7;
    return (w << 3) + ((r & 1) << 2) + (r >> 1);
}

// Quantise `nrows` rows of `cols` values (fp32 in global via a loader) into
// shared memory, 8 lanes per 32-block, each lane 4 consecutive values.
template <bool Q4, typename Loader>
MOE_DEV void quant_rows_smem(Loader load4, int nrows, int cols, int8_t* q, float* d, int32_t* s,
                             int tid, int nthreads) {
    const int nb = cols >> 5;
    const int ngroups = nrows * nb;
    // every block needs all 8 lanes of its group: iterate in whole groups
    for (int base = (tid >> 3); base < ((ngroups + (nthreads >> 3) - 1) / (nthreads >> 3)) * (nthreads >> 3);
         base += (nthreads >> 3)) {
        const int sub = tid & 7;
        const bool valid = base < ngroups;
        const int row = valid ? base / nb : 0, b = valid ? base % nb : 0;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (valid) load4(row, b * 32 + sub * 4, v);
        float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        const float dd = q8_scale(amax);
        const float id = q8_inv(dd);
        int qsum = 0;
        int8_t* qb = q + (size_t)row * cols + b * 32;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int qq = q8_quant(v[j], id);
            qsum += qq;
            const int e = sub * 4 + j;
            if (valid) qb[Q4 ? q4_perm(e) : e] = (int8_t)qq;
        }
        qsum += __shfl_xor_sync(0xffffffffu, qsum, 4);
        qsum += __shfl_xor_sync(0xffffffffu, qsum, 2);
        qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
        if (valid && sub == 0) {
            d[row * nb + b] = dd;
            if (Q4) s[row * nb + b] = qsum;
        }
    }
}

// Exact int32 dot of one 32-block: weights (Q8: 32 bytes, Q4: 16 bytes of
// nibbles) against 32 int8 activations (Q4: permuted, bias 8 via asum).
template <bool Q4>
MOE_DEV int block_dot(const uint4* w, const uint4* a, int asum) {
    if (Q4) {
        const uint4 ww = w[0];
        const uint4 a0 = a[0], a1 = a[1];
        int s = 0;
        s = __dp4a((int)(ww.x & 0x0f0f0f0fu), (int)a0.x, s);
        s = __dp4a((int)((ww.x >> 4) & 0x0f0f0f0fu), (int)a0.y, s);
        s = __dp4a((int)(ww.y & 0x0f0f0f0fu), (int)a0.z, s);
        s = __dp4a((int)((ww.y >> 4) & 0x0f0f0f0fu), (int)a0.w, s);
        s = __dp4a((int)(ww.z & 0x0f0f0f0fu), (int)a1.x, s);
        s = __dp4a((int)((ww.z >> 4) & 0x0f0f0f0fu), (int)a1.y, s);
        s = __dp4a((int)(ww.w & 0x0f0f0f0fu), (int)a1.z, s);
        s = __dp4a((int)((ww.w >> 4) & 0x0f0f0f0fu), (int)a1.w, s);
        return s - 8 * asum;
    } else {
        const uint4 w0 = w[0], w1 = w[1];
        const uint4 a0 = a[0], a1 = a[1];
        int s = 0;
        s = __dp4a((int)w0.x, (int)a0.x, s);
        s = __dp4a((int)w0.y, (int)a0.y, s);
        s = __dp4a((int)w0.z, (int)a0.z, s);
        s = __dp4a((int)w0.w, (int)a0.w, s);
        s = __dp4a((int)w1.x, (int)a1.x, s);
        s = __dp4a((int)w1.y, (int)a1.y, s);
        s = __dp4a((int)w1.z, (int)a1.z, s);
        s = __dp4a((int)w1.w, (int)a1.w, s);
        return s;
    }
}

// Chunk enumeration shared by producer and consumers ------------------------
struct P1Chunk { int u, j0, n; };

struct P1Iter {
    int64_t cur, end;
    int I, per;
    MOE_DEV bool next(P1Chunk& c) {
        if (cur >= end) return false;
        c.u = (int)(cur / I);
        c.j0 = (int)(cur % I);
        int64_t n = end - cur;
        if (n > I - c.j0) n = I - c.j0;
        if (n > per) n = per;
        c.n = (int)n;
        cur += n;
        return true;
    }
};

template <bool Q4>
__global__ void __launch_bounds__(kDecodeThreads, 1) moe_decode_kernel(const DecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int TK = p.T * p.K, E = p.E, H = p.H, I = p.I;
    const int nb1 = H >> 5, nb2 = I >> 5;

    RouteSmem rt = carve_route(reinterpret_cast<int32_t*>(smem), TK, E);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_stage - 16 * p.nstages);
    uint64_t* empty = full + p.nstages;
    uint8_t* stages = smem + p.off_stage;
    __shared__ int s_ok;

    // ---------------- phase 0: routing + barrier init (all warps) --------------
    if (warp == 0) route_warp(p.ids, TK, E, p.e_off, rt, lane);
    if (tid == 32) {
        for (int s = 0; s < p.nstages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_barrier_init();
        s_ok = 1;
    }
    __syncthreads();
    const int U = *rt.nuniq;

    // phase-1 range of units and phase-2 range of rows owned by this CTA
    const int64_t TU = (int64_t)U * I;
    const int64_t u_begin = TU * cta / G, u_end = TU * (cta + 1) / G;
    const int n0 = (int)((int64_t)H * cta / G), n1 = (int)((int64_t)H * (cta + 1) / G);
    const int R = n1 - n0;
    const int nchunk2 = (R > 0 && U > 0) ? (U + p.experts_per_chunk - 1) / p.experts_per_chunk : 0;

    if (warp == kConsumerWarps) {
        // ---------------- producer ----------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            P1Iter it{u_begin, u_end, I, p.units_per_chunk};
            P1Chunk c;
            bool ok = true;
            while (ok && it.next(c)) {
                if (!mbar_wait(&empty[s], ph ^ 1)) { atomicExch(p.err, kErrEmptyWait); ok = false; break; }
                const int e = rt.ue[c.u];
                const uint32_t qb = (uint32_t)c.n * 2u * p.rs1, sb = (uint32_t)c.n * 2u * p.ss1;
                uint8_t* dst = stages + (size_t)s * p.stage_bytes;
                mbar_arrive_expect_tx(&full[s], qb + sb);
                bulk_g2s(dst, p.gu_qs + ((size_t)e * I + c.j0) * 2 * p.rs1, qb, &full[s]);
                bulk_g2s(dst + qb, p.gu_sc + ((size_t)e * I + c.j0) * 2 * p.ss1, sb, &full[s]);
                if (++s == p.nstages) { s = 0; ph ^= 1; }
            }
            for (int ch = 0; ok && ch < nchunk2; ++ch) {
                if (!mbar_wait(&empty[s], ph ^ 1)) { atomicExch(p.err, kErrEmptyWait); ok = false; break; }
                const int ua = ch * p.experts_per_chunk;
                const int ub = min(U, ua + p.experts_per_chunk);
                const uint32_t qrow = (uint32_t)R * p.rs2, srow = (uint32_t)R * p.ss2;
                uint8_t* dst = stages + (size_t)s * p.stage_bytes;
                const uint32_t qtot = (uint32_t)(ub - ua) * qrow;
                mbar_arrive_expect_tx(&full[s], (uint32_t)(ub - ua) * (qrow + srow));
                for (int u = ua; u < ub; ++u) {
                    const int e = rt.ue[u];
                    bulk_g2s(dst + (size_t)(u - ua) * qrow, p.dn_qs + ((size_t)e * H + n0) * p.rs2, qrow, &full[s]);
                    bulk_g2s(dst + qtot + (size_t)(u - ua) * srow, p.dn_sc + ((size_t)e * H + n0) * p.ss2, srow,
                             &full[s]);
                }
                if (++s == p.nstages) { s = 0; ph ^= 1; }
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    int8_t* xq = reinterpret_cast<int8_t*>(smem + p.off_x);
    float* xd = reinterpret_cast<float*>(xq + (size_t)p.T * H);
    int32_t* xs = reinterpret_cast<int32_t*>(xd + (size_t)p.T * nb1);
    {
        const void* x = p.x;
        const int bf = p.act_bf16;
        auto load4 = [&](int row, int col, float* v) {
            const int64_t base = (int64_t)row * H + col;
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = act_to_f32(x, base + j, bf);
        };
        quant_rows_smem<Q4>(load4, p.T, H, xq, xd, xs, tid, kConsumerThreads);
    }
    named_bar_sync(1, kConsumerThreads);

    const bool sbf = p.scale_bf16 != 0;
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;

    // ---------------- phase 1: gate_up + SiLU*up ----------------
    {
        P1Iter it{u_begin, u_end, I, p.units_per_chunk};
        P1Chunk c;
        while (it.next(c)) {
            if (!mbar_wait(&full[s], ph)) { atomicExch(p.err, kErrFullWait); ok = false; break; }
            const uint8_t* st = stages + (size_t)s * p.stage_bytes;
            const uint8_t* qbase = st;
            const uint16_t* sbase = reinterpret_cast<const uint16_t*>(st + (size_t)c.n * 2 * p.rs1);
            const int ps = rt.ups[c.u], cnt = rt.ucnt[c.u];
            for (int jj = warp; jj < c.n; jj += kConsumerWarps) {
                const uint8_t* qg = qbase + (size_t)jj * 2 * p.rs1;
                const uint8_t* qu = qg + p.rs1;
                const uint16_t* sgate = reinterpret_cast<const uint16_t*>(
                    reinterpret_cast<const uint8_t*>(sbase) + (size_t)jj * 2 * p.ss1);
                const uint16_t* sup = reinterpret_cast<const uint16_t*>(
                    reinterpret_cast<const uint8_t*>(sgate) + p.ss1);
                for (int m0 = 0; m0 < cnt; m0 += kTokTile) {
                    float ag[kTokTile], au[kTokTile];
                    int tk[kTokTile];
#pragma unroll
                    for (int m = 0; m < kTokTile; ++m) {
                        ag[m] = 0.f;
                        au[m] = 0.f;
                        tk[m] = (m0 + m < cnt) ? rt.tok[ps + m0 + m] / p.K : -1;
                    }
                    for (int b = lane; b < nb1; b += 32) {
                        const uint4* wg = reinterpret_cast<const uint4*>(qg + (size_t)b * (Q4 ? 16 : 32));
                        const uint4* wu = reinterpret_cast<const uint4*>(qu + (size_t)b * (Q4 ? 16 : 32));
                        const float dg = scale_to_f32(sgate[b], sbf), du = scale_to_f32(sup[b], sbf);
#pragma unroll
                        for (int m = 0; m < kTokTile; ++m) {
                            if (tk[m] < 0) continue;
                            const uint4* a = reinterpret_cast<const uint4*>(xq + (size_t)tk[m] * H + b * 32);
                            const float ad = xd[tk[m] * nb1 + b];
                            const int as = Q4 ? xs[tk[m] * nb1 + b] : 0;
                            const int ig = block_dot<Q4>(wg, a, as);
                            const int iu = block_dot<Q4>(wu, a, as);
                            ag[m] += ((float)ig * dg) * ad;
                            au[m] += ((float)iu * du) * ad;
                        }
                    }
#pragma unroll
                    for (int m = 0; m < kTokTile; ++m) {
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            ag[m] += __shfl_xor_sync(0xffffffffu, ag[m], o);
                            au[m] += __shfl_xor_sync(0xffffffffu, au[m], o);
                        }
                    }
                    if (lane < kTokTile && m0 + lane < cnt) {
                        float g = ag[0], u = au[0];
#pragma unroll
                        for (int m = 1; m < kTokTile; ++m)
                            if (lane == m) { g = ag[m]; u = au[m]; }
                        p.h_ws[(size_t)(ps + m0 + lane) * I + c.j0 + jj] = silu_mul(g, u);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == p.nstages) { s = 0; ph ^= 1; }
        }
    }

    // ---------------- grid barrier ----------------
    named_bar_sync(1, kConsumerThreads);
    if (tid == 0) {
        if (!ok || !grid_barrier(p.bar, (uint32_t)G, p.err)) s_ok = 0;
    }
    named_bar_sync(1, kConsumerThreads);
    ok = ok && s_ok;

    // ---------------- phase 2: requant h, down rows, combine ----------------
    const int P = rt.start[E];
    int8_t* hq = reinterpret_cast<int8_t*>(smem + p.off_x);
    float* hd = reinterpret_cast<float*>(hq + (size_t)P * I);
    int32_t* hs = reinterpret_cast<int32_t*>(hd + (size_t)P * nb2);
    float* outs = reinterpret_cast<float*>(smem + p.off_out);
    if (ok && nchunk2 > 0) {
        const float* h = p.h_ws;
        auto load4 = [&](int row, int col, float* v) {
            const float4 f = __ldcg(reinterpret_cast<const float4*>(h + (size_t)row * I + col));
            v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
        };
        quant_rows_smem<Q4>(load4, P, I, hq, hd, hs, tid, kConsumerThreads);
    }
    named_bar_sync(1, kConsumerThreads);

    const int LPR = p.lanes_per_row, RPG = 32 / LPR;
    const int sub = lane % LPR, rr = lane / LPR;
    const int ngrp = (R + RPG - 1) / RPG;
    for (int ch = 0; ch < nchunk2; ++ch) {
        if (!ok) break;
        if (!mbar_wait(&full[s], ph)) { atomicExch(p.err, kErrFullWait); ok = false; break; }
        const uint8_t* st = stages + (size_t)s * p.stage_bytes;
        const int ua = ch * p.experts_per_chunk;
        const int ub = min(U, ua + p.experts_per_chunk);
        const size_t qrow = (size_t)R * p.rs2, srow = (size_t)R * p.ss2;
        const size_t qtot = (size_t)(ub - ua) * qrow;
        const int nitems = (ub - ua) * ngrp;
        for (int item = warp; item < nitems; item += kConsumerWarps) {
            const int ui = item / ngrp, g = item % ngrp;
            const int u = ua + ui;
            const int row = g * RPG + rr;
            const bool rv = row < R;
            const uint8_t* wrow = st + ui * qrow + (size_t)(rv ? row : 0) * p.rs2;
            const uint16_t* srw = reinterpret_cast<const uint16_t*>(st + qtot + ui * srow + (size_t)(rv ? row : 0) * p.ss2);
            const int ps = rt.ups[u], cnt = rt.ucnt[u];
            for (int m0 = 0; m0 < cnt; m0 += kTokTile) {
                float acc[kTokTile];
#pragma unroll
                for (int m = 0; m < kTokTile; ++m) acc[m] = 0.f;
                if (rv) {
                    for (int b = sub; b < nb2; b += LPR) {
                        const uint4* w = reinterpret_cast<const uint4*>(wrow + (size_t)b * (Q4 ? 16 : 32));
                        const float dw = scale_to_f32(srw[b], sbf);
#pragma unroll
                        for (int m = 0; m < kTokTile; ++m) {
                            if (m0 + m >= cnt) continue;
                            const int pos = ps + m0 + m;
                            const uint4* a = reinterpret_cast<const uint4*>(hq + (size_t)pos * I + b * 32);
                            const int is = block_dot<Q4>(w, a, Q4 ? hs[pos * nb2 + b] : 0);
                            acc[m] += ((float)is * dw) * hd[pos * nb2 + b];
                        }
                    }
                }
#pragma unroll
                for (int m = 0; m < kTokTile; ++m)
                    for (int o = LPR >> 1; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
                if (rv && sub == 0) {
#pragma unroll
                    for (int m = 0; m < kTokTile; ++m)
                        if (m0 + m < cnt) outs[(size_t)(ps + m0 + m) * p.rows_max + row] = acc[m];
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == p.nstages) { s = 0; ph ^= 1; }
    }
    named_bar_sync(1, kConsumerThreads);
    if (!ok) return;

    // combine in k order (q8_gemm.cpp:593-613) and cast (q8_gemm.cpp:636-639)
    for (int idx = tid; idx < p.T * R; idx += kConsumerThreads) {
        const int t = idx / R, r = idx % R;
        float acc = 0.f;
        for (int k = 0; k < p.K; ++k) {
            const int pos = rt.smap[t * p.K + k];
            if (pos < 0) continue;
            acc += p.tw[t * p.K + k] * outs[(size_t)pos * p.rows_max + r];
        }
        const size_t o = (size_t)t * H + n0 + r;
        if (p.out_kind == 2) reinterpret_cast<float*>(p.y)[o] = acc;
        else if (p.out_kind == 1) reinterpret_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(acc);
        else reinterpret_cast<__half*>(p.y)[o] = __float2half_rn(acc);
    }
}

}  // namespace moe
