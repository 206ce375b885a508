// Persistent fused MoE layer kernel for decode-size token counts (Q8_0 / Q4_0 /
// AWQ W4A16).
//
// One CTA per SM (cooperative launch), kWarps warps per CTA, no producer warp:
// every warp streams its own work items with cp.async.bulk into a private ring
// of shared-memory slots (one mbarrier per slot) and computes on them.
//   phase 0  every CTA routes the T*K pairs itself (the stable counting sort of
//            moe_common.cpp:146-184) and quantises the T token rows to Q8_0
//            (gemm_kernels.cpp:25-58) in shared memory;
//   phase 1  gate_up: the U*I units (gate row j + up row j of an active expert)
//            are split into equal contiguous ranges, one per CTA, dealt to its
//            warps round-robin; a unit's rows are dotted with the expert's token
//            rows, SiLU(gate)*up goes to the fp32 workspace h[pos][j];
//   barrier  one grid barrier (bounded spin);
//   phase 2  every CTA requantises h, one thread per 32-block (pack_A_q8_0,
//            gemm_kernels.cpp:394-425), computes the down rows [n0,n1) it owns for
//            ALL active experts and then the k-ordered combine
//            y[t][n] = sum_k w[t,k] out[pos(t,k)][n] (q8_gemm.cpp:593-613).
// AWQ W4A16 keeps the activations 16-bit (no Q8_0 quantisation): a 32-block of a
// weight row contributes s * (sum q*x - z * sum x) with the group's bf16 scale s
// and zero z, and h stays fp32 (no requantisation, no block maxima).
// A warp's ring is issued `slots` items ahead across the phase boundary, so the
// down-projection weights are in flight while the CTAs wait at the grid
// barrier.  Weights cross HBM exactly once per launch.
#pragma once
#include "common.cuh"

namespace moe {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kTokTile = 4;  // token rows held in registers per pass
constexpr int kStamps = 20;

enum Fmt : int { kQ8 = 0, kQ4 = 1, kAWQ = 2 };
// kFlagEvictFirst: weight copies carry an L2 evict-first policy, so the streamed weights do
//   not displace what every launch re-reads (kernel code, tokens, routing, h, the barrier).
// kFlagLateDown: a warp issues its first down-row copy only after its first gate_up item
//   has arrived, so the gate_up bytes (on the critical path) are not queued behind them.
constexpr int kFlagEvictFirst = 1, kFlagLateDown = 2;

// Expert-parallel combine over peer memory (one process per GPU, NVLink P2P).  Every
// rank owns a mailbox [2 parities][world sources][tcap tokens][H] fp32 followed by flags
// [world sources][grid] u64; `data[q]` / `flag[q]` point into rank q's mailbox (this
// process's mapping of it).  CTA c of every rank covers the same output rows, so the
// exchange is CTA-to-CTA: no grid-wide step.
constexpr int kMaxPeers = 8;
struct PeerCombine {
    float* data[kMaxPeers];
    unsigned long long* flag[kMaxPeers];
    int32_t rank, world, tcap;
};
// The exchange epoch of a launch is its index on the engine's launch counter plus one
// (read by every CTA at the start, so graph replays get fresh epochs); ranks that make the
// same sequence of calls count the same epochs.

struct DecodeParams {
    // gate_up unit records [E][I]: gate qs row j (rs1) | up qs row j (rs1) | gate scales (ss1) | up scales (ss1)
    const uint8_t* gu;
    // down row records [E][H]: qs row n (rs2) | scales (ss2)
    const uint8_t* dn;
    int32_t rs1, ss1, rs2, ss2;
    int32_t E, e_off, H, I, T, K;
    const int32_t* emap;  // optional placement map: global expert id -> local id or -1 [emap_n]
    int32_t emap_n;
    int32_t scale_bf16, act_bf16, out_kind;  // out_kind: 0 f16, 1 bf16, 2 f32
    const void* x;
    void* y;
    const int32_t* ids;
    const float* tw;
    float* h_ws;         // [T*K][I]
    const uint8_t* dk;   // split-K kernel: down chunks [E][I/32][H/32] x (32 rows x BB | 32 scales)
    float* part;         // split-K kernel: per-CTA fp32 partial tiles [grid][T][H]
    unsigned long long* bar;  // grid barrier arrival counter (monotonic)
    int32_t* err;        // device error word
    // shared-memory carve-up (bytes)
    int32_t off_x, off_out, off_ring, slot_bytes, slots;
    int32_t rows_max;       // phase-2 rows per CTA (upper bound)
    int32_t lanes_per_row;  // phase-2 lanes per down row (power of two)
    int32_t units_per_item; // phase-1 gate/up units per bulk copy (1, 2 or 4)
    int32_t group;          // AWQ group size along K (multiple of 32)
    int32_t dist_min_blocks;  // Q8/Q4: requantise h before the grid barrier when U*I/32 >= this
    int32_t flags;            // kFlagEvictFirst | kFlagLateDown
    int32_t sk_cost_a;        // split-K kernel: cost of streaming one chunk, in units of one token's compute
    unsigned long long* dbg;  // optional per-CTA phase stamps [grid][kStamps] (globaltimer ns)
    PeerCombine pc;           // pc.world > 1: the output rows are summed over the ranks' partials
};

MOE_DEV void st_out(const DecodeParams& p, size_t o, float v) {
    if (p.out_kind == 2) reinterpret_cast<float*>(p.y)[o] = v;
    else if (p.out_kind == 1) reinterpret_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(v);
    else reinterpret_cast<__half*>(p.y)[o] = __float2half_rn(v);
}

// This rank's partial of output element (t, n) into slot [parity][rank] of every rank's mailbox.
MOE_DEV void pc_put(const DecodeParams& p, unsigned long long epoch, int t, int n, float v) {
    const PeerCombine& pc = p.pc;
    const size_t o = (((size_t)(epoch & 1) * pc.world + pc.rank) * pc.tcap + t) * p.H + n;
    for (int q = 0; q < pc.world; ++q) pc.data[q][o] = v;
}

// After every thread of the CTA has put its rows [n0, n0+R): publish this CTA's flag on
// every rank, wait (bounded) for CTA `cta` of every other rank, then sum the partials in
// rank order (deterministic) and write the output rows.  Returns false when a peer did not
// arrive within the wait budget (the error word is set; the rows are left unwritten).
MOE_DEV bool pc_finish(const DecodeParams& p, unsigned long long epoch, int cta, int G, int n0, int R, int tid) {
    const PeerCombine& pc = p.pc;
    __shared__ int s_pc_ok;
    __syncthreads();
    if (tid == 0) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");  // this CTA's puts before its flags
        for (int q = 0; q < pc.world; ++q)
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(pc.flag[q] + (size_t)pc.rank * G + cta),
                         "l"(epoch)
                         : "memory");
        int ok = 1;
        for (int src = 0; src < pc.world && ok; ++src) {
            if (src == pc.rank) continue;
            const unsigned long long* f = pc.flag[pc.rank] + (size_t)src * G + cta;
            uint32_t it = 0;
            for (;; ++it) {
                unsigned long long v;
                asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(f) : "memory");
                if (v >= epoch) break;
                if (it >= kSpinLimit) { ok = 0; break; }
                if (it > 256) __nanosleep(256);
            }
        }
        if (!ok) set_err(p.err, kErrPeerWait);
        s_pc_ok = ok;
    }
    __syncthreads();
    if (!s_pc_ok) return false;
    const float* mine = pc.data[pc.rank];
    const size_t par = (size_t)(epoch & 1) * pc.world;
    for (int idx = tid; idx < p.T * R; idx += blockDim.x) {
        const int t = idx / R, n = n0 + idx % R;
        float acc = 0.f;
        for (int src = 0; src < pc.world; ++src) acc += __ldcv(mine + ((par + src) * pc.tcap + t) * p.H + n);
        st_out(p, (size_t)t * p.H + n, acc);
    }
    return true;
}

MOE_DEV unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

MOE_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

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
MOE_DEV void route_warp(const int32_t* g_ids, int TK, int K, int E, int e_off, const int32_t* emap, int emap_n, RouteSmem r,
                        int lane) {
#pragma unroll 1
    for (int e = lane; e < E; e += 32) r.cnt[e] = 0;
    __syncwarp();
#pragma unroll 1
    for (int i0 = 0; i0 < TK; i0 += 32) {
        const int i = i0 + lane;
        int e = -1;
        if (i < TK) {
            e = local_expert(g_ids[i], e_off, E, emap, emap_n, i, K);
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
    // exclusive scan of counts -> start, and the unique-expert list: lane l owns the
    // contiguous experts [l*c, l*c + c); one warp scan of (actives << 16 | count).
    const int c = (E + 31) >> 5;
    int loc = 0;
#pragma unroll 1
    for (int k = 0; k < c; ++k) {
        const int e = lane * c + k;
        const int n = e < E ? r.cnt[e] : 0;
        loc += (n > 0 ? (1 << 16) : 0) + n;
    }
    int incl = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    int run = incl - loc;  // exclusive prefix of this lane's chunk
#pragma unroll 1
    for (int k = 0; k < c; ++k) {
        const int e = lane * c + k;
        if (e >= E) break;
        const int n = r.cnt[e];
        const int pos0 = run & 0xffff, u = run >> 16;
        r.start[e] = pos0;
        if (n > 0) {
            r.ue[u] = e;
            r.ups[u] = pos0;
            r.ucnt[u] = n;
        }
        run += (n > 0 ? (1 << 16) : 0) + n;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    const int carry = total & 0xffff, ucarry = total >> 16;
    if (lane == 0) {
        r.start[E] = carry;
        *r.nuniq = ucarry;
    }
    __syncwarp();
#pragma unroll 1
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
// Q4_0 activation byte order inside a 32-block: the weight word w holds
// elements 8w..8w+7 in nibbles 0..7, so its low nibbles are elements
// 8w+{0,2,4,6} and its high nibbles 8w+{1,3,5,7}.
MOE_DEV int q4_perm(int e) {
    const int w = e >> 3, r = e & 7;
    return (w << 3) + ((r & 1) << 2) + (r >> 1);
}

// Quantise one 32-block held by one thread (v[32]) with scale d into 8 packed
// 32-bit words (Q4: the permuted activation order, Q8: natural order) and
// return the sum of the quantised values.
template <bool Q4>
MOE_DEV int quant_block_store(const float* v, float d, int8_t* qb) {
    const float id = q8_inv(d);
    int q[32];
    int sum = 0;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
        q[e] = q8_quant(v[e], id);
        sum += q[e];
    }
    uint32_t wv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        uint32_t w = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int e = Q4 ? 8 * (k >> 1) + (k & 1) + 2 * i : 4 * k + i;
            w |= (uint32_t)(q[e] & 0xff) << (8 * i);
        }
        wv[k] = w;
    }
    uint4* dst = reinterpret_cast<uint4*>(qb);
    dst[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    dst[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
    return sum;
}

// Token rows -> Q8_0 in shared memory, one thread per 32-block (no shuffles,
// one global round trip per block).
template <bool Q4>
MOE_DEV void quant_x_smem(const uint8_t* x, int act_bf16, int nrows, int cols, int8_t* q, float* d, int32_t* s,
                          int tid, int nthreads) {
    const int nb = cols >> 5;
    const int nblk = nrows * nb;
    for (int g = tid; g < nblk; g += nthreads) {
        const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)g * 64);  // rows contiguous: block g at g*32
        uint4 raw[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) raw[k] = __ldg(src + k);
        float v[32];
        float amax = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t w4[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[8 * k + 2 * i] = scale_to_f32((uint16_t)(w4[i] & 0xffffu), act_bf16);
                v[8 * k + 2 * i + 1] = scale_to_f32((uint16_t)(w4[i] >> 16), act_bf16);
            }
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) amax = fmaxf(amax, fabsf(v[e]));
        const float dd = q8_scale(amax);
        const int sum = quant_block_store<Q4>(v, dd, q + (size_t)g * 32);
        d[g] = dd;
        if (Q4) s[g] = sum;
    }
}

// One 32-block of h quantised by a quad of lanes (sub = lane & 3 holds elements
// 8sub..8sub+7 in v and writes output bytes 8sub..8sub+7): the quad reduces the
// maximum and the sum with shuffles, so the result equals the one-thread rule of
// pack_A_q8_0 (max and integer sum do not depend on the order).  For Q4 the byte
// order is the permuted activation order (word 2sub: elements 8sub+{0,2,4,6},
// word 2sub+1: 8sub+{1,3,5,7}); for Q8 it is the natural order.
template <bool Q4>
MOE_DEV void quad_quant(const float (&v)[8], uint32_t qmask, float& d, int& sum, uint2& out) {
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(v[e]));
    amax = fmaxf(amax, __shfl_xor_sync(qmask, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(qmask, amax, 2));
    d = q8_scale(amax);
    const float id = q8_inv(d);
    int q[8];
    sum = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        q[e] = q8_quant(v[e], id);
        sum += q[e];
    }
    sum += __shfl_xor_sync(qmask, sum, 1);
    sum += __shfl_xor_sync(qmask, sum, 2);
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        w0 |= (uint32_t)(q[Q4 ? 2 * i : i] & 0xff) << (8 * i);
        w1 |= (uint32_t)(q[Q4 ? 2 * i + 1 : 4 + i] & 0xff) << (8 * i);
    }
    out = make_uint2(w0, w1);
}

MOE_DEV uint32_t quad_mask(int lane) { return 0xfu << (lane & ~3); }

// Token rows -> Q8_0 in shared memory, a quad of threads per 32-block (8 elements each, the
// block maximum and sum by shuffles): the same result as quant_x_smem with a quarter of its
// code.  nthreads must be a multiple of 4.
template <bool Q4>
MOE_DEV void quant_x_quad(const uint8_t* x, int act_bf16, int nrows, int cols, int8_t* q, float* d, int32_t* s,
                          int tid, int nthreads) {
    const int nblk = nrows * (cols >> 5), sub = tid & 3;
    const uint32_t qm = quad_mask(tid & 31);
#pragma unroll 1
    for (int g = tid >> 2; g < nblk; g += nthreads >> 2) {  // the 4 threads of a quad share g
        float v[8];
        const uint4 r = __ldg(reinterpret_cast<const uint4*>(x + (size_t)g * 64) + sub);
        const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = scale_to_f32((uint16_t)(w4[i] & 0xffffu), act_bf16);
            v[2 * i + 1] = scale_to_f32((uint16_t)(w4[i] >> 16), act_bf16);
        }
        float dd;
        int sum;
        uint2 o;
        quad_quant<Q4>(v, qm, dd, sum, o);
        *reinterpret_cast<uint2*>(q + (size_t)g * 32 + sub * 8) = o;
        if (sub == 0) {
            d[g] = dd;
            if (Q4) s[g] = sum;
        }
    }
}

MOE_DEV void load8(const float* src, float (&v)[8]) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(src));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(src) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Requantise all of h [P][I] (fp32, global) into shared memory, a quad per 32-block.
template <bool Q4>
MOE_DEV void requant_h_smem(const float* h, int P, int I, int8_t* q, float* d, int32_t* s, int tid) {
    const int nblk = P * (I >> 5), sub = tid & 3;
    const uint32_t qm = quad_mask(tid & 31);
    for (int g = tid >> 2; g < nblk; g += kThreads / 4) {
        float v[8];
        load8(h + (size_t)g * 32 + sub * 8, v);
        float dd;
        int sum;
        uint2 o;
        quad_quant<Q4>(v, qm, dd, sum, o);
        *reinterpret_cast<uint2*>(q + (size_t)g * 32 + sub * 8) = o;
        if (sub == 0) {
            d[g] = dd;
            if (Q4) s[g] = sum;
        }
    }
}

// Before the grid barrier: this CTA requantises the 32-blocks [bb, be) of the
// unique-expert x I unit space that its own phase 1 produced, in place: the
// 128-byte fp32 slot h[pos][32jb..32jb+31] becomes q (32 B) | d (4 B) | sum (4 B).
// Only the owning quad reads and writes a slot, so the overwrite is race free.
template <bool Q4>
MOE_DEV void requant_own_blocks(float* h, const RouteSmem& rt, int I, int nb2, int bb, int be, int tid) {
    const int sub = tid & 3;
    const uint32_t qm = quad_mask(tid & 31);
    int t = tid >> 2;
    for (int u = bb / nb2; u * nb2 < be; ++u) {
        const int jb0 = max(bb, u * nb2) - u * nb2, jb1 = min(be, (u + 1) * nb2) - u * nb2;
        const int nj = jb1 - jb0, n = nj * rt.ucnt[u];
        for (; t < n; t += kThreads / 4) {
            const int m = t / nj, jb = jb0 + (t - m * nj);
            float* slot = h + (size_t)(rt.ups[u] + m) * I + jb * 32;
            float v[8];
            load8(slot + sub * 8, v);
            float dd;
            int sum;
            uint2 o;
            quad_quant<Q4>(v, qm, dd, sum, o);  // every lane's loads precede the shuffles, hence the stores
            uint8_t* sb = reinterpret_cast<uint8_t*>(slot);
            *reinterpret_cast<uint2*>(sb + sub * 8) = o;
            if (sub == 0) *reinterpret_cast<float2*>(sb + 32) = make_float2(dd, __int_as_float(sum));
        }
        t -= n;
    }
}

// After the grid barrier: gather the requantised slots of every position into
// shared memory (q [P][I], d and sum [P][I/32]).
template <bool Q4>
MOE_DEV void gather_h_smem(const float* h, int P, int I, int8_t* q, float* d, int32_t* s, int tid) {
    const int nb2 = I >> 5, nblk = P * nb2;
    for (int g = tid >> 1; g < nblk; g += kThreads / 2) {  // a lane pair per slot
        const uint8_t* sb = reinterpret_cast<const uint8_t*>(h + (size_t)g * 32);
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(sb) + (tid & 1));
        const float2 ds = (tid & 1) ? __ldcg(reinterpret_cast<const float2*>(sb + 32)) : make_float2(0.f, 0.f);
        *reinterpret_cast<uint4*>(q + (size_t)g * 32 + (tid & 1) * 16) = v;
        if (tid & 1) {
            d[g] = ds.x;
            if (Q4) s[g] = __float_as_int(ds.y);
        }
    }
}

// ------------------------------------------------------------------ AWQ
// Token rows for AWQ: the raw 16-bit values are kept and each 32-block's sum
// (fp32) is stored beside them, one thread per block.
MOE_DEV void stage_x_awq(const uint8_t* x, int act_bf16, int nrows, int cols, uint16_t* xr, float* xsum, int tid,
                         int nthreads) {
    const int nblk = nrows * (cols >> 5);
    for (int g = tid; g < nblk; g += nthreads) {
        const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)g * 64);
        uint4* dst = reinterpret_cast<uint4*>(xr + (size_t)g * 32);
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 r = __ldg(src + k);
            dst[k] = r;
            const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
                sum += scale_to_f32((uint16_t)(w4[i] & 0xffffu), act_bf16) + scale_to_f32((uint16_t)(w4[i] >> 16), act_bf16);
        }
        xsum[g] = sum;
    }
}

// h [P][I] fp32 (global) -> shared memory with per-block sums, one thread per block.
MOE_DEV void stage_h_awq(const float* h, int P, int I, float* hf, float* hsum, int tid) {
    const int nblk = P * (I >> 5);
    for (int g = tid; g < nblk; g += kThreads) {
        const float4* src = reinterpret_cast<const float4*>(h + (size_t)g * 32);
        float4* dst = reinterpret_cast<float4*>(hf + (size_t)g * 32);
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float4 f = __ldcg(src + k);
            dst[k] = f;
            sum += (f.x + f.y) + (f.z + f.w);
        }
        hsum[g] = sum;
    }
}

MOE_DEV float nib_f(uint32_t w, int n) { return __uint_as_float(0x4B000000u | ((w >> (4 * n)) & 0xFu)) - 8388608.0f; }

// sum over a 32-block of q[e] * x[e], q the sequential nibbles of `qw`, x fp32 or 16-bit.
MOE_DEV float awq_qx_f32(const uint4 qw, const float* x) {
    const uint32_t w4[4] = {qw.x, qw.y, qw.z, qw.w};
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 a = reinterpret_cast<const float4*>(x)[2 * i];
        const float4 b = reinterpret_cast<const float4*>(x)[2 * i + 1];
        acc0 = fmaf(nib_f(w4[i], 0), a.x, acc0);
        acc1 = fmaf(nib_f(w4[i], 1), a.y, acc1);
        acc0 = fmaf(nib_f(w4[i], 2), a.z, acc0);
        acc1 = fmaf(nib_f(w4[i], 3), a.w, acc1);
        acc0 = fmaf(nib_f(w4[i], 4), b.x, acc0);
        acc1 = fmaf(nib_f(w4[i], 5), b.y, acc1);
        acc0 = fmaf(nib_f(w4[i], 6), b.z, acc0);
        acc1 = fmaf(nib_f(w4[i], 7), b.w, acc1);
    }
    return acc0 + acc1;
}

MOE_DEV float awq_qx_16(const uint4 qw, const uint16_t* x, int bf) {
    const uint32_t w4[4] = {qw.x, qw.y, qw.z, qw.w};
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 r = reinterpret_cast<const uint4*>(x)[i];
        const uint32_t xv[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            acc0 = fmaf(nib_f(w4[i], 2 * k), scale_to_f32((uint16_t)(xv[k] & 0xffffu), bf), acc0);
            acc1 = fmaf(nib_f(w4[i], 2 * k + 1), scale_to_f32((uint16_t)(xv[k] >> 16), bf), acc1);
        }
    }
    return acc0 + acc1;
}

// Group scale (bf16) and zero (u8) of 32-block b of a row whose scale field is `sc`.
MOE_DEV void awq_sz(const uint8_t* sc, int b, int blocks_per_group, int ngroups, float& s, float& z) {
    const int g = b / blocks_per_group;
    s = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(sc)[g] << 16);
    z = (float)sc[2 * ngroups + g];
}

// Exact int32 dot of one 32-block: weights (Q8: 32 bytes, Q4: 16 bytes of
// nibbles) against 32 int8 activations (Q4: permuted, bias 8 via asum).
template <bool Q4>
MOE_DEV int block_dot(const uint4* w, const uint4* a, int asum) {
    // four independent dp4a chains (integer sums: the order does not change the result)
    if (Q4) {
        const uint4 ww = w[0];
        const uint4 a0 = a[0], a1 = a[1];
        int s0 = __dp4a((int)(ww.x & 0x0f0f0f0fu), (int)a0.x, 0);
        int s1 = __dp4a((int)(ww.y & 0x0f0f0f0fu), (int)a0.z, 0);
        int s2 = __dp4a((int)(ww.z & 0x0f0f0f0fu), (int)a1.x, 0);
        int s3 = __dp4a((int)(ww.w & 0x0f0f0f0fu), (int)a1.z, 0);
        s0 = __dp4a((int)((ww.x >> 4) & 0x0f0f0f0fu), (int)a0.y, s0);
        s1 = __dp4a((int)((ww.y >> 4) & 0x0f0f0f0fu), (int)a0.w, s1);
        s2 = __dp4a((int)((ww.z >> 4) & 0x0f0f0f0fu), (int)a1.y, s2);
        s3 = __dp4a((int)((ww.w >> 4) & 0x0f0f0f0fu), (int)a1.w, s3);
        return (s0 + s1) + (s2 + s3) - 8 * asum;
    } else {
        const uint4 w0 = w[0], w1 = w[1];
        const uint4 a0 = a[0], a1 = a[1];
        int s0 = __dp4a((int)w0.x, (int)a0.x, 0);
        int s1 = __dp4a((int)w0.y, (int)a0.y, 0);
        int s2 = __dp4a((int)w0.z, (int)a0.z, 0);
        int s3 = __dp4a((int)w0.w, (int)a0.w, 0);
        s0 = __dp4a((int)w1.x, (int)a1.x, s0);
        s1 = __dp4a((int)w1.y, (int)a1.y, s1);
        s2 = __dp4a((int)w1.z, (int)a1.z, s2);
        s3 = __dp4a((int)w1.w, (int)a1.w, s3);
        return (s0 + s1) + (s2 + s3);
    }
}

// Work of one warp.  Phase 1: the warp's contiguous share [u_cur, u_end) of the
// CTA's units, cut into items of up to `upi` consecutive units of one expert.
// Phase 2: items (expert ui, group g of RPG rows), it = warp + k*kWarps.
struct P1Cursor {
    int64_t cur, end;
    int I, upi;
    // next item: unique expert index u, first unit j0, unit count n
    MOE_DEV bool next(int& u, int& j0, int& n) {
        if (cur >= end) return false;
        u = (int)(cur / I);
        j0 = (int)(cur - (int64_t)u * I);
        int64_t m = end - cur;
        if (m > I - j0) m = I - j0;
        if (m > upi) m = upi;
        n = (int)m;
        cur += m;
        return true;
    }
};

struct P2Work {
    int n2, ngrp, RPG, R, n0;
};

MOE_DEV void issue_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    mbar_arrive_expect_tx(bar, bytes);
    if (pol) bulk_g2s_hint(dst, src, bytes, bar, pol);
    else bulk_g2s(dst, src, bytes, bar);
}

MOE_DEV void issue_p1(const DecodeParams& p, const RouteSmem& rt, int u, int j0, int n, uint8_t* slot, uint64_t* bar,
                      uint64_t pol) {
    const uint32_t ub = 2u * (p.rs1 + p.ss1);
    issue_copy(slot, p.gu + ((size_t)rt.ue[u] * p.I + j0) * ub, ub * n, bar, pol);
}

MOE_DEV void issue_p2(const DecodeParams& p, const RouteSmem& rt, const P2Work& w2, int it, uint8_t* slot,
                      uint64_t* bar, uint64_t pol) {
    const int ui = it / w2.ngrp, g = it - ui * w2.ngrp;
    const int r0 = g * w2.RPG;
    const int rows = min(w2.RPG, w2.R - r0);
    const uint32_t rb = (uint32_t)(p.rs2 + p.ss2);
    issue_copy(slot, p.dn + ((size_t)rt.ue[ui] * p.H + w2.n0 + r0) * rb, rows * rb, bar, pol);
}

template <int FMT>
__global__ void __launch_bounds__(kThreads, 1) moe_decode_kernel(const DecodeParams p) {
    constexpr bool Q4 = FMT == kQ4;
    constexpr bool AWQ = FMT == kAWQ;
    constexpr int BB = FMT == kQ8 ? 32 : 16;  // weight bytes per 32-block
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int TK = p.T * p.K, E = p.E, H = p.H, I = p.I;
    const int nb1 = H >> 5, nb2 = I >> 5;
    const int bpg = AWQ ? p.group >> 5 : 1, ng1 = AWQ ? H / p.group : 0, ng2 = AWQ ? I / p.group : 0;
    unsigned long long* dbg = p.dbg ? p.dbg + (size_t)cta * kStamps : nullptr;
    if (dbg && tid == 0) { dbg[0] = global_ns(); dbg[13] = clock64(); }

    RouteSmem rt = carve_route(reinterpret_cast<int32_t*>(smem), TK, E);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_ring - 8 * kWarps * p.slots);
    uint64_t* mybar = bars + warp * p.slots;
    uint8_t* myring = smem + p.off_ring + (size_t)warp * p.slots * p.slot_bytes;
    int8_t* xq = reinterpret_cast<int8_t*>(smem + p.off_x);
    float* xd = reinterpret_cast<float*>(xq + (size_t)p.T * H);
    int32_t* xs = reinterpret_cast<int32_t*>(xd + (size_t)p.T * nb1);
    __shared__ int s_ok;
    __shared__ unsigned long long s_launch;

    // ---------------- phase 0 ----------------
    if (lane == 0)
        for (int s = 0; s < p.slots; ++s) mbar_init(&mybar[s], 1);
    if (warp == kWarps - 1) {  // one warp routes while the others quantise the tokens
        // this launch's barrier target: the load is in flight while the warp routes
        const unsigned long long launch_idx = barrier_launch_index(p.bar, (uint32_t)G);
        route_warp(p.ids, TK, p.K, E, p.e_off, p.emap, p.emap_n, rt, lane);
        if (lane == 0) {
            s_ok = 1;
            s_launch = launch_idx;
            if (dbg) dbg[1] = global_ns();
        }
    } else {
        if constexpr (AWQ)
            stage_x_awq(static_cast<const uint8_t*>(p.x), p.act_bf16, p.T, H, reinterpret_cast<uint16_t*>(xq),
                        reinterpret_cast<float*>(xq + (size_t)p.T * H * 2), tid, kThreads - 32);
        else
            quant_x_smem<Q4>(static_cast<const uint8_t*>(p.x), p.act_bf16, p.T, H, xq, xd, xs, tid, kThreads - 32);
        if (dbg && tid == 0) dbg[2] = global_ns();
    }
    fence_barrier_init();
    __syncthreads();
    if (dbg && tid == 0) dbg[3] = global_ns();

    const int U = *rt.nuniq;
    const unsigned long long launch = s_launch;

    // this warp's phase-1 share and phase-2 items; in the distributed-requant mode a
    // CTA owns whole 32-blocks of units so it can requantise them itself
    const int64_t TU = (int64_t)U * I;
    const int NB = U * nb2;
    const bool dist = !AWQ && NB >= p.dist_min_blocks;
    const int bb = (int)((int64_t)NB * cta / G), be = (int)((int64_t)NB * (cta + 1) / G);
    const int64_t cb = dist ? (int64_t)bb * 32 : TU * cta / G, ce = dist ? (int64_t)be * 32 : TU * (cta + 1) / G;
    P1Cursor c_issue{cb + (ce - cb) * warp / kWarps, cb + (ce - cb) * (warp + 1) / kWarps, I, p.units_per_item};
    P1Cursor c_use = c_issue;
    P2Work w2;
    w2.n0 = (int)((int64_t)H * cta / G);
    w2.R = (int)((int64_t)H * (cta + 1) / G) - w2.n0;
    w2.RPG = 32 / p.lanes_per_row;
    w2.ngrp = (w2.R + w2.RPG - 1) / w2.RPG;
    const int tot2 = U * w2.ngrp;
    w2.n2 = warp < tot2 ? (tot2 - warp + kWarps - 1) / kWarps : 0;
    int issued2 = 0;  // phase-2 items issued so far
    int nissued = 0;  // items issued so far; item k sits in ring slot k % slots
    const uint64_t pol = (p.flags & kFlagEvictFirst) ? l2_evict_first_policy() : 0ull;

    // lane 0 fills the free ring slots (items are consumed in issue order): phase-1
    // items first, then phase-2 items when allowed
    auto top_up = [&](int consumed, bool allow_p2) {
        __syncwarp();  // every lane's reads of the consumed slots are complete before reuse
        if (lane == 0) {
            while (nissued - consumed < p.slots) {
                const int s = nissued % p.slots;
                int u, j0, n;
                if (c_issue.next(u, j0, n)) {
                    issue_p1(p, rt, u, j0, n, myring + (size_t)s * p.slot_bytes, &mybar[s], pol);
                } else if (allow_p2 && issued2 < w2.n2) {
                    issue_p2(p, rt, w2, warp + issued2 * kWarps, myring + (size_t)s * p.slot_bytes, &mybar[s], pol);
                    if (dbg && warp == 0 && issued2 == 0) dbg[15] = global_ns();
                    ++issued2;
                } else {
                    break;
                }
                ++nissued;
            }
        }
        // lane 0 advanced the cursors; keep the other lanes' copies in step
        c_issue.cur = __shfl_sync(0xffffffffu, c_issue.cur, 0);
        issued2 = __shfl_sync(0xffffffffu, issued2, 0);
        nissued = __shfl_sync(0xffffffffu, nissued, 0);
    };
    top_up(0, !(p.flags & kFlagLateDown) || c_issue.cur >= c_issue.end);
    auto refill = [&](int consumed) { top_up(consumed, true); };

    const bool sbf = p.scale_bf16 != 0;
    bool ok = true;
    int item = 0;

    // ---------------- phase 1: gate_up + SiLU*up ----------------
    {
        const int LPU = 32 / p.units_per_item;  // lanes per unit
        const int usub = lane % LPU, uslot = lane / LPU;
        int u, j0, n;
        while (c_use.next(u, j0, n)) {
            const int s = item % p.slots;
            if (!mbar_wait(&mybar[s], (uint32_t)(item / p.slots) & 1u)) { set_err(p.err, kErrFullWait); ok = false; break; }
            if (dbg && tid == 0) dbg[item == 0 ? 4 : 5] = global_ns();
            const bool valid = uslot < n;
            const uint8_t* rec = myring + (size_t)s * p.slot_bytes + (size_t)(valid ? uslot : 0) * 2 * (p.rs1 + p.ss1);
            const uint8_t* qg = rec;
            const uint8_t* qu = rec + p.rs1;
            const uint8_t* sgate_raw = rec + 2 * p.rs1;
            const uint8_t* sup_raw = rec + 2 * p.rs1 + p.ss1;
            const uint16_t* sgate = reinterpret_cast<const uint16_t*>(sgate_raw);
            const uint16_t* sup = reinterpret_cast<const uint16_t*>(sup_raw);
            const int j = j0 + uslot;
            const int ps = rt.ups[u], cnt = rt.ucnt[u];
            for (int m0 = 0; m0 < cnt; m0 += kTokTile) {  // up to kTokTile tokens per weight load
                const int nt = min(kTokTile, cnt - m0);
                int tk[kTokTile];
                float ag[kTokTile], au[kTokTile];
#pragma unroll
                for (int m = 0; m < kTokTile; ++m) {
                    tk[m] = m < nt ? rt.tok[ps + m0 + m] / p.K : 0;
                    ag[m] = 0.f;
                    au[m] = 0.f;
                }
                if (valid) {
#pragma unroll 4
                    for (int b = usub; b < nb1; b += LPU) {
                        const uint4* wg = reinterpret_cast<const uint4*>(qg + (size_t)b * BB);
                        const uint4* wu = reinterpret_cast<const uint4*>(qu + (size_t)b * BB);
                        if constexpr (AWQ) {
                            float sg, zg, su, zu;
                            awq_sz(sgate_raw, b, bpg, ng1, sg, zg);
                            awq_sz(sup_raw, b, bpg, ng1, su, zu);
                            const uint4 qwg = wg[0], qwu = wu[0];
                            const uint16_t* xr = reinterpret_cast<const uint16_t*>(xq);
                            const float* xsum = reinterpret_cast<const float*>(xq + (size_t)p.T * H * 2);
#pragma unroll
                            for (int m = 0; m < kTokTile; ++m) {
                                if (m >= nt) break;
                                const int t = tk[m];
                                const uint16_t* xb = xr + (size_t)t * H + b * 32;
                                const float sx = xsum[t * nb1 + b];
                                ag[m] += sg * (awq_qx_16(qwg, xb, p.act_bf16) - zg * sx);
                                au[m] += su * (awq_qx_16(qwu, xb, p.act_bf16) - zu * sx);
                            }
                        } else {
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
                }
#pragma unroll
                for (int m = 0; m < kTokTile; ++m) {
                    if (m >= nt) break;  // uniform within the warp
                    for (int o = LPU >> 1; o > 0; o >>= 1) {
                        ag[m] += __shfl_xor_sync(0xffffffffu, ag[m], o);
                        au[m] += __shfl_xor_sync(0xffffffffu, au[m], o);
                    }
                }
                // lane usub == m of each unit group finishes token m
                if (valid && usub < nt) {
                    float g = ag[0], uu = au[0];
#pragma unroll
                    for (int m = 1; m < kTokTile; ++m)
                        if (usub == m) { g = ag[m]; uu = au[m]; }
                    const float hv = silu_mul(g, uu);
                    const int pos = ps + m0 + usub;
                    p.h_ws[(size_t)pos * I + j] = hv;
                }
            }
            ++item;
            refill(item);
        }
    }
    if (dbg && tid == 0) dbg[6] = global_ns();

    // ---------------- grid barrier ----------------
    __syncthreads();
    if constexpr (!AWQ) {
        if (dist && ok) {
            requant_own_blocks<Q4>(p.h_ws, rt, I, nb2, bb, be, tid);
            __syncthreads();
        }
    }
    if (dbg && tid == 0) dbg[7] = global_ns();
    if (tid == 1) {  // a lane that issues no bulk copies: its release waits on no copy in flight
        if (!grid_barrier(p.bar, (uint32_t)G, (launch + 1ull) * (uint32_t)G, p.err, dbg ? dbg + 16 : nullptr)) s_ok = 0;
    }
    __syncthreads();
    ok = ok && s_ok;
    if (dbg && tid == 0) dbg[8] = global_ns();

    // ---------------- phase 2: requant h, down rows, combine ----------------
    const int P = rt.start[E];
    int8_t* hq = reinterpret_cast<int8_t*>(smem + p.off_x);
    float* hd = reinterpret_cast<float*>(hq + (size_t)P * I);
    int32_t* hs = reinterpret_cast<int32_t*>(hd + (size_t)P * nb2);
    float* outs = reinterpret_cast<float*>(smem + p.off_out);
    float* hf = reinterpret_cast<float*>(smem + p.off_x);        // AWQ: fp32 h [P][I]
    float* hsum = hf + (size_t)P * I;                              // AWQ: per-block sums
    if (ok && w2.R > 0 && U > 0) {
        if constexpr (AWQ) stage_h_awq(p.h_ws, P, I, hf, hsum, tid);
        else if (dist) gather_h_smem<Q4>(p.h_ws, P, I, hq, hd, hs, tid);
        else requant_h_smem<Q4>(p.h_ws, P, I, hq, hd, hs, tid);
    }
    __syncthreads();
    if (dbg && tid == 0) dbg[9] = global_ns();

    const int LPR = p.lanes_per_row;
    const int sub = lane % LPR, rr = lane / LPR;
    for (int k2 = 0; ok && k2 < w2.n2; ++k2) {
        const int s = item % p.slots;
        if (dbg && tid == 0 && k2 == 0) dbg[19] = global_ns();
        if (!mbar_wait(&mybar[s], (uint32_t)(item / p.slots) & 1u)) { set_err(p.err, kErrFullWait); ok = false; break; }
        if (dbg && tid == 0 && k2 == 0) dbg[10] = global_ns();
        const uint8_t* st = myring + (size_t)s * p.slot_bytes;
        const int it = warp + k2 * kWarps;
        const int ui = it / w2.ngrp, g = it - ui * w2.ngrp;
        const int row = g * w2.RPG + rr;
        const bool rv = row < w2.R;
        const uint8_t* wrow = st + (size_t)rr * (p.rs2 + p.ss2);
        const uint16_t* srw = reinterpret_cast<const uint16_t*>(wrow + p.rs2);
        const int ps = rt.ups[ui], cnt = rt.ucnt[ui];
        for (int m0 = 0; m0 < cnt; m0 += kTokTile) {
            const int nt = min(kTokTile, cnt - m0);
            float acc[kTokTile];
#pragma unroll
            for (int m = 0; m < kTokTile; ++m) acc[m] = 0.f;
            if (rv) {
#pragma unroll 2
                for (int b = sub; b < nb2; b += LPR) {
                    const uint4* w = reinterpret_cast<const uint4*>(wrow + (size_t)b * BB);
                    if constexpr (AWQ) {
                        float sw, zw;
                        awq_sz(wrow + p.rs2, b, bpg, ng2, sw, zw);
                        const uint4 qw = w[0];
#pragma unroll
                        for (int m = 0; m < kTokTile; ++m) {
                            if (m >= nt) break;
                            const int pos = ps + m0 + m;
                            acc[m] += sw * (awq_qx_f32(qw, hf + (size_t)pos * I + b * 32) - zw * hsum[pos * nb2 + b]);
                        }
                    } else {
                        const float dw = scale_to_f32(srw[b], sbf);
#pragma unroll
                        for (int m = 0; m < kTokTile; ++m) {
                            if (m >= nt) break;
                            const int pos = ps + m0 + m;
                            const uint4* a = reinterpret_cast<const uint4*>(hq + (size_t)pos * I + b * 32);
                            const int is = block_dot<Q4>(w, a, Q4 ? hs[pos * nb2 + b] : 0);
                            acc[m] += ((float)is * dw) * hd[pos * nb2 + b];
                        }
                    }
                }
            }
#pragma unroll
            for (int m = 0; m < kTokTile; ++m) {
                if (m >= nt) break;
                for (int o = LPR >> 1; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
            }
            if (rv && sub == 0) {
#pragma unroll
                for (int m = 0; m < kTokTile; ++m)
                    if (m < nt) outs[(size_t)(ps + m0 + m) * p.rows_max + row] = acc[m];
            }
        }
        ++item;
        refill(item);
    }
    if (dbg && tid == 0) dbg[18] = global_ns();
    // drain: a warp that stopped early still waits (bounded) for its copies in flight
    if (!ok && lane == 0)
        for (int i = item; i < nissued; ++i) mbar_wait(&mybar[i % p.slots], (uint32_t)(i / p.slots) & 1u);
    __syncthreads();
    if (dbg && tid == 0) dbg[11] = global_ns();
    if (!ok) return;

    // combine in k order (q8_gemm.cpp:593-613) and cast (q8_gemm.cpp:636-639)
    const int R = w2.R, n0 = w2.n0;
    for (int idx = tid; idx < p.T * R; idx += kThreads) {
        const int t = idx / R, r = idx % R;
        float acc = 0.f;
        for (int k = 0; k < p.K; ++k) {
            const int pos = rt.smap[t * p.K + k];
            if (pos < 0) continue;
            acc += p.tw[t * p.K + k] * outs[(size_t)pos * p.rows_max + r];
        }
        if (p.pc.world > 1) pc_put(p, launch + 1, t, n0 + r, acc);
        else st_out(p, (size_t)t * H + n0 + r, acc);
    }
    if (p.pc.world > 1) pc_finish(p, launch + 1, cta, G, n0, R, tid);
    if (dbg && tid == 0) { dbg[12] = global_ns(); dbg[14] = clock64(); }
}

}  // namespace moe
