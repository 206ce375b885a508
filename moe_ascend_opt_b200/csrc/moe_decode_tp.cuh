// Two-pass decode kernels: the fused MoE layer for decode-size token counts as two short
// streaming kernels instead of one persistent kernel with phases.
//
//   pass 1 (tp_gate_up_kernel): grid (I/16 row tiles) x (pieces).  A CTA takes one row tile
//     (16 gate rows + the same 16 up rows) of one piece and computes
//     h[pair][rows] = SiLU(gate) * up for the piece's pairs, rounded to the activation type
//     (q8_gemm.cpp:421-463 for the SiLU product; AWQ GEMM path for the rounding).
//   pass 2 (tp_down_kernel): grid (H/32 row blocks) x (pieces).  A CTA takes one 32-row
//     block of one piece's down projection over the whole of I, scales the rows by the
//     routing weight of each pair and stores them as fp32 rows of `part` [pair][H].  The CTA
//     that completes a row block's arrival count sums the block's rows of each token's pairs
//     in k order (q8_gemm.cpp:593-613) and casts: the order does not depend on which CTA is
//     last, so the output is deterministic.
//
// A piece is one routed local expert with up to min(8, T) of its pairs (the 8 columns of one
// mma.sync m16n8k16); each expert's pairs are cut into pieces in pair order, experts in
// order of their first pair.  Every CTA routes the pairs itself (moe_common.cpp:146-184)
// with one warp; the grid has one piece slot per routed pair and CTAs of empty slots return
// at once, so the launch does not depend on the routing.
//
// Each warp of a CTA bulk-copies its share of the tile's weight records into shared memory
// at the start (two copies for pass 1, one for pass 2, cp.async.bulk without multicast, one
// mbarrier each, bounded waits), so that a wave of CTAs has the whole layer's weights in
// flight at once.  Both kernels are launched with programmatic dependent launch: pass 2
// routes and starts its weight copies (which do not depend on pass 1) before
// griddepcontrol.wait, then reads h; each kernel releases its dependent only after its own
// wait, so that reads of the routing ids before a wait see the ids of this call.
//
// AWQ W4A16 records (laid out for mma.sync m16n8k16 at weight-load time):
//   gate_up [E][I/16][2][H/64] of 560 B: 16 rows x 32 B nibbles | 16 bf16 scales | 16 u8 zeros
//   down    [E][H/32][I/64]    of 1120 B: 32 rows x 32 B nibbles | 32 bf16 scales | 32 u8 zeros
// with the folded zero point s (D - (M + z) sum_k x_k) per 64 k (awq_mma64).
#pragma once
#include "moe_decode_cl.cuh"

namespace moe {

constexpr int kTpWarpsA = 8;  // pass 1 warps per CTA (the 64-k records of a row tile split 8 ways)
constexpr int kTpWarpsB = 4;  // pass 2 warps per CTA
constexpr int kTpCopiesA = 2;  // pass 1: bulk copies per half (gate / up) of a row tile
constexpr int kTpMaxPairs = 64;  // T * K of one launch
constexpr int kTpCols = 8;       // pairs per piece (mma n)

struct TpParams {
    const uint8_t* gu;  // AWQ gate_up records; Q8_0 / Q4_0 unit records [E][I] (gate row, up row, scales)
    const uint8_t* dn;  // AWQ down records; Q8_0 / Q4_0 down row-slice records [E][H/32][I/32]
    int32_t rs1, ss1;   // Q8_0 / Q4_0: quant and scale bytes of one row of a unit record
    int32_t scale_bf16, act_bf16;
    int32_t E, e_off, H, I, T, K;
    const int32_t* emap;  // global -> local expert map (expert parallel) or null
    int32_t emap_n;
    const void* x;          // tokens [T][H] (bf16 / fp16)
    void* y;                // output [T][H] (out_kind: 0 fp16, 1 bf16, 2 fp32)
    const int32_t* ids;     // [T][K] global expert ids
    const float* tw;        // [T][K] routing weights
    void* h;                // h between the passes [T K][I]: AWQ activation type, Q8_0 / Q4_0 fp32
    float* part;            // [T K][H] weighted fp32 down rows
    unsigned int* cnt;      // [H/32] arrival counters, zero between launches
    int32_t* err;           // sticky device error word (mapped host memory)
    int32_t out_kind, flags;
    int32_t ncol;           // pairs per piece: min(8, T) (more pieces when ids repeat in a token)
    unsigned long long* dbg;  // optional phase stamps (globaltimer ns) [CTA][20]: pass 1 in 0-9, pass 2 in 10-19
};

#define TP_STAMP(i)                                                                              \
    do {                                                                                         \
        if (p.dbg && threadIdx.x == 0)                                                           \
            p.dbg[(size_t)(blockIdx.y * gridDim.x + blockIdx.x) * kStamps + (i)] = global_ns(); \
    } while (0)

// Routing of one launch, computed by one warp of every CTA.
struct TpRoute {
    int32_t le[kTpMaxPairs];              // local expert of each pair, -1 when not this engine's
    int32_t pe[kTpMaxPairs];              // local expert of each piece
    int32_t pn[kTpMaxPairs];              // pairs (columns) of each piece
    int32_t pc[kTpMaxPairs][kTpCols];     // pair of each column
    int32_t P;                            // pieces
};

// The routing ids are read through L2 (ld.global.cg): pass 2 reads them before its
// griddepcontrol.wait, while pass 1 still runs.
MOE_DEV void tp_route(const TpParams& p, TpRoute& r, int lane) {
    const int TK = p.T * p.K;
    // lane holds pairs lane and lane + 32; every comparison below is a register shuffle
    int v[2];
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
        const int j = lane + 32 * jj;
        v[jj] = j < TK ? local_expert(__ldcg(p.ids + j), p.e_off, p.E, p.emap, p.emap_n, j, p.K) : -1;
        if (j < TK) r.le[j] = v[jj];
    }
    if (p.ncol == 1) {  // one token: every valid pair is a piece of its own, in pair order
        const unsigned b0 = __ballot_sync(0xffffffffu, v[0] >= 0), b1 = __ballot_sync(0xffffffffu, v[1] >= 0);
        const unsigned lt1 = (1u << lane) - 1u;
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            if (v[jj] < 0) continue;
            const int pc = jj ? __popc(b0) + __popc(b1 & lt1) : __popc(b0 & lt1);
            r.pc[pc][0] = lane + 32 * jj;
            r.pe[pc] = v[jj];
            r.pn[pc] = 1;
        }
        if (lane == 0) r.P = __popc(b0) + __popc(b1);
        __syncwarp();
        return;
    }
    // per pair: pairs of the same expert before it (rank), in all (cnt), and the first of them;
    // within a half of 32 pairs by match.any, across the halves (T K > 32) by shuffles
    const unsigned lt = (1u << lane) - 1u;
    int rank[2], cnt[2], first[2];
    {
        const unsigned m0 = __match_any_sync(0xffffffffu, v[0]);
        rank[0] = __popc(m0 & lt); cnt[0] = __popc(m0); first[0] = __ffs(m0) - 1;
        rank[1] = 0; cnt[1] = 0; first[1] = lane + 32;
    }
    if (TK > 32) {
        const unsigned m1 = __match_any_sync(0xffffffffu, v[1]);
        unsigned x01 = 0u, x10 = 0u;  // lanes whose first-half pair equals my second, and vice versa
#pragma unroll 8
        for (int l = 0; l < 32; ++l) {
            x10 |= (unsigned)(__shfl_sync(0xffffffffu, v[0], l) == v[1]) << l;
            x01 |= (unsigned)(__shfl_sync(0xffffffffu, v[1], l) == v[0]) << l;
        }
        cnt[0] += __popc(x01);
        rank[1] = __popc(x10) + __popc(m1 & lt);
        cnt[1] = __popc(x10) + __popc(m1);
        first[1] = x10 ? __ffs(x10) - 1 : __ffs(m1) - 1 + 32;
    }
    int npc[2];
#pragma unroll
    for (int jj = 0; jj < 2; ++jj)  // pieces of the expert, counted at its first pair
        npc[jj] = (v[jj] >= 0 && rank[jj] == 0) ? (cnt[jj] + p.ncol - 1) / p.ncol : 0;
    // first piece of each expert: exclusive scan of npc over pairs 0..31, then 32..63
    int base = 0, ps[2];
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
        int incl = npc[jj];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        ps[jj] = base + incl - npc[jj];
        base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) r.P = base;
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {  // the first pair's piece start, from its lane
        const int f = first[jj];
        const int s0 = __shfl_sync(0xffffffffu, ps[0], f & 31), s1 = __shfl_sync(0xffffffffu, ps[1], f & 31);
        if (v[jj] >= 0) {
            const int pc = (f < 32 ? s0 : s1) + rank[jj] / p.ncol, col = rank[jj] % p.ncol;
            r.pc[pc][col] = lane + 32 * jj;
            if (col == 0) {
                r.pe[pc] = v[jj];
                r.pn[pc] = min(p.ncol, cnt[jj] - rank[jj]);  // pairs of the expert from this one on
            }
        }
    }
    __syncwarp();
}

// Wait for the stream predecessor (programmatic dependent launch): one warp waits while the
// others sleep in the CTA barrier (a waiting warp takes issue slots from the warps of other
// CTAs on the SM), then every thread passes its own wait at once.
MOE_DEV void tp_dep_wait(int warp) {
    if (warp == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
    __syncthreads();
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

MOE_DEV void tp_wait(const TpParams& p, uint64_t* bar) {
    if (!mbar_wait(bar, 0u)) {
        set_err(p.err, kErrFullWait);
        mbar_wait(bar, 0u);  // a second bounded wait for the copy before the CTA goes on
    }
}

// Pass 1: gate_up + SiLU * up of one 16-row tile of one piece.
template <bool XBF>
__global__ void __launch_bounds__(kTpWarpsA * 32) tp_gate_up_kernel(const TpParams p) {
    constexpr int kThreads = kTpWarpsA * 32;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ TpRoute rt;
    __shared__ __align__(8) uint64_t bars[2 * kTpWarpsA];
    __shared__ float red[kTpWarpsA][2][16][kTpCols];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = p.H, I = p.I, NK1 = H / kAwqK;
    const int tile = blockIdx.x, slot = blockIdx.y;
    TP_STAMP(0);
    // L2 policy of the weight copies, made before the dependency wait (off the critical path)
    const uint64_t pol = (lane == 0 && (p.flags & kFlagEvictFirst)) ? l2_evict_first_policy() : 0ull;
    if (tid < 2 * kTpWarpsA) mbar_init(&bars[tid], 1);
    fence_barrier_init();
    tp_dep_wait(warp);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    TP_STAMP(1);
    // warp 0 routes while the others stage the T token rows [T][H + 8] and their per-64 sums
    // [T][NK1]; eight neighbouring threads hold one 64-run (stride and trip count are
    // multiples of 8)
    uint16_t* xs = reinterpret_cast<uint16_t*>(smem + (size_t)2 * NK1 * kAwqGuRec);
    float* xsum = reinterpret_cast<float*>(xs + (size_t)p.T * (H + 8));
    if (warp == 0) {
        tp_route(p, rt, lane);
    } else {
        const uint16_t* xg = static_cast<const uint16_t*>(p.x);
        #pragma unroll 1
        for (int i = tid - 32; i < p.T * (H / 8); i += kThreads - 32) {
            const int t = i / (H / 8), k8 = i - t * (H / 8);
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(xg + (size_t)t * H) + k8);
            *reinterpret_cast<uint4*>(xs + (size_t)t * (H + 8) + 8 * k8) = v;
            const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
            float sv = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                sv += from16<XBF>((uint16_t)(w4[j] & 0xffffu)) + from16<XBF>((uint16_t)(w4[j] >> 16));
            const unsigned am = __activemask();  // whole 8-thread runs are active or not
            sv += __shfl_xor_sync(am, sv, 1);
            sv += __shfl_xor_sync(am, sv, 2);
            sv += __shfl_xor_sync(am, sv, 4);
            if ((k8 & 7) == 0) xsum[t * NK1 + (k8 >> 3)] = sv;
        }
    }
    __syncthreads();
    TP_STAMP(2);
    if (slot >= rt.P) return;
    const int e = rt.pe[slot], nc = rt.pn[slot];

    // the tile's gate records [0, NK1) then its up records in shared memory, each half in
    // kTpCopiesA bulk copies issued by as many warps; warp w computes records [k0, k0 + nk)
    uint8_t* wg = smem;
    uint8_t* wu = smem + (size_t)NK1 * kAwqGuRec;
    if (lane == 0 && warp < 2 * kTpCopiesA) {
        const int half = warp / kTpCopiesA, i = warp % kTpCopiesA;
        const int r0 = i * NK1 / kTpCopiesA, n = (i + 1) * NK1 / kTpCopiesA - r0;
        const size_t rec0 = (((size_t)e * (I / 16) + tile) * 2 + half) * NK1 + r0;
        if (n > 0)
            issue_copy((half ? wu : wg) + (size_t)r0 * kAwqGuRec, p.gu + rec0 * kAwqGuRec, (uint32_t)n * kAwqGuRec,
                       &bars[warp], pol);
        else
            mbar_arrive(&bars[warp]);
    }
    const int k0 = warp * NK1 / kTpWarpsA, nk = (warp + 1) * NK1 / kTpWarpsA - k0;
    // copies holding this warp's first and last record (ranges nest: kTpCopiesA divides the warps)
    const int cp0 = k0 * kTpCopiesA / NK1, cp1 = nk > 0 ? (k0 + nk - 1) * kTpCopiesA / NK1 : cp0;
    TP_STAMP(3);

    const int g = lane >> 2, c = lane & 3;  // mma column g: B rows; columns 2c, 2c+1: x sums
    const uint16_t* brow = g < nc ? xs + (size_t)(rt.pc[slot][g] / p.K) * (H + 8) : nullptr;
    const int c0 = rt.pc[slot][min(2 * c, nc - 1)] / p.K, c1 = rt.pc[slot][min(2 * c + 1, nc - 1)] / p.K;
    float tg[4] = {0.f, 0.f, 0.f, 0.f}, tu[4] = {0.f, 0.f, 0.f, 0.f};
    if (nk > 0) {
        for (int cp = cp0; cp <= cp1; ++cp) {
            tp_wait(p, &bars[cp]);
            tp_wait(p, &bars[kTpCopiesA + cp]);
        }
        TP_STAMP(5);
        #pragma unroll 1
        for (int r = 0; r < nk; ++r) {  // gate and up records side by side: two independent chains
            const int kh = k0 + r;
            const uint8_t* rg = wg + (size_t)kh * kAwqGuRec;
            const uint8_t* ru = wu + (size_t)kh * kAwqGuRec;
            const uint16_t* b = brow ? brow + kh * kAwqK : nullptr;
            const float s0 = xsum[c0 * NK1 + kh], s1 = xsum[c1 * NK1 + kh];
            awq_mma64<XBF>(rg, reinterpret_cast<const uint16_t*>(rg + 512), rg + 544, b, s0, s1, lane, tg);
            awq_mma64<XBF>(ru, reinterpret_cast<const uint16_t*>(ru + 512), ru + 544, b, s0, s1, lane, tu);
        }
    }
    TP_STAMP(6);
    red[warp][0][g][2 * c] = tg[0];
    red[warp][0][g][2 * c + 1] = tg[1];
    red[warp][0][g + 8][2 * c] = tg[2];
    red[warp][0][g + 8][2 * c + 1] = tg[3];
    red[warp][1][g][2 * c] = tu[0];
    red[warp][1][g][2 * c + 1] = tu[1];
    red[warp][1][g + 8][2 * c] = tu[2];
    red[warp][1][g + 8][2 * c + 1] = tu[3];
    __syncthreads();
    {
        const int r = tid & 15, n = tid >> 4;  // 16 rows x 8 columns, one per thread
        if (n < nc) {
            float ga = 0.f, ua = 0.f;
#pragma unroll
            for (int w = 0; w < kTpWarpsA; ++w) {
                ga += red[w][0][r][n];
                ua += red[w][1][r][n];
            }
            const float hv = silu_mul(ga, ua);
            if (!XBF && !(fabsf(hv) <= 65504.f)) set_err(p.err, kErrRange);
            static_cast<uint16_t*>(p.h)[(size_t)rt.pc[slot][n] * I + tile * 16 + r] = to16<XBF>(hv);
        }
    }
    TP_STAMP(7);
}

// Pass 2: down projection of one 32-row block of one piece, weighted rows into `part`, and
// the combine of the row block by its last CTA.
template <bool XBF>
__global__ void __launch_bounds__(kTpWarpsB * 32) tp_down_kernel(const TpParams p) {
    constexpr int kThreads = kTpWarpsB * 32;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ TpRoute rt;
    __shared__ __align__(8) uint64_t bars[kTpWarpsB];
    __shared__ float red[kTpWarpsB][32][kTpCols];
    __shared__ unsigned int s_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = p.H, I = p.I, NKD = I / kAwqK, T = p.T, K = p.K;
    const int rb = blockIdx.x, slot = blockIdx.y;
    TP_STAMP(10);
    const uint64_t pol = (lane == 0 && (p.flags & kFlagEvictFirst)) ? l2_evict_first_policy() : 0ull;
    if (tid < kTpWarpsB) mbar_init(&bars[tid], 1);
    fence_barrier_init();
    if (warp == 0) tp_route(p, rt, lane);
    __syncthreads();
    TP_STAMP(11);
    const int P = rt.P;
    if (P == 0) {  // no routed pair on this engine: the output is zero (q8_gemm.cpp:328-333)
        tp_dep_wait(warp);
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        if (slot == 0)
            #pragma unroll 1
            for (int i = tid; i < T * 32; i += kThreads) {
                const size_t o = (size_t)(i >> 5) * H + rb * 32 + (i & 31);
                if (p.out_kind == 2) reinterpret_cast<float*>(p.y)[o] = 0.f;
                else if (p.out_kind == 1) reinterpret_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(0.f);
                else reinterpret_cast<__half*>(p.y)[o] = __float2half_rn(0.f);
            }
        return;
    }
    if (slot >= P) {
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        return;
    }
    const int e = rt.pe[slot], nc = rt.pn[slot];

    // this warp's records [k0, k1) of the row block (contiguous ranges, the CTA's copy regions
    // back to back): weights do not depend on pass 1
    const int k0 = warp * NKD / kTpWarpsB, nk = (warp + 1) * NKD / kTpWarpsB - k0;
    uint8_t* wd = smem + (size_t)k0 * kAwqDnRec;
    if (lane == 0 && nk > 0) {
        const size_t rec0 = ((size_t)e * (H / 32) + rb) * NKD + k0;
        issue_copy(wd, p.dn + rec0 * kAwqDnRec, (uint32_t)nk * kAwqDnRec, &bars[warp], pol);
    }
    TP_STAMP(12);
    const int g = lane >> 2, c = lane & 3;
    if (nk > 0) tp_wait(p, &bars[warp]);  // the records arrive while pass 1 still runs
    TP_STAMP(15);
    tp_dep_wait(warp);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    TP_STAMP(13);

    // h of the piece's pairs [nc][I + 8] and its per-64 sums [nc][NKD]
    uint16_t* hs = reinterpret_cast<uint16_t*>(smem + (size_t)NKD * kAwqDnRec);
    float* hsum = reinterpret_cast<float*>(hs + (size_t)p.ncol * (I + 8));
    #pragma unroll 1
    for (int i = tid; i < nc * (I / 8); i += kThreads) {
        const int n = i / (I / 8), k8 = i - n * (I / 8);
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.h) + (size_t)rt.pc[slot][n] * I) + k8);
        *reinterpret_cast<uint4*>(hs + (size_t)n * (I + 8) + 8 * k8) = v;
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
        float sv = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            sv += from16<XBF>((uint16_t)(w4[j] & 0xffffu)) + from16<XBF>((uint16_t)(w4[j] >> 16));
        const unsigned am = __activemask();  // whole 8-thread runs are active or not
        sv += __shfl_xor_sync(am, sv, 1);
        sv += __shfl_xor_sync(am, sv, 2);
        sv += __shfl_xor_sync(am, sv, 4);
        if ((k8 & 7) == 0) hsum[n * NKD + (k8 >> 3)] = sv;
    }
    __syncthreads();
    TP_STAMP(14);

    const uint16_t* hrow = g < nc ? hs + (size_t)g * (I + 8) : nullptr;
    const int c0 = min(2 * c, nc - 1), c1 = min(2 * c + 1, nc - 1);
    float tot[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    #pragma unroll 1
    for (int r = 0; r < nk; ++r) {
        const uint8_t* rec = wd + (size_t)r * kAwqDnRec;
        const int kh = k0 + r;
        const float x0 = hsum[c0 * NKD + kh], x1 = hsum[c1 * NKD + kh];
#pragma unroll
        for (int tt = 0; tt < 2; ++tt)
            awq_mma64<XBF>(rec + tt * 512, reinterpret_cast<const uint16_t*>(rec + 1024) + 16 * tt,
                           rec + 1088 + 16 * tt, hrow ? hrow + kh * kAwqK : nullptr, x0, x1, lane, tot[tt]);
    }
    TP_STAMP(16);
#pragma unroll
    for (int tt = 0; tt < 2; ++tt) {
        red[warp][16 * tt + g][2 * c] = tot[tt][0];
        red[warp][16 * tt + g][2 * c + 1] = tot[tt][1];
        red[warp][16 * tt + g + 8][2 * c] = tot[tt][2];
        red[warp][16 * tt + g + 8][2 * c + 1] = tot[tt][3];
    }
    __syncthreads();
    {
        const int r = tid & 31;
#pragma unroll
        for (int n = tid >> 5; n < kTpCols; n += kTpWarpsB) {
            if (n >= nc) continue;
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kTpWarpsB; ++w) v += red[w][r][n];
            const int j = rt.pc[slot][n];
            p.part[(size_t)j * H + rb * 32 + r] = __ldg(p.tw + j) * v;
        }
    }
    __syncthreads();
    if (tid == 0) {  // release: the CTA's rows of `part`, ordered before by the barrier
        unsigned int old;
        asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(old) : "l"(p.cnt + rb) : "memory");
        s_last = old == (unsigned int)(P - 1);
        if (s_last) p.cnt[rb] = 0u;  // reset for the next launch (no CTA of this one adds again)
    }
    __syncthreads();
    TP_STAMP(17);
    if (!s_last) return;
    // the row block's combine: every pair's rows are in `part` (acquire above)
    #pragma unroll 1
    for (int i = tid; i < T * 32; i += kThreads) {
        const int t = i >> 5, row = rb * 32 + (i & 31);
        float acc = 0.f;
        #pragma unroll 1
        for (int k0 = 0; k0 < K; k0 += 8) {  // eight loads in flight, summed in k order
            float v8[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int j = t * K + k0 + k;
                v8[k] = (k0 + k < K && rt.le[j] >= 0) ? __ldcg(p.part + (size_t)j * H + row) : 0.f;
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) acc += v8[k];
        }
        const size_t o = (size_t)t * H + row;
        if (p.out_kind == 2) reinterpret_cast<float*>(p.y)[o] = acc;
        else if (p.out_kind == 1) reinterpret_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(acc);
        else reinterpret_cast<__half*>(p.y)[o] = __float2half_rn(acc);
    }
    TP_STAMP(18);
}

// ------------------------------------------------------------------ Q8_0 / Q4_0
// The same two passes on the reference's 32-block formats: exact per-32-block integer dots
// (dp4a) folded with the fp32 scales as gemm_kernels.cpp:66-186 does; the token rows
// quantised to Q8_0 (gemm_kernels.cpp:25-58) by every pass-1 CTA, h kept in fp32 between the
// passes and requantised by every pass-2 CTA for its piece (gemm_kernels.cpp:394-425).
constexpr int kTpUnitsQ = 16;  // pass 1 (Q8/Q4): gate_up units per CTA, two per warp
constexpr int kTpCopiesQ = 4;  // its bulk copies
constexpr int kTpWarpsBQ = 4;  // pass 2 (Q8/Q4) warps per CTA

// The row block's combine by the CTA that completes its arrival count (see the file header).
MOE_DEV void tp_arrive_combine(const TpParams& p, const TpRoute& rt, int rb, int tid, int nthreads,
                               unsigned int* s_last) {
    __syncthreads();
    if (tid == 0) {  // release: the CTA's rows of `part`, ordered before by the barrier
        unsigned int old;
        asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(old) : "l"(p.cnt + rb) : "memory");
        *s_last = old == (unsigned int)(rt.P - 1);
        if (*s_last) p.cnt[rb] = 0u;
    }
    __syncthreads();
    if (!*s_last) return;
    const int H = p.H, K = p.K;
    #pragma unroll 1
    for (int i = tid; i < p.T * 32; i += nthreads) {
        const int t = i >> 5, row = rb * 32 + (i & 31);
        float acc = 0.f;
        #pragma unroll 1
        for (int k0 = 0; k0 < K; k0 += 8) {
            float v8[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int j = t * K + k0 + k;
                v8[k] = (k0 + k < K && rt.le[j] >= 0) ? __ldcg(p.part + (size_t)j * H + row) : 0.f;
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) acc += v8[k];
        }
        const size_t o = (size_t)t * H + row;
        if (p.out_kind == 2) reinterpret_cast<float*>(p.y)[o] = acc;
        else if (p.out_kind == 1) reinterpret_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(acc);
        else reinterpret_cast<__half*>(p.y)[o] = __float2half_rn(acc);
    }
}

// Pass 1 (Q8/Q4): gate_up + SiLU * up of kTpUnitsQ units of one piece -> fp32 h.
template <bool Q4>
__global__ void __launch_bounds__(kTpWarpsA * 32) tp_gate_up_q_kernel(const TpParams p) {
    constexpr int kThreads = kTpWarpsA * 32;
    constexpr int BB = Q4 ? 16 : 32;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ TpRoute rt;
    __shared__ __align__(8) uint64_t bars[kTpCopiesQ];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = p.H, I = p.I, nb1 = H >> 5;
    const int ub = 2 * (p.rs1 + p.ss1);
    const int tile = blockIdx.x, slot = blockIdx.y;
    TP_STAMP(0);
    // L2 policy of the weight copies, made before the dependency wait (off the critical path)
    const uint64_t pol = (lane == 0 && (p.flags & kFlagEvictFirst)) ? l2_evict_first_policy() : 0ull;
    if (tid < kTpCopiesQ) mbar_init(&bars[tid], 1);
    fence_barrier_init();
    tp_dep_wait(warp);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    TP_STAMP(1);
    // warp 0 routes while the others quantise the T token rows (Q8_0, a quad per 32-block)
    int8_t* xq = reinterpret_cast<int8_t*>(smem + (size_t)kTpUnitsQ * ub);
    float* xd = reinterpret_cast<float*>(xq + (size_t)p.T * H);
    int32_t* xsm = reinterpret_cast<int32_t*>(xd + (size_t)p.T * nb1);
    if (warp == 0) tp_route(p, rt, lane);
    else quant_x_quad<Q4>(static_cast<const uint8_t*>(p.x), p.act_bf16, p.T, H, xq, xd, xsm, tid - 32, kThreads - 32);
    __syncthreads();
    TP_STAMP(2);
    if (slot >= rt.P) return;
    const int e = rt.pe[slot], nc = rt.pn[slot];
    const int u0 = tile * kTpUnitsQ, nu = min(kTpUnitsQ, I - u0);
    if (lane == 0 && warp < kTpCopiesQ) {
        const int a = warp * nu / kTpCopiesQ, n = (warp + 1) * nu / kTpCopiesQ - a;
        if (n > 0)
            issue_copy(smem + (size_t)a * ub, p.gu + ((size_t)e * I + u0 + a) * ub, (uint32_t)n * ub, &bars[warp], pol);
        else
            mbar_arrive(&bars[warp]);
    }
    TP_STAMP(3);
    const bool sbf = p.scale_bf16 != 0;
    #pragma unroll 1
    for (int uu = warp * kTpUnitsQ / kTpWarpsA; uu < (warp + 1) * kTpUnitsQ / kTpWarpsA; ++uu) {
        if (uu >= nu) break;
        tp_wait(p, &bars[uu * kTpCopiesQ / nu]);
        const uint8_t* rec = smem + (size_t)uu * ub;
        const uint8_t* qg = rec;
        const uint8_t* qu = rec + p.rs1;
        const uint16_t* sgate = reinterpret_cast<const uint16_t*>(rec + 2 * p.rs1);
        const uint16_t* sup = reinterpret_cast<const uint16_t*>(rec + 2 * p.rs1 + p.ss1);
        #pragma unroll 1
        for (int m = 0; m < nc; ++m) {  // one token at a time: small code, weights from smem
            const int t = rt.pc[slot][m] / p.K;
            const int8_t* xt = xq + (size_t)t * H;
            const float* xdt = xd + (size_t)t * nb1;
            const int32_t* xst = xsm + (size_t)t * nb1;
            float ag = 0.f, au = 0.f;
#pragma unroll 2
            for (int b = lane; b < nb1; b += 32) {
                const uint4* wg = reinterpret_cast<const uint4*>(qg + (size_t)b * BB);
                const uint4* wu4 = reinterpret_cast<const uint4*>(qu + (size_t)b * BB);
                const uint4* a = reinterpret_cast<const uint4*>(xt + b * 32);
                const float ad = xdt[b];
                const int as = Q4 ? xst[b] : 0;
                ag += ((float)block_dot<Q4>(wg, a, as) * scale_to_f32(sgate[b], sbf)) * ad;
                au += ((float)block_dot<Q4>(wu4, a, as) * scale_to_f32(sup[b], sbf)) * ad;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                ag += __shfl_xor_sync(0xffffffffu, ag, o);
                au += __shfl_xor_sync(0xffffffffu, au, o);
            }
            if (lane == 0) static_cast<float*>(p.h)[(size_t)rt.pc[slot][m] * I + u0 + uu] = silu_mul(ag, au);
        }
    }
    TP_STAMP(7);
}

// Pass 2 (Q8/Q4): down rows of one 32-row block of one piece (lane = row of the block's
// row-slice records), weighted into `part`, and the row block's combine.
template <bool Q4>
__global__ void __launch_bounds__(kTpWarpsBQ * 32) tp_down_q_kernel(const TpParams p) {
    constexpr int kThreads = kTpWarpsBQ * 32;
    constexpr int BB = Q4 ? 16 : 32;
    constexpr int SB = 32 * BB + 64;  // row-slice record: 32 rows x one 32-column block, 32 scales
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ TpRoute rt;
    __shared__ __align__(8) uint64_t bars[kTpWarpsBQ];
    __shared__ float red[kTpWarpsBQ][32][kTpCols];
    __shared__ unsigned int s_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = p.H, I = p.I, KB = I >> 5, T = p.T;
    const int rb = blockIdx.x, slot = blockIdx.y;
    TP_STAMP(10);
    const uint64_t pol = (lane == 0 && (p.flags & kFlagEvictFirst)) ? l2_evict_first_policy() : 0ull;
    if (tid < kTpWarpsBQ) mbar_init(&bars[tid], 1);
    fence_barrier_init();
    if (warp == 0) tp_route(p, rt, lane);
    __syncthreads();
    TP_STAMP(11);
    const int P = rt.P;
    if (P == 0) {  // no routed pair on this engine: the output is zero (q8_gemm.cpp:328-333)
        tp_dep_wait(warp);
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        if (slot == 0)
            #pragma unroll 1
            for (int i = tid; i < T * 32; i += kThreads) {
                const size_t o = (size_t)(i >> 5) * H + rb * 32 + (i & 31);
                if (p.out_kind == 2) reinterpret_cast<float*>(p.y)[o] = 0.f;
                else if (p.out_kind == 1) reinterpret_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(0.f);
                else reinterpret_cast<__half*>(p.y)[o] = __float2half_rn(0.f);
            }
        return;
    }
    if (slot >= P) {
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        return;
    }
    const int e = rt.pe[slot], nc = rt.pn[slot];
    const int b0 = warp * KB / kTpWarpsBQ, nbw = (warp + 1) * KB / kTpWarpsBQ - b0;
    uint8_t* wd = smem + (size_t)b0 * SB;
    if (lane == 0 && nbw > 0) {
        issue_copy(wd, p.dn + (((size_t)e * (H / 32) + rb) * KB + b0) * SB, (uint32_t)nbw * SB, &bars[warp], pol);
    }
    TP_STAMP(12);
    if (nbw > 0) tp_wait(p, &bars[warp]);  // the records arrive while pass 1 still runs
    TP_STAMP(15);
    tp_dep_wait(warp);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    TP_STAMP(13);
    // the piece's h rows requantised to Q8_0 [nc][I] | d [nc][KB] | sums [nc][KB], a quad per block
    int8_t* hq = reinterpret_cast<int8_t*>(smem + (size_t)KB * SB);
    float* hd = reinterpret_cast<float*>(hq + (size_t)p.ncol * I);
    int32_t* hs = reinterpret_cast<int32_t*>(hd + (size_t)p.ncol * KB);
    {
        const int sub = tid & 3;
        const uint32_t qm = quad_mask(lane);
        #pragma unroll 1
        for (int g = tid >> 2; g < nc * KB; g += kThreads / 4) {
            const int m = g / KB, b = g - m * KB;
            float v[8];
            load8(static_cast<const float*>(p.h) + (size_t)rt.pc[slot][m] * I + b * 32 + sub * 8, v);
            float dd;
            int sum;
            uint2 o;
            quad_quant<Q4>(v, qm, dd, sum, o);
            *reinterpret_cast<uint2*>(hq + (size_t)g * 32 + sub * 8) = o;
            if (sub == 0) {
                hd[g] = dd;
                if (Q4) hs[g] = sum;
            }
        }
    }
    __syncthreads();
    TP_STAMP(14);
    const bool sbf = p.scale_bf16 != 0;
    float acc[kTpCols];
#pragma unroll
    for (int m = 0; m < kTpCols; ++m) acc[m] = 0.f;
    #pragma unroll 2
    for (int r = 0; r < nbw; ++r) {
        const int b = b0 + r;
        const uint8_t* rec = wd + (size_t)r * SB;
        const uint4* w = reinterpret_cast<const uint4*>(rec + lane * BB);
        const float dw = scale_to_f32(reinterpret_cast<const uint16_t*>(rec + 32 * BB)[lane], sbf);
#pragma unroll
        for (int m = 0; m < kTpCols; ++m) {
            if (m >= nc) break;
            const uint4* a = reinterpret_cast<const uint4*>(hq + (size_t)m * I + b * 32);
            const int is = block_dot<Q4>(w, a, Q4 ? hs[m * KB + b] : 0);
            acc[m] += ((float)is * dw) * hd[m * KB + b];
        }
    }
    TP_STAMP(16);
#pragma unroll
    for (int m = 0; m < kTpCols; ++m) red[warp][lane][m] = acc[m];
    __syncthreads();
    {
        const int r = tid & 31;
#pragma unroll
        for (int n = tid >> 5; n < kTpCols; n += kTpWarpsBQ) {
            if (n >= nc) continue;
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kTpWarpsBQ; ++w) v += red[w][r][n];
            const int j = rt.pc[slot][n];
            p.part[(size_t)j * H + rb * 32 + r] = __ldg(p.tw + j) * v;
        }
    }
    tp_arrive_combine(p, rt, rb, tid, kThreads, &s_last);
    TP_STAMP(17);
}

}  // namespace moe
