// Grouped-GEMM path of the fused MoE layer for large token counts (Q8_0 / Q4_0).
//
// Per launch sequence (all stream ordered):
//   route_count / route_scan / route_place  parallel stable counting sort of the
//        T*K pairs by expert (moe_common.cpp:146-184): counts, starts, positions in
//        (t,k) order, plus per-expert tile offsets for the GEMMs;
//   quant_rows (gemm_kernels.cpp:25-58)     token rows -> Q8_0, in the byte order that
//        matches the weight's nibble order inside one MMA (act_elem);
//   gemm_gate_up                            per (expert, 64-token tile, 64-unit tile):
//        C = A x W^T over the expert's gathered token rows with int8 tensor-core
//        MMAs, one MMA per 32-block and the reference's per-block fold
//        c += (f32(isum) * d_w) * d_a in fp32 registers; epilogue SiLU(gate)*up and
//        the Q8_0 requant of h per 32-unit block (pack_A_q8_0, gemm_kernels.cpp:394-425)
//        -- the tile holds whole blocks, so no cross-CTA step;
//   gemm_down                               out[pos][n] = h_q[pos] . W2[n] (fp32);
//   combine                                 y[t] = sum_k w[t,k] out[pos(t,k)] in k
//        order (q8_gemm.cpp:593-613), cast (q8_gemm.cpp:636-639).
// Tensor-core instruction: mma.sync m16n8k32 (s8 x s8, or s8 x u8 for Q4_0 nibbles
// with the -8 bias removed through the activation block sums).  A 32-block of K is
// exactly one MMA, so the per-block integer dot needs no extra work.
#pragma once
#include "common.cuh"

namespace moe {
namespace gemm {

constexpr int kBM = 64;        // token rows per CTA tile (largest variant; 32 and 16 for few tokens per expert)
constexpr int kBN = 128;       // weight rows per CTA tile (gate_up: 64 units x 2 rows)
constexpr int kKB = 4;         // 32-blocks per pipeline stage (K = 128)
constexpr int kStages = 3;
constexpr int kThreads = 256;  // 8 warps: BM 64: 2 (M) x 4 (N) of 32 x 32; BM 32: 1 x 8 of 32 x 16; BM 16: 1 x 8 of 16 x 16
constexpr int kRowPad = 16;    // smem row padding (bank-conflict-free fragment loads)

// ------------------------------------------------------------------ routing
// Pairs are processed in chunks of kChunk by one CTA each.
constexpr int kChunk = 1024;

__global__ void route_count_kernel(const int32_t* ids, int TK, int K, int E, int e_off, const int32_t* emap,
                                   int emap_n, int32_t* blk_cnt) {
    extern __shared__ int32_t sh[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) sh[e] = 0;
    __syncthreads();
    const int base = blockIdx.x * kChunk;
    for (int i = threadIdx.x; i < kChunk && base + i < TK; i += blockDim.x) {
        const int g = local_expert(ids[base + i], e_off, E, emap, emap_n, base + i, K);
        if (g >= 0) atomicAdd(&sh[g], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) blk_cnt[(size_t)blockIdx.x * E + e] = sh[e];
}

// One CTA of >= E threads: per-block offsets (expert-major), counts, starts, and
// per-expert first tile index of the gate_up / down GEMM tile lists.
__global__ void route_scan_kernel(int32_t* blk_cnt, int nblk, int E, int32_t* counts, int32_t* starts,
                                  int32_t* mtile_start, int bm) {
    extern __shared__ int32_t sh[];  // [2][E]
    const int e = threadIdx.x;
    int tot = 0;
    if (e < E) {
        for (int b = 0; b < nblk; ++b) {
            const int c = blk_cnt[(size_t)b * E + e];
            blk_cnt[(size_t)b * E + e] = tot;  // exclusive offset of block b within expert e
            tot += c;
        }
        sh[e] = tot;
        sh[E + e] = (tot + bm - 1) / bm;
    }
    __syncthreads();
    if (e == 0) {  // serial scan over experts (E <= a few hundred)
        int run = 0, trun = 0;
        for (int k = 0; k < E; ++k) {
            const int c = sh[k], t = sh[E + k];
            counts[k] = c;
            starts[k] = run;
            mtile_start[k] = trun;
            run += c;
            trun += t;
        }
        starts[E] = run;
        mtile_start[E] = trun;
    }
}

// Stable positions: warp 0 walks the chunk 32 pairs at a time in (t,k) order.
__global__ void route_place_kernel(const int32_t* ids, int TK, int K, int E, int e_off, const int32_t* emap, int emap_n,
                                   const int32_t* blk_off,
                                   const int32_t* starts, int32_t* smap, int32_t* tokmap) {
    extern __shared__ int32_t run[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) run[e] = starts[e] + blk_off[(size_t)blockIdx.x * E + e];
    __syncthreads();
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    const int base = blockIdx.x * kChunk;
    for (int i0 = 0; i0 < kChunk && base + i0 < TK; i0 += 32) {
        const int i = base + i0 + lane;
        int e = -1;
        if (i < TK) {
            e = local_expert(ids[i], e_off, E, emap, emap_n, i, K);
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        int b = 0;
        if (e >= 0) b = run[e];
        __syncwarp();
        if (i < TK) {
            const int pos = e >= 0 ? b + rank : -1;
            smap[i] = pos;
            if (pos >= 0) tokmap[pos] = i;
        }
        if (e >= 0 && rank == 0) run[e] = b + __popc(peers);
        __syncwarp();
    }
}

// Byte order of a Q8_0 activation block on the GEMM path.  Q8_0: natural.  Q4_0
// ("split" order): word w < 4 holds elements 8w+{0,2,4,6}, word 4+w holds 8w+{1,3,5,7},
// so that MMA k positions 4w..4w+3 meet the low nibbles of weight word w and positions
// 16+4w.. its high nibbles (weight word w = elements 8w..8w+7, nibble order).
template <bool Q4>
MOE_DEV int act_elem(int word, int byte) {
    return Q4 ? (word < 4 ? 8 * word + 2 * byte : 8 * (word - 4) + 2 * byte + 1) : 4 * word + byte;
}

// Token rows -> Q8_0 (thread per 32-block), bytes in the GEMM path's order (act_elem).
template <bool Q4>
__global__ void quant_rows_kernel(const uint8_t* x, int act_bf16, int rows, int cols, int8_t* q, float* d,
                                  int32_t* s) {
    const int nblk = rows * (cols >> 5);
    for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < nblk; g += gridDim.x * blockDim.x) {
        const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)g * 64);
        float v[32];
        float amax = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 r = __ldg(src + k);
            const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[8 * k + 2 * i] = scale_to_f32((uint16_t)(w4[i] & 0xffffu), act_bf16);
                v[8 * k + 2 * i + 1] = scale_to_f32((uint16_t)(w4[i] >> 16), act_bf16);
            }
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) amax = fmaxf(amax, fabsf(v[e]));
        const float dd = q8_scale(amax);
        const float id = q8_inv(dd);
        int qv[32];
        int sum = 0;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            qv[e] = q8_quant(v[e], id);
            sum += qv[e];
        }
        uint32_t wv[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            uint32_t w = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) w |= (uint32_t)(qv[act_elem<Q4>(k, i)] & 0xff) << (8 * i);
            wv[k] = w;
        }
        uint4* dst = reinterpret_cast<uint4*>(q + (size_t)g * 32);
        dst[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        dst[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
        d[g] = dd;
        if (Q4) s[g] = sum;
    }
}

// ------------------------------------------------------------------ MMA helpers
template <bool BU8>
MOE_DEV void mma_s8(int (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    if (BU8)
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%11,%12,%13};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(0), "r"(0), "r"(0), "r"(0));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%11,%12,%13};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(0), "r"(0), "r"(0), "r"(0));
}

// D = A x B + C with A the s8 activations and B the weights (u8 nibbles for Q4_0, s8 for Q8_0).
template <bool BU8>
MOE_DEV void mma_a8(int (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2], const int (&cin)[4]) {
    if (BU8)
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%11,%12,%13};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(cin[0]), "r"(cin[1]),
              "r"(cin[2]), "r"(cin[3]));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%11,%12,%13};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(cin[0]), "r"(cin[1]),
              "r"(cin[2]), "r"(cin[3]));
}

// D = A x B + C with A the weights (u8 nibbles for Q4_0, s8 for Q8_0) and B the s8 activations.
template <bool AU8>
MOE_DEV void mma_w(int (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2], const int (&cin)[4]) {
    if (AU8)
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%11,%12,%13};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(cin[0]), "r"(cin[1]),
              "r"(cin[2]), "r"(cin[3]));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%11,%12,%13};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(cin[0]), "r"(cin[1]),
              "r"(cin[2]), "r"(cin[3]));
}

// Four 8x8 b16 matrices from shared memory (lane l gives the address of row l&7 of matrix l>>3).
MOE_DEV void ldsm_x4(uint32_t (&r)[4], const void* row) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(row)));
}
MOE_DEV void ldsm_x2(uint32_t (&r)[2], const void* row) {  // lanes 0-15 give the row addresses
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(smem_u32(row)));
}
MOE_DEV float f4_get(const float4& v, int i) { return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w)); }
MOE_DEV int i4_get(const int4& v, int i) { return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w)); }

MOE_DEV void cp_async16(void* smem_dst, const void* gsrc, bool pred) {
    const uint32_t d = smem_u32(smem_dst);
    const int sz = pred ? 16 : 0;  // zero-fill when the source row does not exist
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(gsrc), "r"(sz) : "memory");
}
MOE_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
MOE_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ------------------------------------------------------------------ grouped GEMM
struct GemmParams {
    // A: quantised activation rows (gate_up: token rows [T][K], gathered through
    // tokmap/K; down: position rows [P][K]) with per-block scales (and Q4 sums)
    const int8_t* aq;
    const float* ad;
    const int32_t* as;
    // B: weight records; row n of expert e at wbase + (e*nrec + n/rows_per_rec)*rec + (n%rows_per_rec)*rs
    const uint8_t* wbase;
    int64_t rec;        // record bytes
    int rows_per_rec;   // gate_up: 2 (gate, up), down: 1
    int rs;             // bytes of one row's quants inside a record
    int sc_off;         // byte offset of the scale field of row 0 inside a record
    int ss;             // bytes of one row's scale field
    int nrec;           // records per expert (gate_up: I units, down: H rows)
    int K;              // reduction length (elements)
    int N;              // output columns per expert (gate_up: 2I, down: H)
    int scale_bf16;
    const int32_t* counts;
    const int32_t* starts;
    const int32_t* mtile_start;  // [E+1] first m-tile of each expert
    const int32_t* tokmap;       // gate_up: pair index per position (token = pair / topk)
    int topk;
    int E;
    // outputs
    int8_t* hq;   // gate_up: requantised h [P][I]
    float* hd;    // [P][I/32]
    int32_t* hs;  // [P][I/32] (Q4)
    float* out;   // down: [P][H]
};

// Shared-memory layout of one stage.
template <bool Q4, int BM>
struct Stage {
    static constexpr int kAKB = kKB * 32;               // activation bytes per row per stage
    static constexpr int kARow = kAKB + kRowPad;
    static constexpr int kBKB = kKB * (Q4 ? 16 : 32);  // weight bytes per row per stage
    static constexpr int kBRow = kBKB + kRowPad;
    static constexpr int kA = BM * kARow;
    static constexpr int kB = kBN * kBRow;
    static constexpr int kAd = BM * kKB * 4;
    static constexpr int kAs = BM * kKB * 4;
    static constexpr int kBd = kBN * kKB * 2;
    static constexpr int kBytes = kA + kB + kAd + kAs + kBd;
};

template <bool Q4, bool GATE_UP, int BM>
__global__ void __launch_bounds__(kThreads) grouped_gemm_kernel(const GemmParams p) {
    using S = Stage<Q4, BM>;
    constexpr int WNW = BM >= 64 ? 4 : 8;      // warps along N
    constexpr int WR = BM / (8 / WNW);         // warp tile rows
    constexpr int WC = kBN / WNW;              // warp tile cols
    constexpr int MI = WR / 16, NJ = WC / 8;   // m16 / n8 tiles per warp
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = warp / WNW, wn = warp % WNW;  // warp tile: rows wm*WR.., cols wn*WC..
    const int g = lane >> 2, c = lane & 3;

    // ---- tile -> (expert, m tile, n tile)
    const int ntiles_n = p.N / kBN;
    const int mt_total = p.mtile_start[p.E];
    const int tile = blockIdx.x;
    if (tile >= mt_total * ntiles_n) return;
    const int mt_glob = tile / ntiles_n, nt = tile % ntiles_n;
    int lo = 0, hi = p.E;  // expert e with mtile_start[e] <= mt_glob < mtile_start[e+1]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (p.mtile_start[mid] <= mt_glob) lo = mid;
        else hi = mid;
    }
    const int e = lo;
    const int m0 = (mt_glob - p.mtile_start[e]) * BM;
    const int cnt = p.counts[e];
    const int pos0 = p.starts[e] + m0;
    const int mrows = min(BM, cnt - m0);
    const int n0 = nt * kBN;
    const int nkb = p.K / 32;  // multiple of kKB (K % 128 == 0)

    // source rows of the tile's activations, resolved once (gathered through tokmap for gate_up)
    __shared__ int64_t s_arow[BM];
    for (int r = tid; r < BM; r += kThreads) {
        const int rr = min(r, max(mrows, 1) - 1);
        const int pos = pos0 + rr;
        s_arow[r] = GATE_UP ? (int64_t)(p.tokmap[pos] / p.topk) : (int64_t)pos;
    }
    __syncthreads();
    const uint8_t* wexp = p.wbase + (int64_t)e * p.nrec * p.rec;
    auto b_row_addr = [&](int n) -> const uint8_t* {
        const int gn = n0 + n;
        const int rec = gn / p.rows_per_rec, sub = gn - rec * p.rows_per_rec;
        return wexp + (int64_t)rec * p.rec + (int64_t)sub * p.rs;
    };
    auto b_scale_addr = [&](int n) -> const uint8_t* {
        const int gn = n0 + n;
        const int rec = gn / p.rows_per_rec, sub = gn - rec * p.rows_per_rec;
        return wexp + (int64_t)rec * p.rec + p.sc_off + (int64_t)sub * p.ss;
    };

    // every stage is loaded with cp.async only (quants 16 B, activation scales / sums
    // 16 B = 4 blocks, weight scales 8 B = 4 blocks); K is a multiple of 128.
    auto load_stage = [&](int st, int kb0) {
        uint8_t* base = smem + (size_t)st * S::kBytes;
        int8_t* sA = reinterpret_cast<int8_t*>(base);
        uint8_t* sB = base + S::kA;
        float* sAd = reinterpret_cast<float*>(base + S::kA + S::kB);
        int32_t* sAs = reinterpret_cast<int32_t*>(base + S::kA + S::kB + S::kAd);
        uint16_t* sBd = reinterpret_cast<uint16_t*>(base + S::kA + S::kB + S::kAd + S::kAs);
        for (int ch = tid; ch < BM * (S::kAKB / 16); ch += kThreads) {
            const int r = ch / (S::kAKB / 16), cc = ch % (S::kAKB / 16);
            cp_async16(sA + r * S::kARow + cc * 16, p.aq + s_arow[r] * p.K + (int64_t)kb0 * 32 + cc * 16, r < mrows);
        }
        for (int ch = tid; ch < kBN * (S::kBKB / 16); ch += kThreads) {
            const int n = ch / (S::kBKB / 16), cc = ch % (S::kBKB / 16);
            cp_async16(sB + n * S::kBRow + cc * 16, b_row_addr(n) + (int64_t)kb0 * (Q4 ? 16 : 32) + cc * 16, true);
        }
        for (int r = tid; r < BM; r += kThreads) {
            cp_async16(sAd + r * kKB, p.ad + s_arow[r] * nkb + kb0, r < mrows);
            if (Q4) cp_async16(sAs + r * kKB, p.as + s_arow[r] * nkb + kb0, r < mrows);
        }
        for (int n = tid; n < kBN; n += kThreads) {
            const uint32_t d = smem_u32(sBd + n * kKB);
            asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(d), "l"(b_scale_addr(n) + kb0 * 2) : "memory");
        }
    };

    float acc[MI][NJ][4];
#pragma unroll
    for (int i = 0; i < MI; ++i)
#pragma unroll
        for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[i][j][q] = 0.f;

    const int nsteps = (nkb + kKB - 1) / kKB;
    for (int s = 0; s < kStages - 1; ++s) {
        if (s < nsteps) load_stage(s, s * kKB);
        cp_async_commit();
    }
    const bool sbf = p.scale_bf16 != 0;
    for (int step = 0; step < nsteps; ++step) {
        cp_async_wait<kStages - 2>();
        __syncthreads();
        {   // prefetch step + kStages - 1
            const int nxt = step + kStages - 1;
            if (nxt < nsteps) load_stage(nxt % kStages, nxt * kKB);
            cp_async_commit();
        }
        const uint8_t* base = smem + (size_t)(step % kStages) * S::kBytes;
        const int8_t* sA = reinterpret_cast<const int8_t*>(base);
        const uint8_t* sB = base + S::kA;
        const float* sAd = reinterpret_cast<const float*>(base + S::kA + S::kB);
        const int32_t* sAs = reinterpret_cast<const int32_t*>(base + S::kA + S::kB + S::kAd);
        const uint16_t* sBd = reinterpret_cast<const uint16_t*>(base + S::kA + S::kB + S::kAd + S::kAs);
        // raw weight scales of the thread's columns for the stage's 4 blocks (8 B each)
        uint2 dwr[NJ][2];
#pragma unroll
        for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int h = 0; h < 2; ++h) dwr[j][h] = *reinterpret_cast<const uint2*>(sBd + (wn * WC + j * 8 + 2 * c + h) * kKB);
        const int lm = lane >> 3, lr = lane & 7;  // ldmatrix: lane gives row lr of matrix lm
        for (int kb = 0; kb < kKB; ++kb) {
            uint32_t bf[NJ][2];
            if (Q4 && NJ == 4) {  // matrices = n8 tiles 0..3 of block kb (16 B rows)
                uint32_t x[4];
                ldsm_x4(x, sB + (wn * WC + lm * 8 + lr) * S::kBRow + kb * 16);
#pragma unroll
                for (int j = 0; j < 4; ++j) {  // split activation order: low nibbles k 4c.., high 16+4c..
                    bf[j][0] = x[j] & 0x0f0f0f0fu;
                    bf[j][1] = (x[j] >> 4) & 0x0f0f0f0fu;
                }
            } else if (Q4) {  // NJ == 2: matrices (tile 0, kb), (tile 1, kb), rows 16 B; x2
                uint32_t x[2];
                ldsm_x2(x, sB + (wn * WC + (lm & 1) * 8 + lr) * S::kBRow + kb * 16);
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    bf[j][0] = x[j] & 0x0f0f0f0fu;
                    bf[j][1] = (x[j] >> 4) & 0x0f0f0f0fu;
                }
            } else {  // (tile j0, bytes 0-15), (j0, 16-31), (j0+1, 0-15), (j0+1, 16-31)
#pragma unroll
                for (int j0 = 0; j0 < NJ; j0 += 2) {
                    uint32_t x[4];
                    ldsm_x4(x, sB + (wn * WC + (j0 + (lm >> 1)) * 8 + lr) * S::kBRow + kb * 32 + (lm & 1) * 16);
                    bf[j0][0] = x[0];
                    bf[j0][1] = x[1];
                    bf[j0 + 1][0] = x[2];
                    bf[j0 + 1][1] = x[3];
                }
            }
            float dw[NJ][2];
#pragma unroll
            for (int j = 0; j < NJ; ++j)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t wd = (kb < 2) ? dwr[j][h].x : dwr[j][h].y;
                    dw[j][h] = scale_to_f32((uint16_t)((kb & 1) ? wd >> 16 : wd & 0xffffu), sbf);
                }
#pragma unroll
            for (int i = 0; i < MI; ++i) {
                uint32_t af[4];  // (rows 0-7, bytes 0-15), (8-15, 0-15), (0-7, 16-31), (8-15, 16-31)
                ldsm_x4(af, sA + (wm * WR + i * 16 + (lm & 1) * 8 + lr) * S::kARow + kb * 32 + (lm >> 1) * 16);
                const int r = wm * WR + i * 16 + g;
                const float d0 = sAd[r * kKB + kb], d1 = sAd[(r + 8) * kKB + kb];
                int cin[4] = {0, 0, 0, 0};
                if (Q4) {  // nibble bias: -8 * (sum of the token's block), through the MMA's C input
                    const int s0 = -8 * sAs[r * kKB + kb], s1 = -8 * sAs[(r + 8) * kKB + kb];
                    cin[0] = s0; cin[1] = s0; cin[2] = s1; cin[3] = s1;
                }
#pragma unroll
                for (int j = 0; j < NJ; ++j) {
                    int d[4];
                    mma_a8<Q4>(d, af, bf[j], cin);
                    // d0,d1: token row g, cols 2c,2c+1; d2,d3: token row g+8
                    acc[i][j][0] += ((float)d[0] * dw[j][0]) * d0;
                    acc[i][j][1] += ((float)d[1] * dw[j][1]) * d0;
                    acc[i][j][2] += ((float)d[2] * dw[j][0]) * d1;
                    acc[i][j][3] += ((float)d[3] * dw[j][1]) * d1;
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();

    // ---------------- epilogue ----------------
    if (GATE_UP) {
        // columns interleave (gate, up) per unit: col 2u = gate of unit u, 2u+1 = up.
        // Thread holds cols 2c, 2c+1 of each n8 -> one unit per (j): h = silu(gate)*up.
        float* hsm = reinterpret_cast<float*>(smem);  // [BM][kBN/2 + 1] fp32
        constexpr int HW = kBN / 2 + 1;
#pragma unroll
        for (int i = 0; i < MI; ++i)
#pragma unroll
            for (int j = 0; j < NJ; ++j)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int r = wm * WR + i * 16 + g + h * 8;
                    const int u = (wn * WC + j * 8 + 2 * c) >> 1;
                    hsm[r * HW + u] = silu_mul(acc[i][j][2 * h], acc[i][j][2 * h + 1]);
                }
        __syncthreads();
        // requantise per (row, 32-unit block): thread per block
        const int I = p.N / 2, nbI = I / 32;
        const int u0 = n0 / 2;
        for (int t = tid; t < BM * (kBN / 64); t += kThreads) {
            const int r = t / (kBN / 64), blk = t % (kBN / 64);
            if (r >= mrows) continue;
            float v[32];
            float amax = 0.f;
#pragma unroll
            for (int k = 0; k < 32; ++k) {
                v[k] = hsm[r * HW + blk * 32 + k];
                amax = fmaxf(amax, fabsf(v[k]));
            }
            const float dd = q8_scale(amax);
            const float id = q8_inv(dd);
            int qv[32];
            int sum = 0;
#pragma unroll
            for (int k = 0; k < 32; ++k) {
                qv[k] = q8_quant(v[k], id);
                sum += qv[k];
            }
            uint32_t wv[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                uint32_t w = 0;
#pragma unroll
                for (int q = 0; q < 4; ++q) w |= (uint32_t)(qv[act_elem<Q4>(k, q)] & 0xff) << (8 * q);
                wv[k] = w;
            }
            const int pos = pos0 + r;
            const int b = u0 / 32 + blk;
            uint4* dst = reinterpret_cast<uint4*>(p.hq + (int64_t)pos * I + b * 32);
            dst[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            dst[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
            p.hd[(int64_t)pos * nbI + b] = dd;
            if (Q4) p.hs[(int64_t)pos * nbI + b] = sum;
        }
    } else {
#pragma unroll
        for (int i = 0; i < MI; ++i)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int r = wm * WR + i * 16 + g + h * 8;
                if (r >= mrows) continue;
                float* orow = p.out + (int64_t)(pos0 + r) * p.N + n0;
#pragma unroll
                for (int j = 0; j < NJ; ++j) {
                    const int col = wn * WC + j * 8 + 2 * c;
                    *reinterpret_cast<float2*>(orow + col) = make_float2(acc[i][j][2 * h], acc[i][j][2 * h + 1]);
                }
            }
    }
}

// y[t][n] = sum_k w[t,k] * out[smap[t,k]][n] in k order, cast.
// ------------------------------------------------------------------ weights-on-M grouped GEMM
// For few tokens per expert (<= 16): the weight rows are the MMA's M side (16 per warp,
// 128 per CTA) and the tokens its N side (BT = 8 or 16 per tile), so an expert with 8
// tokens fills every MMA column instead of half of a 16-token M tile.  Same per-block
// fold, same outputs as grouped_gemm_kernel.  gate_up: warp w's m16 tile is gate rows
// (rows 0-7) and up rows (rows 8-15) of the units u0+8w .. u0+8w+7, so one thread holds
// the gate and up accumulators of the same (unit, token) and forms SiLU(gate)*up itself.
template <bool Q4, int BT>
struct StageW {
    static constexpr int kWKB = kKB * (Q4 ? 16 : 32);  // weight bytes per row per stage
    static constexpr int kWRow = kWKB + kRowPad;
    static constexpr int kXKB = kKB * 32;               // activation bytes per token per stage
    static constexpr int kXRow = kXKB + kRowPad;
    static constexpr int kW = kBN * kWRow;
    static constexpr int kX = BT * kXRow;
    static constexpr int kWd = kBN * kKB * 2;
    static constexpr int kXd = BT * kKB * 4;
    static constexpr int kXs = BT * kKB * 4;
    static constexpr int kBytes = kW + kX + kWd + kXd + kXs;
};

template <bool Q4, bool GATE_UP, int BT>
__global__ void __launch_bounds__(kThreads) grouped_gemm_wm_kernel(const GemmParams p) {
    using S = StageW<Q4, BT>;
    constexpr int NJ = BT / 8;
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, c = lane & 3;

    // ---- tile -> (expert, token tile, weight-row tile)
    const int ntiles_n = p.N / kBN;
    const int mt_total = p.mtile_start[p.E];
    const int tile = blockIdx.x;
    if (tile >= mt_total * ntiles_n) return;
    const int mt_glob = tile / ntiles_n, nt = tile % ntiles_n;
    int lo = 0, hi = p.E;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (p.mtile_start[mid] <= mt_glob) lo = mid;
        else hi = mid;
    }
    const int e = lo;
    const int m0 = (mt_glob - p.mtile_start[e]) * BT;
    const int cnt = p.counts[e];
    const int pos0 = p.starts[e] + m0;
    const int mtok = min(BT, cnt - m0);
    const int nkb = p.K / 32;

    __shared__ int64_t s_xrow[BT];
    for (int r = tid; r < BT; r += kThreads) {
        const int pos = pos0 + min(r, max(mtok, 1) - 1);
        s_xrow[r] = GATE_UP ? (int64_t)(p.tokmap[pos] / p.topk) : (int64_t)pos;
    }
    __syncthreads();
    const uint8_t* wexp = p.wbase + (int64_t)e * p.nrec * p.rec;
    // smem weight row r (0..127) -> its quants / its scale field
    auto w_row = [&](int r, int64_t& qoff, int64_t& soff) {
        if (GATE_UP) {
            const int w = r >> 4, rr = r & 15;
            const int64_t unit = (int64_t)nt * (kBN / 2) + w * 8 + (rr & 7);
            const int part = rr >> 3;  // 0 gate, 1 up
            qoff = unit * p.rec + (int64_t)part * p.rs;
            soff = unit * p.rec + p.sc_off + (int64_t)part * p.ss;
        } else {
            const int64_t row = (int64_t)nt * kBN + r;
            qoff = row * p.rec;
            soff = row * p.rec + p.sc_off;
        }
    };

    auto load_stage = [&](int st, int kb0) {
        uint8_t* base = smem + (size_t)st * S::kBytes;
        uint8_t* sW = base;
        int8_t* sX = reinterpret_cast<int8_t*>(base + S::kW);
        uint16_t* sWd = reinterpret_cast<uint16_t*>(base + S::kW + S::kX);
        float* sXd = reinterpret_cast<float*>(base + S::kW + S::kX + S::kWd);
        int32_t* sXs = reinterpret_cast<int32_t*>(base + S::kW + S::kX + S::kWd + S::kXd);
        for (int ch = tid; ch < kBN * (S::kWKB / 16); ch += kThreads) {
            const int r = ch / (S::kWKB / 16), cc = ch % (S::kWKB / 16);
            int64_t qo, so;
            w_row(r, qo, so);
            cp_async16(sW + r * S::kWRow + cc * 16, wexp + qo + (int64_t)kb0 * (Q4 ? 16 : 32) + cc * 16, true);
        }
        for (int ch = tid; ch < BT * (S::kXKB / 16); ch += kThreads) {
            const int r = ch / (S::kXKB / 16), cc = ch % (S::kXKB / 16);
            cp_async16(sX + r * S::kXRow + cc * 16, p.aq + s_xrow[r] * p.K + (int64_t)kb0 * 32 + cc * 16, r < mtok);
        }
        for (int r = tid; r < kBN; r += kThreads) {
            int64_t qo, so;
            w_row(r, qo, so);
            const uint32_t d = smem_u32(sWd + r * kKB);
            asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(d), "l"(wexp + so + kb0 * 2) : "memory");
        }
        for (int r = tid; r < BT; r += kThreads) {
            cp_async16(sXd + r * kKB, p.ad + s_xrow[r] * nkb + kb0, r < mtok);
            if (Q4) cp_async16(sXs + r * kKB, p.as + s_xrow[r] * nkb + kb0, r < mtok);
        }
    };

    float acc[NJ][4];
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[j][q] = 0.f;

    const int nsteps = (nkb + kKB - 1) / kKB;
    for (int s = 0; s < kStages - 1; ++s) {
        if (s < nsteps) load_stage(s, s * kKB);
        cp_async_commit();
    }
    const bool sbf = p.scale_bf16 != 0;
    const int r0 = warp * 16 + g;  // this thread's weight rows r0, r0 + 8
    for (int step = 0; step < nsteps; ++step) {
        cp_async_wait<kStages - 2>();
        __syncthreads();
        {
            const int nxt = step + kStages - 1;
            if (nxt < nsteps) load_stage(nxt % kStages, nxt * kKB);
            cp_async_commit();
        }
        const uint8_t* base = smem + (size_t)(step % kStages) * S::kBytes;
        const uint8_t* sW = base;
        const int8_t* sX = reinterpret_cast<const int8_t*>(base + S::kW);
        const uint16_t* sWd = reinterpret_cast<const uint16_t*>(base + S::kW + S::kX);
        const float* sXd = reinterpret_cast<const float*>(base + S::kW + S::kX + S::kWd);
        const int32_t* sXs = reinterpret_cast<const int32_t*>(base + S::kW + S::kX + S::kWd + S::kXd);
        // per-stage scales: the weight rows' 4 block scales (8 B each row), the tokens' 4
        // block scales and sums (16 B each token)
        float dw0[kKB], dw1[kKB];
        {
            const uint2 s0 = *reinterpret_cast<const uint2*>(sWd + r0 * kKB);
            const uint2 s1 = *reinterpret_cast<const uint2*>(sWd + (r0 + 8) * kKB);
            const uint16_t h0[4] = {(uint16_t)(s0.x & 0xffff), (uint16_t)(s0.x >> 16), (uint16_t)(s0.y & 0xffff),
                                    (uint16_t)(s0.y >> 16)};
            const uint16_t h1[4] = {(uint16_t)(s1.x & 0xffff), (uint16_t)(s1.x >> 16), (uint16_t)(s1.y & 0xffff),
                                    (uint16_t)(s1.y >> 16)};
#pragma unroll
            for (int kb = 0; kb < kKB; ++kb) {
                dw0[kb] = scale_to_f32(h0[kb], sbf);
                dw1[kb] = scale_to_f32(h1[kb], sbf);
            }
        }
        float4 da[NJ][2];
        int4 sb[NJ][2];
#pragma unroll
        for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int t = j * 8 + 2 * c + h;
                da[j][h] = *reinterpret_cast<const float4*>(sXd + t * kKB);
                if (Q4) {
                    const int4 v = *reinterpret_cast<const int4*>(sXs + t * kKB);
                    sb[j][h] = make_int4(-8 * v.x, -8 * v.y, -8 * v.z, -8 * v.w);  // nibble bias removal
                }
            }
        // fragments through ldmatrix: lane l addresses row (l & 7) of matrix (l >> 3)
        const int lm = lane >> 3, lr = lane & 7;
#pragma unroll
        for (int kp = 0; kp < kKB; kp += 2) {
            uint32_t af[2][4];
            if (Q4) {  // matrices: rows 0-7 / 8-15 of the warp's m16, blocks kp / kp+1 (16 B each)
                uint32_t x[4];
                ldsm_x4(x, sW + (warp * 16 + (lm & 1) * 8 + lr) * S::kWRow + (kp + (lm >> 1)) * 16);
#pragma unroll
                for (int q = 0; q < 2; ++q) {  // word c: low nibbles -> k 4c.., high nibbles -> k 16+4c..
                    af[q][0] = x[2 * q] & 0x0f0f0f0fu;
                    af[q][1] = x[2 * q + 1] & 0x0f0f0f0fu;
                    af[q][2] = (x[2 * q] >> 4) & 0x0f0f0f0fu;
                    af[q][3] = (x[2 * q + 1] >> 4) & 0x0f0f0f0fu;
                }
            } else {  // one block = rows 0-7 / 8-15 x bytes 0-15 / 16-31
#pragma unroll
                for (int q = 0; q < 2; ++q)
                    ldsm_x4(af[q], sW + (warp * 16 + (lm & 1) * 8 + lr) * S::kWRow + (kp + q) * 32 + (lm >> 1) * 16);
            }
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                uint32_t bx[4];  // tokens j*8.. : (block kp, bytes 0-15), (kp, 16-31), (kp+1, 0-15), (kp+1, 16-31)
                ldsm_x4(bx, sX + (j * 8 + lr) * S::kXRow + kp * 32 + lm * 16);
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int kb = kp + q;
                    const uint32_t bf[2] = {bx[2 * q], bx[2 * q + 1]};
                    const float da0 = f4_get(da[j][0], kb), da1 = f4_get(da[j][1], kb);
                    int cin[4] = {0, 0, 0, 0};
                    if (Q4) {
                        const int s0 = i4_get(sb[j][0], kb), s1 = i4_get(sb[j][1], kb);
                        cin[0] = s0; cin[1] = s1; cin[2] = s0; cin[3] = s1;
                    }
                    int d[4];
                    mma_w<Q4>(d, af[q], bf, cin);
                    // d0: (row r0, token t0), d1: (r0, t0+1), d2: (r0+8, t0), d3: (r0+8, t0+1)
                    acc[j][0] += ((float)d[0] * dw0[kb]) * da0;
                    acc[j][1] += ((float)d[1] * dw0[kb]) * da1;
                    acc[j][2] += ((float)d[2] * dw1[kb]) * da0;
                    acc[j][3] += ((float)d[3] * dw1[kb]) * da1;
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();

    if (GATE_UP) {
        // h[token][unit] = SiLU(gate) * up, staged [BT][kBN/2 + 1] fp32, then requantised per
        // (token, 32-unit block)
        float* hsm = reinterpret_cast<float*>(smem);
        constexpr int HW = kBN / 2 + 1;
        const int ul = warp * 8 + g;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            const int t0 = j * 8 + 2 * c;
            hsm[t0 * HW + ul] = silu_mul(acc[j][0], acc[j][2]);
            hsm[(t0 + 1) * HW + ul] = silu_mul(acc[j][1], acc[j][3]);
        }
        __syncthreads();
        const int I = p.N / 2, nbI = I / 32;
        const int u0 = nt * (kBN / 2);
        for (int t = tid; t < BT * (kBN / 64); t += kThreads) {
            const int r = t / (kBN / 64), blk = t % (kBN / 64);
            if (r >= mtok) continue;
            float v[32];
            float amax = 0.f;
#pragma unroll
            for (int k = 0; k < 32; ++k) {
                v[k] = hsm[r * HW + blk * 32 + k];
                amax = fmaxf(amax, fabsf(v[k]));
            }
            const float dd = q8_scale(amax);
            const float id = q8_inv(dd);
            int qv[32];
            int sum = 0;
#pragma unroll
            for (int k = 0; k < 32; ++k) {
                qv[k] = q8_quant(v[k], id);
                sum += qv[k];
            }
            uint32_t wv[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                uint32_t w = 0;
#pragma unroll
                for (int q = 0; q < 4; ++q) w |= (uint32_t)(qv[act_elem<Q4>(k, q)] & 0xff) << (8 * q);
                wv[k] = w;
            }
            const int pos = pos0 + r;
            const int b = u0 / 32 + blk;
            uint4* dst = reinterpret_cast<uint4*>(p.hq + (int64_t)pos * I + b * 32);
            dst[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            dst[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
            p.hd[(int64_t)pos * nbI + b] = dd;
            if (Q4) p.hs[(int64_t)pos * nbI + b] = sum;
        }
    } else {
        const int n0 = nt * kBN;
#pragma unroll
        for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int t = j * 8 + 2 * c + (q & 1);
                if (t >= mtok) continue;
                const int row = n0 + r0 + (q >> 1) * 8;
                p.out[(int64_t)(pos0 + t) * p.N + row] = acc[j][q];
            }
    }
}

__global__ void combine_kernel(const float* out, const int32_t* smap, const float* tw, int T, int K, int H,
                               void* y, int out_kind) {
    const int64_t total = (int64_t)T * (H / 4);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / (H / 4)), n4 = (int)(i % (H / 4)) * 4;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        for (int k = 0; k < K; ++k) {
            const int pos = smap[t * K + k];
            if (pos < 0) continue;
            const float w = tw[t * K + k];
            const float4 v = *reinterpret_cast<const float4*>(out + (int64_t)pos * H + n4);
            a0 += w * v.x;
            a1 += w * v.y;
            a2 += w * v.z;
            a3 += w * v.w;
        }
        const int64_t o = (int64_t)t * H + n4;
        if (out_kind == 2) {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + o) = make_float4(a0, a1, a2, a3);
        } else if (out_kind == 1) {
            __nv_bfloat16* yb = reinterpret_cast<__nv_bfloat16*>(y) + o;
            yb[0] = __float2bfloat16_rn(a0); yb[1] = __float2bfloat16_rn(a1);
            yb[2] = __float2bfloat16_rn(a2); yb[3] = __float2bfloat16_rn(a3);
        } else {
            __half* yh = reinterpret_cast<__half*>(y) + o;
            yh[0] = __float2half_rn(a0); yh[1] = __float2half_rn(a1);
            yh[2] = __float2half_rn(a2); yh[3] = __float2half_rn(a3);
        }
    }
}

}  // namespace gemm
}  // namespace moe
