// Grouped GEMMs of the fused MoE layer on the 5th-generation tensor cores (tcgen05 +
// TMEM), for many tokens per expert.
//
// Arithmetic.  The reference folds every 32-block's integer dot with two fp32 scales
// (gemm_kernels.cpp:66-186), which keeps the int8 MMA kernels of moe_gemm.cuh busy on the
// CUDA cores.  Here both operands are dequantised once into fp16 instead:
//   A  = fp16(q_a * d_a): the token rows after the reference's Q8_0 activation
//        quantisation (gemm_kernels.cpp:25-58), resp. h after its requantisation
//        (gemm_kernels.cpp:394-425) -- the reference's quantisation noise is reproduced,
//        only rounded to fp16 (2^-11 relative);
//   B  = fp16(q_w * d_w) (Q4_0: (nibble - 8) * d_w), dequantised in shared memory;
// and the contraction runs in fp16 x fp16 -> fp32 on tcgen05.mma (kind::f16), one
// accumulator tile of 128 token rows x 128 weight rows in TMEM.  The result equals the
// reference's to the fp16 rounding of the operands (tolerance parity, not bit-exact).
// fp16 rather than bf16: bf16's 2^-9 rounding left the FFN output at the edge of the
// 1e-2 tolerance.  A 32-block whose magnitude exceeds the fp16 range (|x| > 65504) sets
// device error kErrRange; such activations need the int8 path (MOE_TC_MIN_PER_EXPERT).
//
// Tile schedule: one CTA per (expert, 128-token tile, 128-weight-row tile), 256 threads,
// 3 CTAs per SM; K is streamed in steps of 64 elements (one 128-byte swizzle atom per row)
// through kStagesTc stages:
//   cp.async  A rows (gathered token rows, fp16) straight into the SWIZZLE_128B K-major
//             layout, one step ahead;
//   dequant   every thread expands half a B row (one 32-block, loaded into registers two
//             steps ahead) into the fp16 B tile;
//   mma       one thread issues 4 x tcgen05.mma (K = 16 each) and commits them to the
//             stage's mbarrier, which the refill of that stage waits on.
// (A warp-specialised variant with 3 stages and 2 CTAs per SM measured slower.)
// All waits are bounded; a wait that runs out sets the error word and the tile is dropped.
// Epilogue: warps w and w+4 read TMEM lane quarter w%4, columns [64*(w/4), +64):
//   gate_up  columns interleave (gate, up) per unit, so a thread holds 32 units of its
//            token: SiLU(gate)*up, the Q8_0 requantisation of that 32-unit block, and
//            fp16(q_h * d_h) as the down GEMM's A row;
//   down     fp32 rows of out[pos][n], combined by combine_kernel.
// No multicast, no cluster, one GPU's memory only.
#pragma once
#include "moe_gemm.cuh"

namespace moe {
namespace gemm {

constexpr int kTcM = 128, kTcN = 128, kTcK = 64;  // tile rows (tokens), cols (weight rows), K step
constexpr int kStagesTc = 2;  // x 32 KB: with 1 KB alignment slack and 80 registers, 3 CTAs per SM

template <bool NIB>  // NIB: 4-bit weights (Q4_0, AWQ)
struct StageTc {
    static constexpr int kA = kTcM * 128;                // fp16 A tile, 128 B per row (SW128 K-major)
    static constexpr int kB = kTcN * 128;                // fp16 B tile
    static constexpr int kRawRow = NIB ? 32 : 64;        // quantised bytes of one row per step
    static constexpr int kBytes = kA + kB;                // 32 KB: stages stay 1024-aligned
};

// ---------------------------------------------------------------- tcgen05 helpers
// Shared-memory matrix descriptor, SWIZZLE_128B, K-major: start address >> 4 (bits 0-13),
// leading byte offset (ignored for swizzled K-major, 16 B) >> 4 (bits 16-29), stride byte
// offset = 1024 B between 8-row groups >> 4 (bits 32-45), descriptor version 1 (bits
// 46-47), base offset 0, layout type 2 = SWIZZLE_128B (bits 61-63).
MOE_DEV uint64_t tc_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)(16u >> 4) << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor, kind::f16: D fp32 (bits 4-5 = 1), A and B fp16 (bits 7-9 and
// 10-12 = 0), both K-major (bits 15, 16 = 0), N >> 3 (bits 17-22), M >> 4 (bits 24-28).
__host__ __device__ constexpr uint32_t tc_idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// The same with A and B bf16 (bits 7-9 and 10-12 = 1): the AWQ path with bf16 activations.
__host__ __device__ constexpr uint32_t tc_idesc_bf16(int M, int N) {
    return tc_idesc_f16(M, N) | (1u << 7) | (1u << 10);
}

MOE_DEV void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

MOE_DEV void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

MOE_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MOE_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
MOE_DEV void tc_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

MOE_DEV void cp_async4(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}

// Token rows -> fp16(q * d) with the reference's Q8_0 rule (thread per 32-block).
__global__ void quant_rows_f16_kernel(const uint8_t* x, int act_bf16, int rows, int cols, __half* out, int32_t* err) {
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
        if (amax > 65504.f) set_err(err, kErrRange);
        const float dd = q8_scale(amax);
        const float id = q8_inv(dd);
        uint32_t packed[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
            const __half2 b = __floats2half2_rn((float)q8_quant(v[e], id) * dd, (float)q8_quant(v[e + 1], id) * dd);
            packed[e / 2] = *reinterpret_cast<const uint32_t*>(&b);
        }
        uint4* dst = reinterpret_cast<uint4*>(out + (size_t)g * 32);
#pragma unroll
        for (int k = 0; k < 4; ++k) dst[k] = make_uint4(packed[4 * k], packed[4 * k + 1], packed[4 * k + 2], packed[4 * k + 3]);
    }
}

struct TcParams {
    const __half* a;  // gate_up: token rows [T][K] (gathered through tokmap/topk); down: position rows [P][K]
    const uint8_t* wbase;    // weight records, as GemmParams
    int64_t rec;
    int rows_per_rec, rs, sc_off, ss, nrec, K, N, scale_bf16;
    const int32_t* counts;
    const int32_t* starts;
    const int32_t* mtile_start;  // tiles of kTcM rows per expert
    const int32_t* tokmap;
    int topk, E;
    int group, ngk;  // AWQ: group size along K and K / group
    int bf16ops;     // AWQ with bf16 activations: bf16 operands (exact x); otherwise fp16
    __half* ha;  // gate_up output: the down GEMM's A rows [P][I] (fp16(q_h * d_h); AWQ: h in the operand type)
    float* out;         // down output: [P][H]
    int32_t* err;
};

constexpr int kTcProducers = 256;  // all threads copy A, dequantise B and run the epilogue
constexpr int kTcThreads = kTcProducers;

template <int WF, bool GATE_UP>  // WF: 0 Q8_0, 1 Q4_0, 2 AWQ
__global__ void __launch_bounds__(kTcThreads, 1) grouped_gemm_tc_kernel(const TcParams p) {
    constexpr bool NIB = WF != 0, AWQ = WF == 2;
    using S = StageTc<NIB>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the swizzled tiles need 1024-byte alignment
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t s_empty[kStagesTc], s_done;
    __shared__ uint32_t s_tmem;
    __shared__ int64_t s_arow[kTcM];
    __shared__ int s_ok;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const int ntiles_n = p.N / kTcN;
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
    const int m0 = (mt_glob - p.mtile_start[e]) * kTcM;
    const int cnt = p.counts[e];
    const int pos0 = p.starts[e] + m0;
    const int mrows = min(kTcM, cnt - m0);
    const int nsteps = p.K / kTcK;
    const uint8_t* wexp = p.wbase + (int64_t)e * p.nrec * p.rec;

    for (int r = tid; r < kTcM; r += kTcThreads) {
        const int pos = pos0 + min(r, max(mrows, 1) - 1);
        s_arow[r] = GATE_UP ? (int64_t)(p.tokmap[pos] / p.topk) : (int64_t)pos;
    }
    if (tid == 0) {
        for (int s = 0; s < kStagesTc; ++s) mbar_init(&s_empty[s], 1);  // tcgen05.commit of the step's MMAs
        mbar_init(&s_done, 1);
        s_ok = 1;
    }
    if (warp == 0) {  // TMEM: 128 fp32 columns x 128 lanes for the accumulator tile
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;" ::"r"(smem_u32(&s_tmem))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_barrier_init();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    // weight row n (0..127) of this tile -> offsets of its quants and its scale field
    auto w_row = [&](int n, int64_t& qoff, int64_t& soff) {
        const int64_t gn = (int64_t)nt * kTcN + n;
        const int64_t rec = gn / p.rows_per_rec, sub = gn - rec * p.rows_per_rec;
        qoff = rec * p.rec + sub * p.rs;
        soff = rec * p.rec + p.sc_off + sub * p.ss;
    };
    auto load_stage = [&](int st, int ks) {
        uint8_t* base = smem + (size_t)st * S::kBytes;
        uint8_t* sA = base;
        // A: 128 rows x 8 chunks of 16 B, chunk c of row r at position c ^ (r & 7)
        for (int ch = tid; ch < kTcM * 8; ch += kTcProducers) {
            const int r = ch >> 3, c = ch & 7;
            const __half* src = p.a + s_arow[r] * p.K + (int64_t)ks * kTcK + c * 8;
            cp_async16(sA + r * 128 + ((c ^ (r & 7)) << 4), src, r < mrows);
        }
    };

    // raw B of this thread's (row tid/2, 32-block tid%2) per step, loaded into registers two
    // steps ahead of its dequantisation (no shared staging: 3 CTAs fit on an SM)
    struct RawB {
        uint4 q0, q1;  // 4-bit formats: q0 only
        uint16_t sc, z;  // block (Q4/Q8) or group (AWQ) scale; AWQ zero point
    };
    auto load_raw = [&](int ks, RawB& rb) {
        const int n = tid >> 1, h = tid & 1;
        int64_t qo, so;
        w_row(n, qo, so);
        const uint4* src = reinterpret_cast<const uint4*>(wexp + qo + (int64_t)ks * S::kRawRow + h * (NIB ? 16 : 32));
        rb.q0 = __ldg(src);
        if (!NIB) rb.q1 = __ldg(src + 1);
        if (AWQ) {  // the 32-block's group: bf16 scale, then the u8 zero points after all scales
            const int grp = (ks * kTcK + h * 32) / p.group;
            rb.sc = __ldg(reinterpret_cast<const unsigned short*>(wexp + so) + grp);
            rb.z = __ldg(wexp + so + 2 * p.ngk + grp);
        } else {
            rb.sc = __ldg(reinterpret_cast<const unsigned short*>(wexp + so) + 2 * ks + h);
        }
    };
    RawB rb0{}, rb1{};
    if (tid < kTcProducers) {
        if (0 < nsteps) load_raw(0, rb0);
        if (1 < nsteps) load_raw(1, rb1);
    }
    const bool bfo = AWQ && p.bf16ops;
    const uint32_t idesc = bfo ? tc_idesc_bf16(kTcM, kTcN) : tc_idesc_f16(kTcM, kTcN);
    auto pack2 = [&](float a, float b) -> uint32_t {
        if (bfo) {
            const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
            return *reinterpret_cast<const uint32_t*>(&v);
        }
        const __half2 v = __floats2half2_rn(a, b);
        return *reinterpret_cast<const uint32_t*>(&v);
    };
    const bool sbf = p.scale_bf16 != 0;
    bool ok = true;
    for (int s = 0; s < kStagesTc - 1; ++s) {
        if (s < nsteps) load_stage(s, s);
        cp_async_commit();
    }
    for (int s = 0; s < nsteps; ++s) {
        const int st = s % kStagesTc;
        uint8_t* base = smem + (size_t)st * S::kBytes;
        cp_async_wait<kStagesTc - 2>();
        __syncthreads();
        {   // dequantise B: thread -> (row tid/2, 32-block tid%2) -> 16 fp16 pairs = 4 chunks
            const int n = tid >> 1, h = tid & 1;
            const RawB cur = rb0;
            rb0 = rb1;
            if (s + 2 < nsteps) load_raw(s + 2, rb1);
            const float dw = AWQ ? __uint_as_float((uint32_t)cur.sc << 16) : scale_to_f32(cur.sc, sbf);
            // 2^23 + n as float bits minus 2^23 + offset: exact n - 8 (Q4_0) or n - z (AWQ)
            const float off = AWQ ? 8388608.0f + (float)cur.z : 8388616.0f;
            uint32_t pk[16];
            if (NIB) {  // word i = elements 8i..8i+7, nibble j = element 8i+j
                const uint32_t qq[4] = {cur.q0.x, cur.q0.y, cur.q0.z, cur.q0.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 8; j += 2) {
                        const float v0 = (__uint_as_float(((qq[i] >> (4 * j)) & 15u) | 0x4B000000u) - off) * dw;
                        const float v1 = (__uint_as_float(((qq[i] >> (4 * j + 4)) & 15u) | 0x4B000000u) - off) * dw;
                        pk[4 * i + j / 2] = pack2(v0, v1);
                    }
            } else {  // word i = elements 4i..4i+3 (int8)
                const uint32_t qq[8] = {cur.q0.x, cur.q0.y, cur.q0.z, cur.q0.w, cur.q1.x, cur.q1.y, cur.q1.z, cur.q1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < 4; j += 2) {
                        // byte b ^ 0x80 = q + 128: 2^23 + q + 128 as float bits, minus 2^23 + 128
                        const float v0 = (__uint_as_float((((qq[i] >> (8 * j)) & 0xffu) ^ 0x80u) | 0x4B000000u) - 8388736.0f) * dw;
                        const float v1 = (__uint_as_float((((qq[i] >> (8 * j + 8)) & 0xffu) ^ 0x80u) | 0x4B000000u) - 8388736.0f) * dw;
                        pk[2 * i + j / 2] = pack2(v0, v1);
                    }
            }
            uint8_t* rowp = base + S::kA + n * 128;
#pragma unroll
            for (int i = 0; i < 4; ++i)
                *reinterpret_cast<uint4*>(rowp + (((4 * h + i) ^ (n & 7)) << 4)) =
                    make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
        // generic-proxy writes (cp.async A, the dequantised B) -> visible to the tensor core
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t sa = smem_u32(base), sb = smem_u32(base + S::kA);
#pragma unroll
            for (int k = 0; k < kTcK / 16; ++k)  // K = 16 per MMA: advance 32 B inside the swizzle atom
                tc_mma(tmem, tc_desc_sw128(sa + 32 * k), tc_desc_sw128(sb + 32 * k), idesc, s > 0 || k > 0);
            tc_commit(&s_empty[st]);
        }
        // refill: step s + kStagesTc - 1 goes to the stage last read by the MMAs of step s - 1
        if (s >= 1) {
            const int ps = s - 1;
            if (!mbar_wait(&s_empty[ps % kStagesTc], (uint32_t)(ps / kStagesTc) & 1u)) ok = false;
        }
        if (s + kStagesTc - 1 < nsteps) load_stage((s + kStagesTc - 1) % kStagesTc, s + kStagesTc - 1);
        cp_async_commit();
    }
    cp_async_wait<0>();
    if (tid == 0) tc_commit(&s_done);  // arrives once every MMA issued above has completed
    if (!ok) set_err(p.err, kErrFullWait);
    // bounded wait for the accumulator (on a failure path as well, before TMEM is released)
    if (!mbar_wait(&s_done, 0u)) {
        set_err(p.err, kErrFullWait);
        ok = false;
    }
    if (!ok) s_ok = 0;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---------------- epilogue: lane quarter warp%4, columns [64*(warp/4), +64) ----------------
    if (s_ok && tid < kTcProducers) {
        const int r = (warp & 3) * 32 + lane;  // token row of the tile (TMEM lane)
        const int c0 = (warp >> 2) * 64;
        const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)c0;
        float v[64];
        {
            float t0[32], t1[32];
            tc_ld32(taddr, t0);
            tc_ld32(taddr + 32, t1);
#pragma unroll
            for (int i = 0; i < 32; ++i) { v[i] = t0[i]; v[32 + i] = t1[i]; }
        }
        if (r < mrows) {
            const int pos = pos0 + r;
            if (GATE_UP) {  // columns (2u, 2u+1) = (gate, up) of unit u0 + u
                const int I = p.N / 2;
                const int u0 = nt * (kTcN / 2) + c0 / 2;  // a 32-unit block
                float hv[32];
                float amax = 0.f;
#pragma unroll
                for (int u = 0; u < 32; ++u) {
                    hv[u] = silu_mul(v[2 * u], v[2 * u + 1]);
                    amax = fmaxf(amax, fabsf(hv[u]));
                }
                if (amax > 65504.f && !bfo) set_err(p.err, kErrRange);
                uint32_t pk[16];
                if (AWQ) {  // W4A16: h stays 16-bit (no requantisation)
#pragma unroll
                    for (int u = 0; u < 32; u += 2) pk[u / 2] = pack2(hv[u], hv[u + 1]);
                } else {
                    const float dd = q8_scale(amax);
                    const float id = q8_inv(dd);
#pragma unroll
                    for (int u = 0; u < 32; u += 2)
                        pk[u / 2] = pack2((float)q8_quant(hv[u], id) * dd, (float)q8_quant(hv[u + 1], id) * dd);
                }
                uint4* dst = reinterpret_cast<uint4*>(p.ha + (int64_t)pos * I + u0);
#pragma unroll
                for (int k = 0; k < 4; ++k) dst[k] = make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
            } else {
                float4* dst = reinterpret_cast<float4*>(p.out + (int64_t)pos * p.N + nt * kTcN + c0);
#pragma unroll
                for (int k = 0; k < 16; ++k) dst[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;" ::"r"(tmem) : "memory");
    }
}

}  // namespace gemm
}  // namespace moe
