// Cluster decode kernel: the fused MoE layer for decode-size token counts, without a
// grid-wide barrier.  Thread-block clusters of `cs` CTAs (cs = 4 by default) each take
// "work units": one routed expert restricted to a K-range of its intermediate dimension
// (q of Q equal ranges of the I units; Q is chosen on the device from the number of active
// experts so that the work units fill the clusters; an expert with more routed pairs than
// tokens in the call, which only duplicate ids cause, is also cut into slices of T pairs).
// Inside a cluster, CTA r owns
//   gate_up  units [q I/Q + r I/(Q cs), ...) of the K-range (gate row j + up row j), and
//   down     rows  [r H/cs, (r+1) H/cs) over the K-range (a partial sum of the down row).
// Per work unit:
//   1. gate_up + SiLU*up of the CTA's units for the unit's tokens -> h slice;
//   2. the slice goes into every cluster CTA's h buffer through distributed shared memory
//      (st.shared::cluster), then one cluster barrier (hardware; a second barrier before the
//      next unit's stores keeps the single h buffer free of readers);
//   3. requantisation of the K-range of h (Q8_0 / Q4_0, gemm_kernels.cpp:394-425) or its
//      16-bit per-64 sums (AWQ), then the CTA's down rows over the K-range -> fp32 rows of
//      `part` (one row per routed pair and K-range).
// Combine (q8_gemm.cpp:593-613): the output rows are cut into 32 row blocks, each with an
// arrival counter; a CTA adds its work-unit count to the counters of its rows (release /
// acquire) and the CTA that completes a block's count sums, for the block's rows, the K-range
// partials of each routed pair and those in k order, then casts.  The order does not depend
// on which CTA arrives last, so the output is deterministic.
//
// Every CTA routes the pairs itself (moe_common.cpp:146-184) and stages the tokens.
// Weights stream with cp.async.bulk (contiguous items of up to ~8 KB, no multicast) into
// per-warp byte rings of shared memory (an item goes where it fits, wrapping to the ring's
// start), one mbarrier per item in flight with bounded waits, issued in consumption order
// across work units.
//
// Formats.  Q8_0 / Q4_0: gate_up from the unit records of the other decode kernels; down
// from row-slice records [E][H/32][I/32] of 32 rows x one 32-column block (weights, then
// 32 scales), so a lane owns a row and a warp's K-range of a 32-row slice is one copy; exact
// per-32-block integer dots (dp4a) and the reference's fold.  AWQ W4A16: records of 16
// (gate_up) or 32 (down) rows x 64 k laid out for mma.sync m16n8k16: each lane's nibbles of
// a row are 8 contiguous bytes, the pair (k, k+1) at nibble positions (p, p+4) so that
// (w >> 4p) & 0x000F000F | magic is two 16-bit values M + q exactly (bf16: M = 128, fp16:
// M = 1024); the tensor cores accumulate sum_k (M + q_k) x_k in fp32 per 64 k and the term
// s * (D - (M + z) * sum_k x_k) = sum_k s (q_k - z) x_k is folded in fp32.  h between the
// projections is rounded to the activation type (bf16 / fp16), as in the AWQ GEMM path.
#pragma once
#include "moe_decode.cuh"

namespace moe {

constexpr int kClWarps = 16;
constexpr int kClThreads = kClWarps * 32;
constexpr int kClMaxQ = 16;        // K-ranges per expert (Q) are powers of two up to this
constexpr int kClRowBlocks = 32;   // output row blocks of the combine
constexpr int kClInFlight = 16;    // bulk copies in flight per warp (one mbarrier each)
constexpr int kAwqK = 64;          // k per AWQ record
constexpr int kAwqGuRec = 560;     // 16 rows x 32 B nibbles | 16 bf16 scales | 16 u8 zeros
constexpr int kAwqDnRec = 1120;    // 32 rows x 32 B nibbles | 32 bf16 scales | 32 u8 zeros

struct ClParams {
    // Q8_0 / Q4_0: unit records [E][I] and row-slice records [E][H/32][I/32];
    // AWQ: gate_up records [E][I/16][2][H/64], down records [E][H/32][I/64]
    const uint8_t* gu;
    const uint8_t* dn;
    int32_t rs1, ss1;    // Q8/Q4 unit record fields (DecodeParams layout)
    int32_t E, e_off, H, I, T, K;
    const int32_t* emap;
    int32_t emap_n;
    int32_t scale_bf16, act_bf16, out_kind;
    const void* x;
    void* y;
    const int32_t* ids;
    const float* tw;
    float* part;         // [T*K*Q][H] fp32 partial down rows per routed pair and K-range
    unsigned int* cnt;   // [kClRowBlocks] combine arrival counters (zero between launches)
    int32_t* err;
    int32_t qmask;       // allowed Q values (bit log2 Q)
    int32_t* meta;       // separate-combine mode (non-null): Q, then the routing's scatter map [T*K]
    // shared-memory carve-up (bytes)
    int32_t off_wl, off_x, off_h, off_hq, off_p, off_out, off_ring;
    int32_t ring_bytes;  // per-warp byte ring (items of different sizes, up to kClInFlight in flight)
    int32_t upi;         // Q8/Q4: gate_up units per item; AWQ: gate_up records per item
    int32_t kpi;         // Q8/Q4: down 32-column blocks per item; AWQ: down records per item
    int32_t hbuf_bytes;  // the h exchange buffer
    int32_t flags;
    unsigned long long* dbg;  // optional per-CTA stamps [grid][kStamps] (globaltimer ns)
};

MOE_DEV uint32_t cl_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
MOE_DEV uint32_t cl_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
MOE_DEV uint32_t cl_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
MOE_DEV uint32_t cl_count() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
MOE_DEV void cl_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
MOE_DEV void cl_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
MOE_DEV void cl_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// Address of the same shared-memory location in cluster CTA `rank`.
MOE_DEV uint32_t cl_map(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
MOE_DEV void st_cl_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
MOE_DEV void st_cl_v4(uint32_t addr, float4 v) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}
MOE_DEV unsigned int atom_add_acq_rel_gpu(unsigned int* p, unsigned int v) {
    unsigned int old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// D += A * B, m16n8k16, 16-bit inputs (bf16 or fp16), fp32 accumulators.
template <bool BF>
MOE_DEV void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if constexpr (BF)
        asm(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
        asm(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <bool BF>
MOE_DEV uint16_t to16(float v) {
    if constexpr (BF) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
    else return __half_as_ushort(__float2half_rn(v));
}
template <bool BF>
MOE_DEV float from16(uint16_t b) {
    if constexpr (BF) return __uint_as_float((uint32_t)b << 16);
    else return __half2float(__ushort_as_half(b));
}

// The A fragments of one 16-row x 64-k AWQ tile (q at `q`, 32 B per row) for the four
// k16 steps of mma.sync m16n8k16: a[4 s + i] = register i of step s, each two 16-bit values
// M + q exactly (bf16: M = 128, fp16: M = 1024).
template <bool BF>
MOE_DEV void awq_frag64(const uint8_t* q, int lane, uint32_t (&a)[16]) {
    constexpr uint32_t kMagic = BF ? 0x43004300u : 0x64006400u;
    const int g = lane >> 2, c = lane & 3;
    const uint2 qa = *reinterpret_cast<const uint2*>(q + g * 32 + c * 8);
    const uint2 qb = *reinterpret_cast<const uint2*>(q + (g + 8) * 32 + c * 8);
    const uint32_t wa[2] = {qa.x, qa.y}, wb[2] = {qb.x, qb.y};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const int j = s >> 1, sh = (s & 1) * 8;
        a[4 * s + 0] = ((wa[j] >> sh) & 0x000F000Fu) | kMagic;        // row g,   k 2c, 2c+1
        a[4 * s + 1] = ((wb[j] >> sh) & 0x000F000Fu) | kMagic;        // row g+8, k 2c, 2c+1
        a[4 * s + 2] = ((wa[j] >> (sh + 4)) & 0x000F000Fu) | kMagic;  // row g,   k 2c+8, 2c+9
        a[4 * s + 3] = ((wb[j] >> (sh + 4)) & 0x000F000Fu) | kMagic;  // row g+8, k 2c+8, 2c+9
    }
}

// The tile's products from its fragments against the B rows of up to 8 positions: brow = this
// lane's 16-bit row (position lane/4) at the tile's first k, or nullptr; xs0 / xs1 = the sums
// of the B rows of positions 2c / 2c+1 over the tile's k; s0 / s1 and z0 / z1 = scale and zero
// point of rows g and g+8.  Adds s (D - (M + z) sum_k x_k) to tot[4] = rows (g, g+8) x
// positions (2c, 2c+1).
template <bool BF>
MOE_DEV void awq_mma64_frag(const uint32_t (&a)[16], float s0, float s1, float z0, float z1, const uint16_t* brow,
                            float xs0, float xs1, int lane, float (&tot)[4]) {
    constexpr float kM = BF ? 128.0f : 1024.0f;
    const int c = lane & 3;
    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        uint32_t b0 = 0, b1 = 0;
        if (brow) {
            b0 = *reinterpret_cast<const uint32_t*>(brow + 16 * s + 2 * c);
            b1 = *reinterpret_cast<const uint32_t*>(brow + 16 * s + 2 * c + 8);
        }
        const uint32_t as[4] = {a[4 * s], a[4 * s + 1], a[4 * s + 2], a[4 * s + 3]};
        mma16816<BF>(d, as, b0, b1);
    }
    const float m0 = kM + z0, m1 = kM + z1;
    tot[0] = fmaf(s0, fmaf(-m0, xs0, d[0]), tot[0]);
    tot[1] = fmaf(s0, fmaf(-m0, xs1, d[1]), tot[1]);
    tot[2] = fmaf(s1, fmaf(-m1, xs0, d[2]), tot[2]);
    tot[3] = fmaf(s1, fmaf(-m1, xs1, d[3]), tot[3]);
}

// One 16-row x 64-k AWQ tile (q at `q`, 32 B per row; scales `sc`, zeros `zp`, one per
// row): awq_frag64 then awq_mma64_frag.
template <bool BF>
MOE_DEV void awq_mma64(const uint8_t* q, const uint16_t* sc, const uint8_t* zp, const uint16_t* brow, float xs0,
                       float xs1, int lane, float (&tot)[4]) {
    uint32_t a[16];
    awq_frag64<BF>(q, lane, a);
    const int g = lane >> 2;
    awq_mma64_frag<BF>(a, __uint_as_float((uint32_t)sc[g] << 16), __uint_as_float((uint32_t)sc[g + 8] << 16),
                       (float)zp[g], (float)zp[g + 8], brow, xs0, xs1, lane, tot);
}

// Contiguous per-warp ranges [floor(w N / W), floor((w+1) N / W)) of N items.
MOE_DEV int range_lo(int w, int N) { return (int)((int64_t)w * N / kClWarps); }
// Warp owning item `it` under that split.
MOE_DEV int item_owner(int it, int N) { return (kClWarps * (it + 1) + N - 1) / N - 1; }

// Sum of 64 16-bit values by one warp (fixed shuffle tree; lanes 0-15 hold 4 each).
template <bool BF>
MOE_DEV float warp_sum64(const uint16_t* row, int lane) {
    float s = 0.f;
    if (lane < 16) {
        const uint2 v = *reinterpret_cast<const uint2*>(row + 4 * lane);
        s = (from16<BF>((uint16_t)(v.x & 0xffffu)) + from16<BF>((uint16_t)(v.x >> 16))) +
            (from16<BF>((uint16_t)(v.y & 0xffffu)) + from16<BF>((uint16_t)(v.y >> 16)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
}

// Requantise h [mc][KR] fp32 (shared) into q [mc][KR] / d / s (shared), a quad per 32-block.
template <bool Q4>
MOE_DEV void requant_smem(const float* h, int mc, int KR, int8_t* q, float* d, int32_t* s, int tid) {
    const int nblk = mc * (KR >> 5), sub = tid & 3;
    const uint32_t qm = quad_mask(tid & 31);
    #pragma unroll 1
    for (int g = tid >> 2; g < nblk; g += kClThreads / 4) {
        float v[8];
        const float4 a = *reinterpret_cast<const float4*>(h + (size_t)g * 32 + sub * 8);
        const float4 b = *reinterpret_cast<const float4*>(h + (size_t)g * 32 + sub * 8 + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
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

// Per-warp item bookkeeping of the cluster kernel (shared memory; lane 0 issues).
struct ClWarp {
    int32_t g_lo, g_n, d_lo, d_n;  // gate_up units / AWQ records, down slices / row blocks of the warp
    int32_t n1, n2, per_slice, total;
    int32_t nissued, head;
};
// Work geometry of one launch (every thread computes it).
struct ClGeo {
    int32_t NC, cid, rank, n_my, Q, KR, UPC, KB, KH, RPC, NK1;
};

// gate_up item i of a warp -> (first unit / record, count): runs of <= upi units (Q8/Q4) or
// of <= upi records inside one 16-row tile (AWQ, NK1 records per tile).
template <bool AWQ>
MOE_DEV void cl_gu_item(const ClWarp& w, int upi, int NK1, int i, int& first, int& cnt) {
    if constexpr (AWQ) {
        int it = w.g_lo;
        while (true) {
            const int rti = it / NK1, end = min(w.g_lo + w.g_n, (rti + 1) * NK1);
            const int ni = (end - it + upi - 1) / upi;
            if (i < ni) {
                first = it + i * upi;
                cnt = min(upi, end - first);
                return;
            }
            i -= ni;
            it = end;
        }
    } else {
        first = w.g_lo + i * upi;
        cnt = min(upi, w.g_lo + w.g_n - first);
    }
}

// Issue this warp's next items into its byte ring while they fit (lane 0).  Items are issued
// in consumption order: gate_up items of work unit 0, its down items, then unit 1's, ...  An
// item goes at `head` if it fits before the ring's end, else at 0, and never over the oldest
// item still in use.
template <int FMT>
__device__ __forceinline__ void cl_top_up(const ClParams& p, const ClGeo& g, ClWarp& w, const int32_t* wl,
                                       const int32_t* ue, uint8_t* ring, uint64_t* bar, int32_t* off, int consumed,
                                       uint64_t pol) {
    constexpr bool AWQ = FMT == kAWQ;
    constexpr int SB = 32 * (FMT == kQ8 ? 32 : 16) + 64;
    const int H = p.H, I = p.I, per = w.n1 + w.n2;
    while (w.nissued < w.total && w.nissued - consumed < kClInFlight) {
        const int k = w.nissued / per, r = w.nissued - k * per;
        const int wu = wl[g.cid + k * g.NC];
        const int e = ue[wu >> 16], q = wu & 15;
        const uint8_t* src;
        uint32_t bytes;
        if (r < w.n1) {
            int first, cnt;
            cl_gu_item<AWQ>(w, p.upi, g.NK1, r, first, cnt);
            if constexpr (AWQ) {
                // records (e, ut, half, kh): the CTA's unit tiles start at unit q KR + rank UPC
                const size_t base = ((size_t)e * (I / 16) + (q * g.KR + g.rank * g.UPC) / 16) * 2 * g.NK1;
                src = p.gu + (base + first) * kAwqGuRec;
                bytes = (uint32_t)cnt * kAwqGuRec;
            } else {
                const uint32_t ub = 2u * (p.rs1 + p.ss1);
                src = p.gu + ((size_t)e * I + q * g.KR + g.rank * g.UPC + first) * ub;
                bytes = ub * cnt;
            }
        } else {
            const int j = r - w.n1, sl = w.d_lo + j / w.per_slice, pc = j % w.per_slice;
            const int grow = g.rank * (g.RPC / 32) + sl;  // 32-row slice / block index in the expert
            if constexpr (AWQ) {
                const int k0 = q * g.KH + pc * p.kpi, nn = min(p.kpi, g.KH - pc * p.kpi);
                src = p.dn + (((size_t)e * (H / 32) + grow) * (I / kAwqK) + k0) * kAwqDnRec;
                bytes = (uint32_t)nn * kAwqDnRec;
            } else {
                const int k0 = q * g.KB + pc * p.kpi, nn = min(p.kpi, g.KB - pc * p.kpi);
                src = p.dn + (((size_t)e * (H / 32) + grow) * (I / 32) + k0) * SB;
                bytes = (uint32_t)nn * SB;
            }
        }
        int at;
        if (w.nissued == consumed) {
            at = 0;  // nothing in flight: every lane's reads of the ring are complete
        } else {
            const int tail = off[consumed % kClInFlight];
            if (w.head == tail) break;  // full up to the oldest item
            if (w.head > tail) {
                if (w.head + (int)bytes <= p.ring_bytes) at = w.head;
                else if ((int)bytes <= tail) at = 0;
                else break;
            } else {
                if (w.head + (int)bytes <= tail) at = w.head;
                else break;
            }
        }
        const int s = w.nissued % kClInFlight;
        off[s] = at;
        issue_copy(ring + at, src, bytes, &bar[s], pol);
        w.head = at + (int)bytes;
        ++w.nissued;
    }
}

template <int FMT, bool XBF, int TF>
__global__ void __launch_bounds__(kClThreads, 1) moe_decode_cl_kernel(const ClParams p) {
    constexpr bool Q4 = FMT == kQ4;
    constexpr bool AWQ = FMT == kAWQ;
    constexpr int BB = FMT == kQ8 ? 32 : 16;  // Q8/Q4 weight bytes per 32-block
    constexpr int SB = 32 * BB + 64;          // Q8/Q4 down row-slice record
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // TF > 0: the token count fixed at compile time (the one-token decode variant is a smaller
    // program); 0: p.T
    const int T = TF > 0 ? TF : p.T;
    const int TK = T * p.K, E = p.E, H = p.H, I = p.I;
    const int nb1 = H >> 5;
    const int cs = (int)cl_size(), rank = (int)cl_rank(), cid = (int)cl_id(), NC = (int)cl_count();
    const int RPC = H / cs;  // down rows of this CTA
    const int NK1 = H / kAwqK;
    // optional phase stamps (globaltimer ns), kept in shared memory and written out at the end so
    // that the stores do not wait behind the kernel's fences
    unsigned long long* dbg = p.dbg ? p.dbg + (size_t)blockIdx.x * kStamps : nullptr;
    __shared__ unsigned long long s_st[kStamps];
    auto stamp = [&](int i) {
        if (dbg && tid == 0) s_st[i] = global_ns();
    };
    auto flush_stamps = [&]() {
        if (dbg && tid == 0)
            #pragma unroll 1
            for (int i = 0; i < kStamps; ++i) dbg[i] = s_st[i];
    };
    if (dbg && tid == 0)
        #pragma unroll 1
        for (int i = 0; i < kStamps; ++i) s_st[i] = 0;
    stamp(0);

    RouteSmem rt = carve_route(reinterpret_cast<int32_t*>(smem), TK, E);
    int32_t* wl = reinterpret_cast<int32_t*>(smem + p.off_wl);  // work units: u << 16 | m0 << 4 | q
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_ring - 12 * kClWarps * kClInFlight);
    uint64_t* mybar = bars + warp * kClInFlight;
    int32_t* myoff = reinterpret_cast<int32_t*>(bars + kClWarps * kClInFlight) + warp * kClInFlight;  // item offsets
    uint8_t* myring = smem + p.off_ring + (size_t)warp * p.ring_bytes;
    __shared__ int s_nwu, s_q;
    __shared__ unsigned int s_last;

    // ---------------- routing, work units, token staging ----------------
    if (tid == 0) s_last = 0u;
    if (lane == 0)
        #pragma unroll 1
        for (int s = 0; s < kClInFlight; ++s) mbar_init(&mybar[s], 1);
    // Programmatic dependent launch: the next kernel on the stream may be scheduled now (it
    // waits for this grid's completion before it reads anything); this grid waits here for
    // the kernel before it, which may have written the inputs, before its first read.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (warp == kClWarps - 1) {
        route_warp(p.ids, TK, p.K, E, p.e_off, p.emap, p.emap_n, rt, lane);
        // pieces: each expert in slices of at most T positions (one unless ids repeat inside a
        // token); lane l owns the contiguous experts [l cu, l cu + cu), a warp scan gives their
        // first piece
        const int U = *rt.nuniq, cu = (U + 31) >> 5;
        int loc = 0;
        #pragma unroll 1
        for (int k = 0; k < cu; ++k) {
            const int u = lane * cu + k;
            if (u < U) loc += (rt.ucnt[u] + T - 1) / T;
        }
        int incl = loc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        const int P = __shfl_sync(0xffffffffu, incl, 31);
        // Q minimises the busiest cluster's share ceil(P Q / NC) / Q, ties to the smaller Q
        int bq = 1, bnum = 0x7fffffff, bden = 1;
        #pragma unroll 1
        for (int lq = 0; (1 << lq) <= kClMaxQ; ++lq) {
            if (!((p.qmask >> lq) & 1)) continue;
            const int q = 1 << lq, num = (P * q + NC - 1) / NC;  // share = num / q
            if ((int64_t)num * bden < (int64_t)bnum * q) { bq = q; bnum = num; bden = q; }
        }
        int w0 = (incl - loc) * bq;
        #pragma unroll 1
        for (int k = 0; k < cu; ++k) {
            const int u = lane * cu + k;
            if (u >= U) break;
            #pragma unroll 1
            for (int m0 = 0; m0 < rt.ucnt[u]; m0 += T)
                for (int q = 0; q < bq; ++q) wl[w0++] = (u << 16) | (m0 << 4) | q;
        }
        if (lane == 0) {
            s_nwu = P * bq;
            s_q = bq;
        }
    } else {
        if constexpr (AWQ) {
            // tokens as 16-bit rows [T][H + 8] (padded against bank conflicts)
            // and the per-64 sums of each row [T][H/64]: eight neighbouring lanes hold one
            // 64-run (the stride and the trip count are multiples of 8, so a run is never split)
            uint16_t* xs = reinterpret_cast<uint16_t*>(smem + p.off_x);
            float* xsum_w = reinterpret_cast<float*>(smem + p.off_x + (size_t)T * (H + 8) * 2);
            const uint16_t* xg = static_cast<const uint16_t*>(p.x);
            #pragma unroll 1
            for (int i = tid; i < T * (H / 8); i += kClThreads - 32) {
                const int t = i / (H / 8), k8 = i - t * (H / 8);
                const uint4 v = __ldg(reinterpret_cast<const uint4*>(xg + (size_t)t * H) + k8);
                *reinterpret_cast<uint4*>(xs + (size_t)t * (H + 8) + 8 * k8) = v;
                float sv = 0.f;
                const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    sv += from16<XBF>((uint16_t)(w4[j] & 0xffffu)) + from16<XBF>((uint16_t)(w4[j] >> 16));
                const unsigned am = __activemask();
                sv += __shfl_xor_sync(am, sv, 1);
                sv += __shfl_xor_sync(am, sv, 2);
                sv += __shfl_xor_sync(am, sv, 4);
                if ((k8 & 7) == 0) xsum_w[t * NK1 + (k8 >> 3)] = sv;
            }
        } else {
            int8_t* xq = reinterpret_cast<int8_t*>(smem + p.off_x);
            float* xd = reinterpret_cast<float*>(xq + (size_t)T * H);
            int32_t* xsm = reinterpret_cast<int32_t*>(xd + (size_t)T * nb1);
            quant_x_quad<Q4>(static_cast<const uint8_t*>(p.x), p.act_bf16, T, H, xq, xd, xsm, tid, kClThreads - 32);
        }
    }
    stamp(12);
    fence_barrier_init();
    __syncthreads();
    stamp(13);
    float* xsum = nullptr;  // AWQ: per-64 sums of the token rows [T][H/64]
    if constexpr (AWQ) {
        xsum = reinterpret_cast<float*>(smem + p.off_x + (size_t)T * (H + 8) * 2);
    }
    stamp(1);
    const int NW = s_nwu, Q = s_q;
    const int n_my = cid < NW ? (NW - cid + NC - 1) / NC : 0;

    if (p.meta && cid == 0 && rank == 0) {  // the separate combine kernel reads Q and the scatter map
        if (tid == 0) p.meta[0] = Q;
        #pragma unroll 1
        for (int i = tid; i < TK; i += kClThreads) p.meta[1 + i] = rt.smap[i];
    }
    if (NW == 0) {  // no routed pair on this engine: the output is zero (q8_gemm.cpp:328-333)
        if (cid == 0 && !p.meta)
            #pragma unroll 1
            for (int idx = tid; idx < T * RPC; idx += kClThreads) {
                const int t = idx / RPC, n = rank * RPC + idx % RPC;
                const size_t o = (size_t)t * H + n;
                if (p.out_kind == 2) reinterpret_cast<float*>(p.y)[o] = 0.f;
                else if (p.out_kind == 1) reinterpret_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(0.f);
                else reinterpret_cast<__half*>(p.y)[o] = __float2half_rn(0.f);
            }
        return;
    }
    if (n_my == 0) return;  // more clusters than work units
    cl_arrive_relaxed();    // start phase: every CTA of the cluster runs before any DSMEM store

    // geometry of one work unit under Q
    const int KR = I / Q;          // K-range (units) of a work unit
    const int UPC = KR / cs;       // gate_up units of this CTA
    const int KB = KR >> 5;        // Q8/Q4: 32-column blocks of the K-range
    const int KH = KR / kAwqK;     // AWQ: 64-k records of the K-range

    // ---------------- this warp's items ----------------
    ClGeo geo;
    geo.NC = NC; geo.cid = cid; geo.rank = rank; geo.n_my = n_my; geo.Q = Q;
    geo.KR = KR; geo.UPC = UPC; geo.KB = KB; geo.KH = KH; geo.RPC = RPC; geo.NK1 = NK1;
    __shared__ ClWarp wst[kClWarps];
    ClWarp& W = wst[warp];
    if (lane == 0) {
        if constexpr (AWQ) {
            const int N1 = 2 * (UPC / 16) * NK1;
            W.g_lo = range_lo(warp, N1);
            W.g_n = range_lo(warp + 1, N1) - W.g_lo;
            int n1 = 0;  // runs of <= upi records inside each row tile
            #pragma unroll 1
            for (int it = W.g_lo; it < W.g_lo + W.g_n;) {
                const int rti = it / NK1, end = min(W.g_lo + W.g_n, (rti + 1) * NK1);
                n1 += (end - it + p.upi - 1) / p.upi;
                it = end;
            }
            W.n1 = n1;
            W.per_slice = (KH + p.kpi - 1) / p.kpi;
        } else {
            W.g_lo = range_lo(warp, UPC);
            W.g_n = range_lo(warp + 1, UPC) - W.g_lo;
            W.n1 = (W.g_n + p.upi - 1) / p.upi;
            W.per_slice = (KB + p.kpi - 1) / p.kpi;
        }
        const int nsl = RPC / 32;  // 32-row slices (Q8/Q4) / row blocks (AWQ) of this CTA
        W.d_lo = range_lo(warp, nsl);
        W.d_n = range_lo(warp + 1, nsl) - W.d_lo;
        W.n2 = W.d_n * W.per_slice;
        W.total = n_my * (W.n1 + W.n2);
        W.nissued = 0;
        W.head = 0;
    }
    __syncwarp();
    stamp(14);
    const int n1 = W.n1, d_lo = W.d_lo, d_n = W.d_n, per_slice = W.per_slice;
    const int dpi = p.kpi;  // records / blocks per down item
    const uint64_t pol = (p.flags & kFlagEvictFirst) ? l2_evict_first_policy() : 0ull;
    stamp(15);
    if (lane == 0) cl_top_up<FMT>(p, geo, W, wl, rt.ue, myring, mybar, myoff, 0, pol);
    __syncwarp();
    stamp(6);

    bool ok = true;
    int consumed = 0;
    auto wait_item = [&]() -> const uint8_t* {
        const int s = consumed % kClInFlight;
        if (!mbar_wait(&mybar[s], (uint32_t)(consumed / kClInFlight) & 1u)) {
            if (ok) set_err(p.err, kErrFullWait);
            ok = false;
        }
        if (consumed == 0) stamp(2);
        return myring + myoff[s];
    };
    auto done_item = [&]() {
        ++consumed;
        __syncwarp();  // every lane's reads of the item are complete before its space is reused
        if (lane == 0) cl_top_up<FMT>(p, geo, W, wl, rt.ue, myring, mybar, myoff, consumed, pol);
        __syncwarp();
    };
    auto gu_item = [&](int i, int& first, int& cnt) { cl_gu_item<AWQ>(W, p.upi, NK1, i, first, cnt); };

    const int cap = T;  // positions per work unit
    const bool sbf = p.scale_bf16 != 0;
    uint8_t* hbuf = smem + p.off_h;  // Q8/Q4 fp32 [cap][KR]; AWQ 16-bit [cap][KR + 8]
    uint8_t* hl = smem + p.off_p;    // this CTA's h slice [cap][UPC] (fp32 / 16-bit)
    float* outs = reinterpret_cast<float*>(smem + p.off_out);  // [cap][RPC]
    uint8_t* hqb = smem + p.off_hq;  // Q8/Q4: q [cap][KR] | d | s; AWQ: GU slots, then h sums

    // -------- gate_up of work unit k into hl --------
    auto gate_up = [&](int k) {
        const int wu = wl[cid + k * NC];
        const int u = wu >> 16, m0 = (wu >> 4) & 0xfff;
        const int ps = rt.ups[u] + m0, mc = min(cap, rt.ucnt[u] - m0);
        if constexpr (AWQ) {
            const uint16_t* xs = reinterpret_cast<const uint16_t*>(smem + p.off_x);
            const int g = lane >> 2, c = lane & 3;
            const int tg = g < mc ? rt.tok[ps + g] / p.K : -1;
            const int t0 = 2 * c < mc ? rt.tok[ps + 2 * c] / p.K : 0;
            const int t1 = 2 * c + 1 < mc ? rt.tok[ps + 2 * c + 1] / p.K : 0;
            const int N1 = 2 * (UPC / 16) * NK1;
            const int nslot = (kClWarps + 2 * (UPC / 16) - 1) / (2 * (UPC / 16)) + 1;  // >= warps per row tile
            float* P1 = reinterpret_cast<float*>(hqb);  // [row tiles][nslot][16 rows][cap positions]
            float tot[4] = {0.f, 0.f, 0.f, 0.f};
            int cur = -1;
            auto flush = [&]() {
                if (cur < 0) return;
                const int slot = warp - item_owner(cur * NK1, N1);
                float* dst = P1 + ((size_t)cur * nslot + slot) * 16 * cap;
                if (2 * c < mc) {
                    dst[g * cap + 2 * c] = tot[0];
                    dst[(g + 8) * cap + 2 * c] = tot[2];
                }
                if (2 * c + 1 < mc) {
                    dst[g * cap + 2 * c + 1] = tot[1];
                    dst[(g + 8) * cap + 2 * c + 1] = tot[3];
                }
                tot[0] = tot[1] = tot[2] = tot[3] = 0.f;
            };
            #pragma unroll 1
            for (int i = 0; i < n1; ++i) {
                const uint8_t* slot = wait_item();
                int first, cnt;
                gu_item(i, first, cnt);
                const int rti = first / NK1;
                if (rti != cur) { flush(); cur = rti; }
                #pragma unroll 1
                for (int r = 0; r < cnt; ++r) {
                    const int kh = first + r - rti * NK1;
                    const uint8_t* rec = slot + (size_t)r * kAwqGuRec;
                    const uint16_t* brow = tg >= 0 ? xs + (size_t)tg * (H + 8) + kh * kAwqK : nullptr;
                    const float x0 = xsum[t0 * NK1 + kh], x1 = xsum[t1 * NK1 + kh];
                    awq_mma64<XBF>(rec, reinterpret_cast<const uint16_t*>(rec + 512), rec + 544, brow, x0, x1, lane,
                                   tot);
                }
                done_item();
            }
            flush();
            __syncthreads();
            // h[m][j] = SiLU(gate) * up over the CTA's units, slots summed in warp order
            uint16_t* hl16 = reinterpret_cast<uint16_t*>(hl);
            #pragma unroll 1
            for (int idx = tid; idx < mc * UPC; idx += kClThreads) {
                const int m = idx / UPC, j = idx - m * UPC;
                const int ut = j >> 4, r = j & 15;
                float gu2[2];
                #pragma unroll 1
                for (int half = 0; half < 2; ++half) {
                    const int rti = 2 * ut + half;
                    const int ns = item_owner(rti * NK1 + NK1 - 1, N1) - item_owner(rti * NK1, N1) + 1;
                    float acc = 0.f;
                    #pragma unroll 1
                    for (int sl = 0; sl < ns; ++sl) acc += P1[((size_t)rti * nslot + sl) * 16 * cap + r * cap + m];
                    gu2[half] = acc;
                }
                const float hv = silu_mul(gu2[0], gu2[1]);
                if (!XBF && !(fabsf(hv) <= 65504.f)) set_err(p.err, kErrRange);
                hl16[idx] = to16<XBF>(hv);
            }
        } else {
            const int8_t* xq = reinterpret_cast<const int8_t*>(smem + p.off_x);
            const float* xd = reinterpret_cast<const float*>(xq + (size_t)T * H);
            const int32_t* xsm = reinterpret_cast<const int32_t*>(xd + (size_t)T * nb1);
            float* hlf = reinterpret_cast<float*>(hl);
            const int ub = 2 * (p.rs1 + p.ss1);
            #pragma unroll 1
            for (int i = 0; i < n1; ++i) {
                const uint8_t* slot = wait_item();
                int first, cnt;
                gu_item(i, first, cnt);
                #pragma unroll 1
                for (int uu = 0; uu < cnt; ++uu) {  // one unit at a time, all lanes over its blocks
                    const uint8_t* rec = slot + (size_t)uu * ub;
                    const uint8_t* qg = rec;
                    const uint8_t* qu = rec + p.rs1;
                    const uint16_t* sgate = reinterpret_cast<const uint16_t*>(rec + 2 * p.rs1);
                    const uint16_t* sup = reinterpret_cast<const uint16_t*>(rec + 2 * p.rs1 + p.ss1);
                    const int jl = first + uu;  // CTA-local unit
#pragma unroll 1
                    for (int m = 0; m < mc; ++m) {  // one token at a time: small code, weights from smem
                        const int t = rt.tok[ps + m] / p.K;
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
                        if (lane == 0) hlf[(size_t)m * UPC + jl] = silu_mul(ag, au);
                    }
                }
                done_item();
            }
        }
        __syncthreads();
    };

    // -------- this CTA's h slice of work unit k into h buffer `buf` of every cluster CTA --------
    auto push = [&](int k, int buf) {
        const int wu = wl[cid + k * NC];
        const int u = wu >> 16, m0 = (wu >> 4) & 0xfff;
        const int mc = min(cap, rt.ucnt[u] - m0);
        uint8_t* hb = hbuf + (size_t)buf * p.hbuf_bytes;
        if constexpr (AWQ) {
            const uint32_t* src = reinterpret_cast<const uint32_t*>(hl);  // pairs of 16-bit values
            const int np = UPC / 2;
            #pragma unroll 1
            for (int idx = tid; idx < cs * mc * np; idx += kClThreads) {
                const int qr = idx / (mc * np), rem = idx - qr * (mc * np);
                const int m = rem / np, pr = rem - m * np;
                uint16_t* dst = reinterpret_cast<uint16_t*>(hb) + (size_t)m * (KR + 8) + rank * UPC + 2 * pr;
                st_cl_u32(cl_map(dst, (uint32_t)qr), src[m * np + pr]);
            }
        } else {
            const float4* src = reinterpret_cast<const float4*>(hl);
            const int nv = UPC / 4;
            #pragma unroll 1
            for (int idx = tid; idx < cs * mc * nv; idx += kClThreads) {
                const int qr = idx / (mc * nv), rem = idx - qr * (mc * nv);
                const int m = rem / nv, v = rem - m * nv;
                float* dst = reinterpret_cast<float*>(hb) + (size_t)m * KR + rank * UPC + 4 * v;
                st_cl_v4(cl_map(dst, (uint32_t)qr), src[m * nv + v]);
            }
        }
    };

    // -------- down rows of work unit k over its K-range, from h buffer `buf`, into `part` --------
    auto down = [&](int k, int buf) {
        const int wu = wl[cid + k * NC];
        const int u = wu >> 16, m0 = (wu >> 4) & 0xfff, q = wu & 15;
        const int ps = rt.ups[u] + m0, mc = min(cap, rt.ucnt[u] - m0);
        const uint8_t* hb = hbuf + (size_t)buf * p.hbuf_bytes;
        if constexpr (AWQ) {
            const uint16_t* h16 = reinterpret_cast<const uint16_t*>(hb);
            float* hsum = reinterpret_cast<float*>(hqb);  // [cap][KH] per-64 sums of h (GU slots are free)
            #pragma unroll 1
            for (int i = warp; i < mc * KH; i += kClWarps) {
                const int m = i / KH, kh = i - m * KH;
                const uint16_t* r = h16 + (size_t)m * (KR + 8) + kh * kAwqK;
                const float sv = warp_sum64<XBF>(r, lane);
                if (lane == 0) hsum[i] = sv;
            }
            __syncthreads();
            const int g = lane >> 2, c = lane & 3;
            const uint16_t* hrow = g < mc ? h16 + (size_t)g * (KR + 8) : nullptr;
            const int c0 = min(2 * c, mc - 1), c1 = min(2 * c + 1, mc - 1);
            #pragma unroll 1
            for (int sl = 0; sl < d_n; ++sl) {  // a 32-row block, its whole K-range in this warp
                float tot[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
                #pragma unroll 1
                for (int pc = 0; pc < per_slice; ++pc) {
                    const uint8_t* slot = wait_item();
                    const int nn = min(dpi, KH - pc * dpi);
                    #pragma unroll 1
                    for (int r = 0; r < nn; ++r) {
                        const int kh = pc * dpi + r;  // K-range local
                        const uint8_t* rec = slot + (size_t)r * kAwqDnRec;
                        const uint16_t* brow = hrow ? hrow + kh * kAwqK : nullptr;
                        const float x0 = hsum[c0 * KH + kh], x1 = hsum[c1 * KH + kh];
#pragma unroll
                        for (int tt = 0; tt < 2; ++tt) {
                            const uint8_t* qt = rec + tt * 512;
                            const uint16_t* sc = reinterpret_cast<const uint16_t*>(rec + 1024) + 16 * tt;
                            const uint8_t* zp = rec + 1088 + 16 * tt;
                            awq_mma64<XBF>(qt, sc, zp, brow, x0, x1, lane, tot[tt]);
                        }
                    }
                    done_item();
                }
                const int rowb = (d_lo + sl) * 32;  // CTA-local first row of the block
#pragma unroll
                for (int tt = 0; tt < 2; ++tt) {
                    const int r0 = rowb + 16 * tt + g;
                    if (2 * c < mc) {
                        outs[(size_t)(2 * c) * RPC + r0] = tot[tt][0];
                        outs[(size_t)(2 * c) * RPC + r0 + 8] = tot[tt][2];
                    }
                    if (2 * c + 1 < mc) {
                        outs[(size_t)(2 * c + 1) * RPC + r0] = tot[tt][1];
                        outs[(size_t)(2 * c + 1) * RPC + r0 + 8] = tot[tt][3];
                    }
                }
            }
        } else {
            const float* hf = reinterpret_cast<const float*>(hb);
            int8_t* hq = reinterpret_cast<int8_t*>(hqb);
            float* hd = reinterpret_cast<float*>(hq + (size_t)cap * KR);
            int32_t* hs = reinterpret_cast<int32_t*>(hd + (size_t)cap * KB);
            requant_smem<Q4>(hf, mc, KR, hq, hd, hs, tid);
            __syncthreads();
            #pragma unroll 1
            for (int sl = 0; sl < d_n; ++sl) {  // lane = row of the 32-row slice
                float acc[8];
#pragma unroll
                for (int m = 0; m < 8; ++m) acc[m] = 0.f;
                #pragma unroll 1
                for (int pc = 0; pc < per_slice; ++pc) {
                    const uint8_t* slot = wait_item();
                    const int nn = min(dpi, KB - pc * dpi);
#pragma unroll 1
                    for (int m = 0; m < mc; ++m) {  // one token at a time: small code
                        float am = 0.f;
                        #pragma unroll 1
                        for (int r = 0; r < nn; ++r) {
                            const int b = pc * dpi + r;  // K-range local 32-block
                            const uint8_t* rec = slot + (size_t)r * SB;
                            const uint4* w = reinterpret_cast<const uint4*>(rec + lane * BB);
                            const float dw = scale_to_f32(reinterpret_cast<const uint16_t*>(rec + 32 * BB)[lane], sbf);
                            const uint4* a = reinterpret_cast<const uint4*>(hq + (size_t)m * KR + b * 32);
                            const int is = block_dot<Q4>(w, a, Q4 ? hs[m * KB + b] : 0);
                            am += ((float)is * dw) * hd[m * KB + b];
                        }
#pragma unroll
                        for (int mm = 0; mm < 8; ++mm)
                            if (mm == m) acc[mm] += am;
                    }
                    done_item();
                }
                const int row = (d_lo + sl) * 32 + lane;
#pragma unroll
                for (int m = 0; m < 8; ++m)
                    if (m < mc) outs[(size_t)m * RPC + row] = acc[m];
            }
        }
        __syncthreads();
        // the routed pairs' partial rows of this CTA into `part` [(pos * Q + q)][H] (coalesced)
        #pragma unroll 1
        for (int idx = tid; idx < mc * RPC; idx += kClThreads) {
            const int m = idx / RPC, r = idx - m * RPC;
            __stcg(p.part + ((size_t)(ps + m) * Q + q) * H + rank * RPC + r, outs[idx]);
        }
        __syncthreads();  // outs / hq are reused by the next work unit
    };

    // ---------------- work units ----------------
    #pragma unroll 1
    for (int k = 0; k < n_my; ++k) {
        gate_up(k);
        if (k == 0) stamp(3);
        cl_wait();  // k == 0: the start phase; else: every CTA finished unit k-1's down (the h buffer)
        if (k == 0) stamp(4);
        push(k, 0);
        cl_arrive();
        cl_wait();  // unit k's whole K-range of h is in place
        if (k == 0) stamp(5);
        down(k, 0);
        if (k + 1 < n_my) cl_arrive();
    }
    stamp(7);

    // drain: a warp that stopped early still waits (bounded) for its copies in flight
    if (!ok && lane == 0)
        #pragma unroll 1
        for (int i = consumed; i < W.nissued; ++i) mbar_wait(&mybar[i % kClInFlight], (uint32_t)(i / kClInFlight) & 1u);

    // ---------------- combine ----------------
    if (p.meta) {  // the combine runs as its own kernel (cl_combine_kernel) after this grid
        flush_stamps();
        return;
    }
    const int RB = H / kClRowBlocks;                // rows per combine block
    const int nblk = RPC / RB, blk0 = rank * nblk;  // this CTA's blocks
    // the CTA barrier orders every thread's partial stores before the counter updates, whose
    // release (cumulative) publishes them at gpu scope
    __syncthreads();
    if (tid < nblk) {
        const unsigned int old = atom_add_acq_rel_gpu(p.cnt + blk0 + tid, (unsigned int)n_my);
        if (old + (unsigned int)n_my == (unsigned int)NW) atomicOr(&s_last, 1u << tid);
    }
    if (tid == 0) stamp(8);
    __syncthreads();
    const unsigned int last = s_last;
    if (!last) {
        flush_stamps();
        return;
    }
    stamp(11);
    // the completed blocks' elements, one per thread (consecutive threads: consecutive rows, so
    // every load is coalesced): for each routed pair in k order, its Q K-range partials, all
    // loads of 4 pairs in flight together, summed in q order, weighted and accumulated in k order
    const int nl = __popc(last);
    #pragma unroll 1
    for (int idx = tid; idx < nl * T * RB; idx += kClThreads) {
        const int bi = idx / (T * RB), rem = idx - bi * (T * RB);
        int b = 0;
        #pragma unroll 1
        for (int seen = -1; ; ++b)
            if ((last >> b) & 1u) { if (++seen == bi) break; }
        const int t = rem / RB, n = (blk0 + b) * RB + rem % RB;
        float acc = 0.f;
        #pragma unroll 1
        for (int k0 = 0; k0 < p.K; k0 += 4) {
            int pos[4];
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                pos[j] = k0 + j < p.K ? rt.smap[t * p.K + k0 + j] : -1;
                v[j] = 0.f;
            }
            #pragma unroll 1
            for (int q0 = 0; q0 < Q; q0 += 4) {
                float a[4][4];
#pragma unroll
                for (int j = 0; j < 4; ++j)
#pragma unroll
                    for (int qq = 0; qq < 4; ++qq)
                        a[j][qq] = (pos[j] >= 0 && q0 + qq < Q)
                                       ? __ldcg(p.part + ((size_t)pos[j] * Q + q0 + qq) * H + n) : 0.f;
#pragma unroll
                for (int j = 0; j < 4; ++j) v[j] += ((a[j][0] + a[j][1]) + (a[j][2] + a[j][3]));
            }
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (pos[j] >= 0) acc += p.tw[t * p.K + k0 + j] * v[j];
        }
        const size_t o = (size_t)t * H + n;
        if (p.out_kind == 2) reinterpret_cast<float*>(p.y)[o] = acc;
        else if (p.out_kind == 1) reinterpret_cast<__nv_bfloat16*>(p.y)[o] = __float2bfloat16_rn(acc);
        else reinterpret_cast<__half*>(p.y)[o] = __float2half_rn(acc);
    }
    if (tid < nblk && ((last >> tid) & 1u)) p.cnt[blk0 + tid] = 0u;  // the next launch starts from zero
    stamp(9);
    flush_stamps();
}

// The combine as a kernel of its own (launched right after moe_decode_cl_kernel, with
// programmatic dependent launch): one thread per output element (t, n), consecutive threads on
// consecutive rows (coalesced); for each routed pair in k order its Q K-range partials, summed
// in q order, weighted, accumulated in k order and cast (q8_gemm.cpp:593-641).  Deterministic.
__global__ void __launch_bounds__(256) cl_combine_kernel(const float* part, const int32_t* meta, const float* tw,
                                                         int T, int K, int H, void* y, int out_kind) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the decode grid has completed
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= T * H) return;
    const int t = idx / H, n = idx - t * H;
    const int Q = __ldcg(meta);
    const int32_t* smap = meta + 1;
    float acc = 0.f;
    #pragma unroll 1
    for (int k0 = 0; k0 < K; k0 += 4) {
        int pos[4];
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            pos[j] = k0 + j < K ? __ldcg(smap + t * K + k0 + j) : -1;
            v[j] = 0.f;
        }
        #pragma unroll 1
        for (int q0 = 0; q0 < Q; q0 += 4) {
            float a[4][4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int qq = 0; qq < 4; ++qq)
                    a[j][qq] = (pos[j] >= 0 && q0 + qq < Q) ? __ldcg(part + ((size_t)pos[j] * Q + q0 + qq) * H + n) : 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] += ((a[j][0] + a[j][1]) + (a[j][2] + a[j][3]));
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (pos[j] >= 0) acc += tw[t * K + k0 + j] * v[j];
    }
    const size_t o = (size_t)t * H + n;
    if (out_kind == 2) reinterpret_cast<float*>(y)[o] = acc;
    else if (out_kind == 1) reinterpret_cast<__nv_bfloat16*>(y)[o] = __float2bfloat16_rn(acc);
    else reinterpret_cast<__half*>(y)[o] = __float2half_rn(acc);
}

}  // namespace moe
