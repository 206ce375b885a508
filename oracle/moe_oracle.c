/*
 * TEST INFRASTRUCTURE ONLY -- the parity checker, never the product.
 *
 * Plain-C restatement of the reference CPU fused-MoE algorithm
 * (Qeeweew/MoE-Ascend-Opt, directory Int8-gemm/).  Only tests/, the smoke
 * check and bench.py's cpu_baseline leg may load this library.  It is pinned
 * against the reference engine itself (compiled unmodified from its sources
 * by oracle/Makefile `ref`) through the golden fixtures in tests/golden/.
 *
 * Each function names the reference lines it restates.  Scalar, single
 * threaded, fp32 arithmetic in the reference's order of operations.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QK 32

/* ------------------------------------------------------------------ */
/* scalar conversions                                                  */
/* ------------------------------------------------------------------ */
static float f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1f, m = h & 0x3ff, u;
    if (e == 0) {
        if (m == 0) { u = s; }
        else {  /* subnormal: renormalise */
            int sh = 0;
            while (!(m & 0x400)) { m <<= 1; ++sh; }
            m &= 0x3ff;
            u = s | ((uint32_t)(113 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        u = s | 0x7f800000u | (m << 13);
    } else {
        u = s | ((e + 127 - 15) << 23) | (m << 13);
    }
    float f; memcpy(&f, &u, 4); return f;
}

static float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16; float f; memcpy(&f, &u, 4); return f;
}

/* round-to-nearest-even fp32 -> fp16 bits (the c10::Half conversion result) */
static uint16_t f32_to_f16(float f) {
    uint32_t x; memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);           /* rounds to inf */
    if (ax < 0x38800000u) {                                              /* fp16 subnormal/zero */
        float af; memcpy(&af, &ax, 4);
        uint32_t q = (uint32_t)nearbyintf(af * 16777216.0f);             /* units of 2^-24, RNE */
        return (uint16_t)(sign | q);
    }
    /* normal: rebias exponent by (15-127), round the 13 dropped bits to nearest even */
    uint32_t mant_odd = (ax >> 13) & 1u;
    ax += ((uint32_t)(15 - 127) << 23) + 0xfffu + mant_odd;
    return (uint16_t)(sign | (ax >> 13));
}

static uint16_t f32_to_bf16(float f) {
    uint32_t x; memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

static float scale_to_f32(uint16_t v, int scale_is_bf16) {
    return scale_is_bf16 ? bf16_to_f32(v) : f16_to_f32(v);
}

static int8_t sat_rne_i8(float v) {
    /* vcvtnq_s32_f32 then vqmovn_s32 / vqmovn_s16: RNE, saturate to int8 */
    if (v != v) return 0;
    float r = nearbyintf(v);
    if (r > 127.0f) return 127;
    if (r < -128.0f) return -128;
    return (int8_t)r;
}


/*
 * exp(x) as the reference's 4-wide SiLU path computes it: the ggml
 * range-reduced polynomial of Int8-gemm/vec_simd.h:9-33 (ggml_v_expf),
 * restated per lane with fmaf for its fused multiply-adds.  The vector
 * version's "any lane out of range" branch gives the same per-lane result
 * as this per-lane select.  Used so the oracle's SiLU matches the
 * reference bit for bit (the scalar tail at vec_simd.h:58-62 uses expf,
 * reached only when I is not a multiple of 4).
 */
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float ggml_expf_lane(float x) {
    const float r = 0x1.8p23f;
    const float z = fmaf(x, 0x1.715476p+0f, r);
    const float n = z - r;
    const float b = fmaf(-n, 0x1.7f7d1cp-20f, fmaf(-n, 0x1.62e4p-1f, x));
    const uint32_t e = f2u(z) << 23;
    const float k = u2f(e + f2u(1.0f));
    const int c = fabsf(n) > 126.0f;
    const float u = b * b;
    const float j = fmaf(fmaf(fmaf(0x1.0e4020p-7f, b, 0x1.573e2ep-5f), u,
                              fmaf(0x1.555e66p-3f, b, 0x1.fffdb6p-2f)),
                         u, 0x1.ffffecp-1f * b);
    if (!c) return fmaf(k, j, k);
    const uint32_t d = (n <= 0.0f) ? 0x82000000u : 0u;
    const float s1 = u2f(d + 0x7f000000u);
    const float s2 = u2f(e - d);
    if (fabsf(n) > 192.0f) return s1 * s1;
    return fmaf(s2, j, s2) * s1;
}

/* SiLU(gate) * up over one [gate | up] row, vec_simd.h:36-64. */
static void silu_and_mul_row(float* row, int I) {
    const int nvec = I & ~3;
    for (int j = 0; j < I; ++j) {
        const float g = row[j];
        const float eg = (j < nvec) ? ggml_expf_lane(-g) : expf(-g);
        row[j] = row[I + j] * (g / (1.0f + eg));
    }
}

/* ------------------------------------------------------------------ */
/* exported helpers                                                    */
/* ------------------------------------------------------------------ */
void orc_f32_to_bf16(const float* in, uint16_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = f32_to_bf16(in[i]);
}
void orc_f32_to_f16(const float* in, uint16_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = f32_to_f16(in[i]);
}

/*
 * Stable counting sort of the (t,k) routing pairs by expert.
 * Restates Int8-gemm/moe_common.cpp:146-184 (preprocess_moe_routing_template):
 * counts over valid ids, exclusive scan into starts[E+1], then positions in
 * (t,k) order; an id outside [0,E) gets scatter_map = -1 and no position.
 * token_map holds (t,k) pairs, two int32 per position.
 * Returns the number of valid pairs.
 */
int orc_route_preprocess(int E, int K, int T, const int32_t* ids,
                         int32_t* counts, int32_t* starts,
                         int32_t* token_map, int32_t* scatter_map) {
    for (int e = 0; e < E; ++e) counts[e] = 0;
    for (int t = 0; t < T; ++t)
        for (int k = 0; k < K; ++k) {
            int e = ids[t * K + k];
            if (e >= 0 && e < E) counts[e]++;
        }
    starts[0] = 0;
    for (int e = 0; e < E; ++e) starts[e + 1] = starts[e] + counts[e];
    int32_t* cur = (int32_t*)calloc((size_t)E + 1, sizeof(int32_t));
    for (int t = 0; t < T; ++t)
        for (int k = 0; k < K; ++k) {
            int e = ids[t * K + k];
            if (e >= 0 && e < E) {
                int pos = starts[e] + cur[e]++;
                token_map[2 * pos] = t;
                token_map[2 * pos + 1] = k;
                scatter_map[t * K + k] = pos;
            } else {
                scatter_map[t * K + k] = -1;
            }
        }
    free(cur);
    return starts[E];
}

/*
 * One Q8_0 block: Int8-gemm/gemm_kernels.cpp:25-58 (quantize_block_q8_0).
 * amax over 32 values, d = amax/127, id = d != 0 ? 1/d : 0,
 * q = saturate_int8(round_nearest_even(x * id)).  d is returned in fp32.
 * The reference is built with -ffast-math (Int8-gemm/setup.py:21), under which
 * the compiler turns `amax / 127.0f` into `amax * (1.0f / 127.0f)`; this
 * restatement uses that product, which is what the reference's binary computes
 * (checked bit for bit against the reference objects).
 */
float orc_quantize_block_q8_0(const float* x, int8_t* qs) {
    float amax = 0.0f;
    for (int j = 0; j < QK; ++j) { float a = fabsf(x[j]); if (a > amax) amax = a; }
    const float d = amax * (1.0f / 127.0f);
    const float id = (d != 0.0f) ? 1.0f / d : 0.0f;
    for (int j = 0; j < QK; ++j) qs[j] = sat_rne_i8(x[j] * id);
    return d;
}

/* Activation rows -> Q8_0 with fp32 scales (stage A, Int8-gemm/q8_gemm.cpp:360-377). */
void orc_quantize_rows_q8_0_f32scale(const float* x, int64_t rows, int64_t cols,
                                     int8_t* qs, float* d) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b = 0; b < cols / QK; ++b)
            d[r * (cols / QK) + b] = orc_quantize_block_q8_0(x + r * cols + b * QK, qs + r * cols + b * QK);
}

/* Weight rows -> Q8_0 with fp16 scales (Int8-gemm/q8_gemm.cpp:197-260, scale cast at gemm_kernels.cpp:57). */
void orc_quantize_weight_q8_0(const float* w, int64_t rows, int64_t cols,
                              int8_t* qs, uint16_t* d_f16) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b = 0; b < cols / QK; ++b) {
            float d = orc_quantize_block_q8_0(w + r * cols + b * QK, qs + r * cols + b * QK);
            d_f16[r * (cols / QK) + b] = f32_to_f16(d);
        }
}

/*
 * Harness-side Q4_0 weight quantizer (the reference has none; online Q4_0 is
 * rejected at Int8-gemm/nanovllm_ops.cpp:360-363).  Per block of 32 along K:
 * d = amax/7 stored fp16, q = clamp(rne(w * (1/d)), -8, 7) + 8, packed
 * sequentially 8 nibbles per uint32: element k of a row sits in word k/8 at
 * bits 4*(k%8), value nibble-8 -- the input contract the reference's
 * repack_B_q4_0 consumes (Int8-gemm/gemm_kernels.cpp:510-579,
 * Int8-gemm/test/fused_moe_cpu_int4.py:52-71).
 */
void orc_quantize_weight_q4_0(const float* w, int64_t rows, int64_t cols,
                              uint32_t* qs, uint16_t* d_f16) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b = 0; b < cols / QK; ++b) {
            const float* x = w + r * cols + b * QK;
            float amax = 0.0f;
            for (int j = 0; j < QK; ++j) { float a = fabsf(x[j]); if (a > amax) amax = a; }
            const float d = amax / 7.0f;
            const float id = (d != 0.0f) ? 1.0f / d : 0.0f;
            uint32_t* wq = qs + r * (cols / 8) + b * 4;
            for (int j = 0; j < 4; ++j) wq[j] = 0;
            for (int j = 0; j < QK; ++j) {
                float v = nearbyintf(x[j] * id);
                if (v > 7.0f) v = 7.0f;
                if (v < -8.0f) v = -8.0f;
                uint32_t nib = (uint32_t)((int)v + 8) & 0xfu;
                wq[j / 8] |= nib << (4 * (j % 8));
            }
            d_f16[r * (cols / QK) + b] = f32_to_f16(d);
        }
}

/* Decode one weight value of a Q8_0 / Q4_0 row-major matrix (input contract). */
static inline int wq_at(int quant_type, const void* qs, int64_t row, int64_t cols, int64_t k) {
    if (quant_type == 0) return ((const int8_t*)qs)[row * cols + k];
    uint32_t word = ((const uint32_t*)qs)[row * (cols / 8) + k / 8];
    return (int)((word >> (4 * (k % 8))) & 0xfu) - 8;
}

/* Decode a whole quantized matrix to int8 values (bit-exact decode check). */
void orc_decode_q(int quant_type, const void* qs, int64_t rows, int64_t cols, int8_t* out) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t k = 0; k < cols; ++k) out[r * cols + k] = (int8_t)wq_at(quant_type, qs, r, cols, k);
}

/*
 * One quantized GEMV row: C = sum over blocks b in order of
 * (f32(isum_b) * d_w[b]) * d_a[b] with isum_b the exact int32 dot of 32
 * values.  Restates the fold of Int8-gemm/gemm_kernels.cpp:156-179 (Q8_0)
 * and :335-358 (Q4_0, with b = nibble - 8).
 */
static float qdot_row(int quant_type, int scale_is_bf16, const void* qs, const uint16_t* d,
                      int64_t row, int64_t cols, const int8_t* a_qs, const float* a_d) {
    float c = 0.0f;
    const int64_t nb = cols / QK;
    for (int64_t b = 0; b < nb; ++b) {
        int32_t isum = 0;
        for (int j = 0; j < QK; ++j)
            isum += wq_at(quant_type, qs, row, cols, b * QK + j) * (int32_t)a_qs[b * QK + j];
        const float dw = scale_to_f32(d[row * nb + b], scale_is_bf16);
        c = c + ((float)isum * dw) * a_d[b];
    }
    return c;
}

/*
 * Full fused-MoE forward for Q8_0 (quant_type 0) / Q4_0 (quant_type 1),
 * tp = 1.  Restates the batched path of Int8-gemm/q8_gemm.cpp:276-646:
 *   routing (moe_common.cpp:146-184); stage A Q8_0 quantisation of x rows;
 *   per routed position: GEMM1 over the 2I gate|up rows, silu_and_mul
 *   (vec_simd.h:36-64, with its exp polynomial), Q8_0 requant of h (gemm_kernels.cpp:394-425),
 *   GEMM2 over the H down rows; combine y[t] = sum_k w[t,k] * out[pos(t,k)] in
 *   k order skipping pos = -1 (q8_gemm.cpp:593-613).
 * x is given in fp32 (exactly representable bf16/fp16 values); y is fp32
 * before the final cast (q8_gemm.cpp:636-639), which the caller applies.
 * Weight inputs follow the row-major contract:
 *   gate_up_qs [E, 2I, H] (int8, or uint32 [E,2I,H/8]), gate_up_d [E,2I,H/32],
 *   down_qs [E, H, I] (or [E,H,I/8]), down_d [E, H, I/32]; scales fp16/bf16 bits.
 * Optional h_out [T*K, I] receives the fp32 SiLU*up intermediate per position.
 */
void orc_moe_forward_q(int quant_type, int scale_is_bf16,
                       int E, int H, int I, int T, int K,
                       const float* x, const int32_t* ids, const float* topk_w,
                       const void* gate_up_qs, const uint16_t* gate_up_d,
                       const void* down_qs, const uint16_t* down_d,
                       float* y, float* h_out) {
    const int HB = H / QK, IB = I / QK;
    int32_t* counts = (int32_t*)calloc((size_t)E + 1, 4);
    int32_t* starts = (int32_t*)calloc((size_t)E + 1, 4);
    int32_t* tmap = (int32_t*)calloc((size_t)T * K * 2 + 2, 4);
    int32_t* smap = (int32_t*)calloc((size_t)T * K + 1, 4);
    const int P = orc_route_preprocess(E, K, T, ids, counts, starts, tmap, smap);

    int8_t* xq = (int8_t*)malloc((size_t)T * H + 1);
    float* xd = (float*)malloc((size_t)T * HB * 4 + 4);
    orc_quantize_rows_q8_0_f32scale(x, T, H, xq, xd);

    float* out = (float*)calloc((size_t)(P ? P : 1) * H, 4);
    float* inter = (float*)malloc((size_t)2 * I * 4);
    int8_t* hq = (int8_t*)malloc((size_t)I);
    float* hd = (float*)malloc((size_t)IB * 4);

    for (int e = 0; e < E; ++e) {
        for (int p = starts[e]; p < starts[e + 1]; ++p) {
            const int t = tmap[2 * p];
            const int8_t* aq = xq + (size_t)t * H;
            const float* ad = xd + (size_t)t * HB;
            for (int n = 0; n < 2 * I; ++n)
                inter[n] = qdot_row(quant_type, scale_is_bf16, gate_up_qs, gate_up_d,
                                    (int64_t)e * 2 * I + n, (int64_t)H, aq, ad);
            silu_and_mul_row(inter, I);
            if (h_out) memcpy(h_out + (size_t)p * I, inter, (size_t)I * 4);
            orc_quantize_rows_q8_0_f32scale(inter, 1, I, hq, hd);
            for (int n = 0; n < H; ++n)
                out[(size_t)p * H + n] = qdot_row(quant_type, scale_is_bf16, down_qs, down_d,
                                                  (int64_t)e * H + n, (int64_t)I, hq, hd);
        }
    }
    for (int t = 0; t < T; ++t) {
        float* acc = y + (size_t)t * H;
        for (int n = 0; n < H; ++n) acc[n] = 0.0f;
        for (int k = 0; k < K; ++k) {
            const int pos = smap[t * K + k];
            if (pos == -1) continue;
            const float w = topk_w[t * K + k];
            for (int n = 0; n < H; ++n) acc[n] += w * out[(size_t)pos * H + n];
        }
    }
    free(counts); free(starts); free(tmap); free(smap); free(xq); free(xd);
    free(out); free(inter); free(hq); free(hd);
}

/*
 * AWQ W4A16 fused-MoE forward (the reference checkout has no implementation:
 * the Ascend grouped_gemv kernel lives in an absent submodule).
 * Format (AutoAWQ "GEMM" packing, as consumed by AWQ MoE layers):
 *   w13_qweight [E, H, 2I/8] int32: for input row k and output column n,
 *     word n/8, nibble position AWQ_POS[n%8] with AWQ_POS = {0,4,1,5,2,6,3,7};
 *   w13_scales  [E, H/G, 2I] (bf16 bits); w13_qzeros [E, H/G, 2I/8] packed
 *     like qweight; w2_* likewise with K = I, N = H.
 *   W[n][k] = (q - z) * s  (fp32), output columns [0,I) = gate, [I,2I) = up.
 * 16-bit activations in, fp32 arithmetic: gate/up dot in fp32, SiLU*up in
 * fp32, down dot over the fp32 intermediate, k-ordered combine.
 */
static const int AWQ_POS[8] = {0, 4, 1, 5, 2, 6, 3, 7};

static inline int awq_nib(const int32_t* packed, int64_t row, int64_t n_cols, int64_t n) {
    uint32_t w = (uint32_t)packed[row * (n_cols / 8) + n / 8];
    return (int)((w >> (4 * AWQ_POS[n % 8])) & 0xfu);
}

static inline float awq_w(const int32_t* qw, const uint16_t* sc, const int32_t* qz,
                          int64_t N, int G, int64_t n, int64_t k) {
    const int q = awq_nib(qw, k, N, n);
    const int z = awq_nib(qz, k / G, N, n);
    const float s = bf16_to_f32(sc[(k / G) * N + n]);
    return (float)(q - z) * s;
}

void orc_awq_dequant(const int32_t* qw, const uint16_t* sc, const int32_t* qz,
                     int64_t Kd, int64_t N, int G, float* W_nk) {
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < Kd; ++k) W_nk[n * Kd + k] = awq_w(qw, sc, qz, N, G, n, k);
}

void orc_moe_forward_awq(int E, int H, int I, int G, int T, int K,
                         const float* x, const int32_t* ids, const float* topk_w,
                         const int32_t* w13_qw, const uint16_t* w13_sc, const int32_t* w13_qz,
                         const int32_t* w2_qw, const uint16_t* w2_sc, const int32_t* w2_qz,
                         float* y) {
    const int N1 = 2 * I;
    int32_t* counts = (int32_t*)calloc((size_t)E + 1, 4);
    int32_t* starts = (int32_t*)calloc((size_t)E + 1, 4);
    int32_t* tmap = (int32_t*)calloc((size_t)T * K * 2 + 2, 4);
    int32_t* smap = (int32_t*)calloc((size_t)T * K + 1, 4);
    const int P = orc_route_preprocess(E, K, T, ids, counts, starts, tmap, smap);
    float* out = (float*)calloc((size_t)(P ? P : 1) * H, 4);
    float* inter = (float*)malloc((size_t)N1 * 4);
    for (int e = 0; e < E; ++e) {
        const int32_t* qw1 = w13_qw + (size_t)e * H * (N1 / 8);
        const uint16_t* sc1 = w13_sc + (size_t)e * (H / G) * N1;
        const int32_t* qz1 = w13_qz + (size_t)e * (H / G) * (N1 / 8);
        const int32_t* qw2 = w2_qw + (size_t)e * I * (H / 8);
        const uint16_t* sc2 = w2_sc + (size_t)e * (I / G) * H;
        const int32_t* qz2 = w2_qz + (size_t)e * (I / G) * (H / 8);
        for (int p = starts[e]; p < starts[e + 1]; ++p) {
            const float* xt = x + (size_t)tmap[2 * p] * H;
            for (int n = 0; n < N1; ++n) {
                float c = 0.0f;
                for (int k = 0; k < H; ++k) c += awq_w(qw1, sc1, qz1, N1, G, n, k) * xt[k];
                inter[n] = c;
            }
            for (int j = 0; j < I; ++j) {
                const float g = inter[j];
                inter[j] = inter[I + j] * (g / (1.0f + expf(-g)));
            }
            for (int n = 0; n < H; ++n) {
                float c = 0.0f;
                for (int k = 0; k < I; ++k) c += awq_w(qw2, sc2, qz2, H, G, n, k) * inter[k];
                out[(size_t)p * H + n] = c;
            }
        }
    }
    for (int t = 0; t < T; ++t) {
        float* acc = y + (size_t)t * H;
        for (int n = 0; n < H; ++n) acc[n] = 0.0f;
        for (int k = 0; k < K; ++k) {
            const int pos = smap[t * K + k];
            if (pos == -1) continue;
            const float w = topk_w[t * K + k];
            for (int n = 0; n < H; ++n) acc[n] += w * out[(size_t)pos * H + n];
        }
    }
    free(counts); free(starts); free(tmap); free(smap); free(out); free(inter);
}

/*
 * Router: top-K of logits (descending value, ties -> lower index first),
 * then softmax over the K selected values when renormalize != 0, else softmax
 * over all E gathered at the selection.  Restates
 * Int8-gemm/test/fused_moe_cpu.py:20-37.
 */
void orc_topk_softmax(const float* logits, int T, int E, int K, int renormalize,
                      int32_t* ids, float* w) {
    for (int t = 0; t < T; ++t) {
        const float* l = logits + (size_t)t * E;
        int32_t* id = ids + (size_t)t * K;
        for (int k = 0; k < K; ++k) {
            int best = -1;
            for (int e = 0; e < E; ++e) {
                int taken = 0;
                for (int j = 0; j < k; ++j) if (id[j] == e) { taken = 1; break; }
                if (taken) continue;
                if (best < 0 || l[e] > l[best]) best = e;
            }
            id[k] = best;
        }
        float* wt = w + (size_t)t * K;
        if (renormalize) {
            const float m = l[id[0]];
            float s = 0.0f;
            for (int k = 0; k < K; ++k) { wt[k] = expf(l[id[k]] - m); s += wt[k]; }
            for (int k = 0; k < K; ++k) wt[k] = wt[k] / s;
        } else {
            float m = l[0];
            for (int e = 1; e < E; ++e) if (l[e] > m) m = l[e];
            float s = 0.0f;
            for (int e = 0; e < E; ++e) s += expf(l[e] - m);
            for (int k = 0; k < K; ++k) wt[k] = expf(l[id[k]] - m) / s;
        }
    }
}
