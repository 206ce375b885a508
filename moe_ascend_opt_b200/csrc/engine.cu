// C ABI of the fused-MoE expert engine (include/moe_b200.h): engine object,
// load-time packing of weights into the device layout, workspace, forward
// dispatch, routing and quantisation entry points.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/moe_b200.h"
#include "common.cuh"
#include "moe_decode_cl.cuh"
#include "moe_decode_tp.cuh"
#include "moe_decode_sk.cuh"
#include "moe_gemm_tc.cuh"

using namespace moe;

// ------------------------------------------------------------------ errors
static thread_local std::string g_last_error;

static int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

#define CUDA_TRY(expr)                                                                       \
    do {                                                                                     \
        cudaError_t _e = (expr);                                                             \
        if (_e != cudaSuccess)                                                               \
            return fail(MOE_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
    } while (0)

extern "C" const char* moe_last_error(void) { return g_last_error.c_str(); }

static inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// ------------------------------------------------------------------ engine
struct moe_engine {
    moe_config cfg{};
    int num_sms = 0;
    int max_smem = 0;
    bool loaded = false;
    int scale_bf16 = 0;
    // Q8_0 / Q4_0 device layout
    // gate_up unit records [E][I]: gate qs row j | up qs row j | gate scales | up scales
    uint8_t* gu = nullptr;
    // down row records [E][H]: qs row | scales
    uint8_t* dn = nullptr;
    int rs1 = 0, ss1 = 0, rs2 = 0, ss2 = 0;
    // AWQ: per-row scale field = [bf16 scales x ngroups][u8 zeros x ngroups], padded
    int64_t unit_bytes() const { return 2 * (int64_t)(rs1 + ss1); }
    int64_t row_bytes() const { return (int64_t)(rs2 + ss2); }
    // down weights re-laid for the split-K decode kernel (Q8_0 / Q4_0): [E][I/32][H/32] slices
    uint8_t* dk = nullptr;
    bool use_sk = true;  // decode through moe_decode_sk_kernel when the layout allows
    // layouts of the cluster decode kernel: AWQ records gate_up [E][I/16][2][H/64] (agu) and
    // down [E][H/32][I/64] (adn); Q8_0 / Q4_0 down row slices [E][H/32][I/32] (adn)
    uint8_t* agu = nullptr;
    uint8_t* adn = nullptr;
    int tp_max_tokens = -1;  // two-pass decode kernels (tp_gate_up / tp_down) up to this many tokens (-1: by format)
    int tp_slice_max = -1;   // and in slices of tp_max_tokens up to this many (-1: by format)
    int cl_max_tokens = -1;  // cluster decode kernel (moe_decode_cl_kernel) up to this many tokens (-1: by format)
    int cl_size = 4;         // its CTAs per cluster
    bool pdl = true;         // launch it with programmatic stream serialization
    int cl_combine = -1;     // its combine: 0 last arrivers in the kernel, 1 a separate kernel, -1 by T (> 1: kernel)
    int64_t cl_item_bytes = 6144;  // target bytes of one bulk copy of its weight streams
    int32_t* clmeta = nullptr;       // that kernel's input: Q | scatter map [clmeta_cap]
    int64_t clmeta_cap = 0;
    int cl_clusters[3] = {-1, -1, -1};  // co-resident clusters per format (-1: not queried)
    float* clpart = nullptr;  // its per-pair fp32 down rows [clpart_cap][H]
    int64_t clpart_cap = 0;
    int32_t* emap = nullptr;  // optional placement map: global expert id -> local id or -1 (+ replica split)
    int32_t emap_n = 0;
    std::vector<int32_t> emap_host;  // the map as set (flags included)
    int32_t rep_rank = 0, rep_world = 1;  // replicated experts: pairs with (token + id) % world == rank
    void* dense_ids = nullptr;  // dense forward: routing ids [cap] (the expert) | weights [cap] (1.0)
    int64_t dense_cap = 0, dense_expert = -1;
    int32_t sk_cost_a = 3;  // its chunk cost model: streaming share per chunk vs one token of compute
    int32_t sk_min_chunks_per_cta = 2;  // use it from this many (unique expert x I/32) chunks per CTA
    // expert-parallel combine over peer memory (moe_engine_p2p_mailbox / _connect)
    uint8_t* mbox = nullptr;   // this rank's mailbox: data [2][world][tcap][H] fp32 | flags [world][num_sms] u64
    int64_t mbox_data_bytes = 0;
    int p2p_world = 1, p2p_rank = 0, p2p_tcap = 0;
    bool p2p_active = false;  // connected and enabled: decode launches sum over the ranks
    void* peer_base[kMaxPeers] = {};  // opened peer mailboxes (nullptr for this rank)
    float* part = nullptr;  // per-CTA fp32 partial tiles [num_sms][part_cap][H] of the split-K kernel
    int64_t part_cap = 0;
    // workspace
    float* h_ws = nullptr;
    int64_t h_cap = 0;  // positions
    uint32_t* bar = nullptr;
    // error word: mapped pinned host memory, written by kernels (set_err) and read by the
    // host at the entry of every call without synchronising; err is its device address
    int32_t* herr = nullptr;
    int32_t* err = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    bool timed = false;
    int64_t gemm_min_tokens = 8;  // forwards with more tokens take the grouped-GEMM path
    int32_t decode_flags = kFlagEvictFirst;
    int32_t gemm_bm = 0;  // grouped-GEMM tile kind (gemm_tile_rows codes); 0 = by tokens per expert
    int64_t tc_min_per_expert = 48;  // tcgen05 GEMMs from this many expected tokens per expert
    int64_t awq_gemm_min_tokens = 24;  // AWQ: the tcgen05 GEMMs for calls with more tokens
    int32_t dist_min_blocks = -1;  // decode: requantise h before the barrier from this many blocks (-1: 2 x SMs)
    // grouped-GEMM path workspace (one allocation, carved per call)
    uint8_t* gws = nullptr;
    size_t gws_bytes = 0;
    unsigned long long* timeline = nullptr;  // per-CTA phase stamps when enabled
    int timeline_ctas = 0;
};

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// Load-time packing: copy `bytes` of every source row into its record.
// kGateUp: source row e*2I + r*I + j (r = 0 gate, 1 up) -> record (e*I + j) at
//          offset base + r*part; kDown: source row e*H + n -> record (e*H + n) at base.
enum RowMap { kDown = 0, kGateUp = 1 };

MOE_DEV int64_t record_of(int map, int64_t srow, int64_t I, int64_t* r) {
    if (map == kGateUp) {
        const int64_t e = srow / (2 * I), rem = srow % (2 * I);
        *r = rem / I;
        return e * I + rem % I;
    }
    *r = 0;
    return srow;
}

__global__ void pack_rows_kernel(uint8_t* dst, const uint8_t* src, int64_t nrows, int64_t bytes, int64_t rec_bytes,
                                 int64_t base, int64_t part, int map, int64_t I) {
    const int64_t srow = blockIdx.x;
    if (srow >= nrows) return;
    int64_t r;
    const int64_t rec = record_of(map, srow, I, &r);
    uint8_t* d = dst + rec * rec_bytes + base + r * part;
    const uint8_t* s = src + srow * bytes;
    for (int64_t c = threadIdx.x; c < bytes; c += blockDim.x) d[c] = s[c];
}

// Inverse of pack_rows_kernel (export / bit-exact decode check): record fields -> source rows.
__global__ void unpack_rows_kernel(uint8_t* dst, const uint8_t* src, int64_t nrows, int64_t bytes, int64_t rec_bytes,
                                   int64_t base, int64_t part, int map, int64_t I) {
    const int64_t srow = blockIdx.x;
    if (srow >= nrows) return;
    int64_t r;
    const int64_t rec = record_of(map, srow, I, &r);
    const uint8_t* s = src + rec * rec_bytes + base + r * part;
    for (int64_t c = threadIdx.x; c < bytes; c += blockDim.x) dst[srow * bytes + c] = s[c];
}

// Online Q8_0 quantisation of one weight matrix [rows, cols] straight into the
// device layout (quantize_weight_only, Int8-gemm/q8_gemm.cpp:197-260: fp16 scale).
__global__ void quantize_weight_rows_kernel(const void* w, int w_dtype, int64_t rows, int64_t cols,
                                            uint8_t* qs_base, uint8_t* sc_base, int64_t row_stride) {
    // one warp per 32-block; lane = element
    const int lane = threadIdx.x & 31;
    const int64_t nb = cols / 32;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (gw >= rows * nb) return;
    const int64_t r = gw / nb, b = gw % nb;
    const int64_t i = r * cols + b * 32 + lane;
    float v;
    if (w_dtype == MOE_F32) v = reinterpret_cast<const float*>(w)[i];
    else if (w_dtype == MOE_BF16) v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w)[i]);
    else v = __half2float(reinterpret_cast<const __half*>(w)[i]);
    float amax = fabsf(v);
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = q8_scale(amax);
    const float id = q8_inv(d);
    uint8_t* qrow = qs_base + r * row_stride;
    qrow[b * 32 + lane] = (uint8_t)(int8_t)q8_quant(v, id);
    if (lane == 0) {
        uint16_t* srow = reinterpret_cast<uint16_t*>(sc_base + r * row_stride);
        srow[b] = __half_as_ushort(__float2half_rn(d));
    }
}

__global__ void quantize_rows_kernel(const void* x, int dtype, int64_t rows, int64_t cols, int8_t* qs, float* d) {
    const int lane = threadIdx.x & 31;
    const int64_t nb = cols / 32;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (gw >= rows * nb) return;
    const int64_t i = gw * 32 + lane;  // rows are contiguous: block gw covers [gw*32, gw*32+32)
    float v;
    if (dtype == MOE_F32) v = reinterpret_cast<const float*>(x)[i];
    else v = act_to_f32(x, i, dtype == MOE_BF16);
    float amax = fabsf(v);
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float dd = q8_scale(amax);
    qs[i] = (int8_t)q8_quant(v, q8_inv(dd));
    if (lane == 0) d[gw] = dd;
}

// Standalone stable permutation (one warp, global memory), moe_route_permute.
__global__ void route_permute_kernel(const int32_t* ids, int TK, int E, int32_t* counts, int32_t* starts,
                                     int32_t* token_map, int32_t* scatter_map, int32_t* tmp_ids) {
    const int lane = threadIdx.x;
    RouteSmem r;
    r.ids = tmp_ids;
    r.smap = scatter_map;
    r.tok = token_map + TK;  // second half as pair-index scratch; rewritten below
    r.cnt = counts;
    r.start = starts;
    r.ue = r.ups = r.ucnt = nullptr;
    r.nuniq = nullptr;
    // counts + ranks
    for (int e = lane; e < E; e += 32) r.cnt[e] = 0;
    __syncwarp();
    for (int i0 = 0; i0 < TK; i0 += 32) {
        const int i = i0 + lane;
        int e = -1;
        if (i < TK) {
            const int g = ids[i];
            e = (g >= 0 && g < E) ? g : -1;
            r.ids[i] = e;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        int base = 0;
        if (e >= 0) base = r.cnt[e];
        __syncwarp();
        if (i < TK) r.smap[i] = (e >= 0) ? base + rank : -1;
        if (e >= 0 && rank == 0) r.cnt[e] = base + __popc(peers);
        __syncwarp();
        __threadfence_block();
    }
    int carry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
        const int e = e0 + lane;
        const int c = (e < E) ? r.cnt[e] : 0;
        int incl = c;
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        if (e < E) r.start[e] = carry + incl - c;
        carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) r.start[E] = carry;
    __syncwarp();
    __threadfence_block();
    for (int i = lane; i < TK; i += 32) {
        const int e = r.ids[i];
        if (e >= 0) r.smap[i] = r.start[e] + r.smap[i];
    }
    __syncwarp();
    __threadfence_block();
}

__global__ void token_map_kernel(const int32_t* scatter_map, int TK, int K, int32_t* token_map) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= TK) return;
    const int pos = scatter_map[i];
    if (pos >= 0) {
        token_map[2 * pos] = i / K;
        token_map[2 * pos + 1] = i % K;
    }
}

// Router: one warp per token; K rounds of warp argmax (ties -> lower id).
__global__ void route_topk_kernel(const float* logits, int T, int E, int K, int renorm, int32_t* ids,
                                  float* w) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const float* l = logits + (size_t)warp * E;
    extern __shared__ uint32_t taken_all[];
    uint32_t* taken = taken_all + (threadIdx.x >> 5) * ((E + 31) / 32);
    for (int i = lane; i < (E + 31) / 32; i += 32) taken[i] = 0;
    __syncwarp();
    float sel_v[16];
    int sel_i[16];
    for (int k = 0; k < K; ++k) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int e = lane; e < E; e += 32) {
            if ((taken[e >> 5] >> (e & 31)) & 1u) continue;
            const float v = l[e];
            if (bi == 0x7fffffff || v > bv) { bv = v; bi = e; }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != 0x7fffffff && (bi == 0x7fffffff || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
        }
        if (lane == 0) taken[bi >> 5] |= 1u << (bi & 31);
        __syncwarp();
        if (k < 16) { sel_v[k] = bv; sel_i[k] = bi; }
    }
    if (lane == 0) {
        float m, s = 0.f;
        if (renorm) {
            m = sel_v[0];
            for (int k = 0; k < K; ++k) s += expf(sel_v[k] - m);
            for (int k = 0; k < K; ++k) {
                ids[(size_t)warp * K + k] = sel_i[k];
                w[(size_t)warp * K + k] = expf(sel_v[k] - m) / s;
            }
        } else {
            m = sel_v[0];  // the overall maximum
            for (int e = 0; e < E; ++e) s += expf(l[e] - m);
            for (int k = 0; k < K; ++k) {
                ids[(size_t)warp * K + k] = sel_i[k];
                w[(size_t)warp * K + k] = expf(sel_v[k] - m) / s;
            }
        }
    }
}

// Router GEMM fused with top-k (the attention-side pre-step of a MoE layer): one CTA per
// token.  The token row goes to shared memory as fp32; warp w computes the logits of
// experts w, w + 8, ... (each lane a strided slice of H, 16-byte weight loads, a fixed
// shuffle tree), then warp 0 selects the top K (K rounds of warp argmax, ties to the lower
// id) and forms the weights as route_topk_kernel does.  Optional fp32 logits out.
constexpr int kRgWarps = 8;
__global__ void __launch_bounds__(kRgWarps * 32) route_gemm_topk_kernel(const void* x, int x_bf16, const void* wr,
                                                                       int w_kind, int H, int E, int K, int renorm,
                                                                       int32_t* ids, float* tw, float* logits_out) {
    extern __shared__ float rg_smem[];
    float* xs = rg_smem;          // [H]
    float* lg = rg_smem + H;      // [E]
    uint32_t* taken = reinterpret_cast<uint32_t*>(lg + E);  // [E/32]
    const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < H; i += blockDim.x) xs[i] = act_to_f32(x, (int64_t)t * H + i, x_bf16);
    for (int i = tid; i < (E + 31) / 32; i += blockDim.x) taken[i] = 0;
    __syncthreads();
    for (int e = warp; e < E; e += kRgWarps) {
        float acc = 0.f;
        if (w_kind == MOE_F32) {
            const float4* wrow = reinterpret_cast<const float4*>(static_cast<const float*>(wr) + (size_t)e * H);
            for (int i = lane; i < H / 4; i += 32) {
                const float4 v = __ldg(wrow + i);
                acc = fmaf(v.x, xs[4 * i], acc);
                acc = fmaf(v.y, xs[4 * i + 1], acc);
                acc = fmaf(v.z, xs[4 * i + 2], acc);
                acc = fmaf(v.w, xs[4 * i + 3], acc);
            }
        } else {
            const uint4* wrow = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(wr) + (size_t)e * H);
            const int wbf = w_kind == MOE_BF16;
            for (int i = lane; i < H / 8; i += 32) {
                const uint4 v = __ldg(wrow + i);
                const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc = fmaf(scale_to_f32((uint16_t)(w4[j] & 0xffffu), wbf), xs[8 * i + 2 * j], acc);
                    acc = fmaf(scale_to_f32((uint16_t)(w4[j] >> 16), wbf), xs[8 * i + 2 * j + 1], acc);
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
            lg[e] = acc;
            if (logits_out) logits_out[(size_t)t * E + e] = acc;
        }
    }
    __syncthreads();
    if (warp != 0) return;
    float sel_v[16];
    int sel_i[16];
    for (int k = 0; k < K; ++k) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int e = lane; e < E; e += 32) {
            if ((taken[e >> 5] >> (e & 31)) & 1u) continue;
            const float v = lg[e];
            if (bi == 0x7fffffff || v > bv) { bv = v; bi = e; }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != 0x7fffffff && (bi == 0x7fffffff || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
        }
        if (lane == 0) taken[bi >> 5] |= 1u << (bi & 31);
        __syncwarp();
        sel_v[k] = bv;
        sel_i[k] = bi;
    }
    if (lane == 0) {
        const float m = sel_v[0];
        float s = 0.f;
        if (renorm) {
            for (int k = 0; k < K; ++k) s += expf(sel_v[k] - m);
        } else {
            for (int e = 0; e < E; ++e) s += expf(lg[e] - m);
        }
        for (int k = 0; k < K; ++k) {
            ids[(size_t)t * K + k] = sel_i[k];
            tw[(size_t)t * K + k] = expf(sel_v[k] - m) / s;
        }
    }
}

int check_engine(moe_engine* eng) {
    if (!eng) return fail(MOE_ERR_INVALID, "engine is null");
    return MOE_OK;
}

// Copy a host or device source to a fresh device buffer (or alias it).
int stage_to_device(const void* src, size_t bytes, int on_device, cudaStream_t st, const uint8_t** out,
                    uint8_t** owned) {
    *owned = nullptr;
    if (on_device) {
        *out = static_cast<const uint8_t*>(src);
        return MOE_OK;
    }
    uint8_t* d = nullptr;
    CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&d), bytes ? bytes : 16, st));
    CUDA_TRY(cudaMemcpyAsync(d, src, bytes, cudaMemcpyHostToDevice, st));
    *owned = d;
    *out = d;
    return MOE_OK;
}

int64_t sk_slice_bytes(const moe_engine* eng) {
    return 32 * (eng->cfg.quant_type == MOE_Q4_0 ? 16 : 32) + 64;
}

int alloc_q_layout(moe_engine* eng) {
    const int64_t E = eng->cfg.num_experts, H = eng->cfg.hidden_size, I = eng->cfg.intermediate_size;
    const int qt = eng->cfg.quant_type;
    if (qt == MOE_AWQ) {
        const int64_t G = eng->cfg.group_size;
        eng->rs1 = (int)round_up(H / 2, 16);
        eng->ss1 = (int)round_up((H / G) * 3, 16);
        eng->rs2 = (int)round_up(I / 2, 16);
        eng->ss2 = (int)round_up((I / G) * 3, 16);
        eng->scale_bf16 = 1;
    } else {
        const bool q4 = qt == MOE_Q4_0;
        eng->rs1 = (int)round_up(q4 ? H / 2 : H, 16);
        eng->ss1 = (int)round_up((H / 32) * 2, 16);
        eng->rs2 = (int)round_up(q4 ? I / 2 : I, 16);
        eng->ss2 = (int)round_up((I / 32) * 2, 16);
    }
    if (!eng->gu) {
        CUDA_TRY(cudaMalloc(&eng->gu, (size_t)E * I * eng->unit_bytes()));
        CUDA_TRY(cudaMalloc(&eng->dn, (size_t)E * H * eng->row_bytes()));
        CUDA_TRY(cudaMemset(eng->gu, 0, (size_t)E * I * eng->unit_bytes()));
        CUDA_TRY(cudaMemset(eng->dn, 0, (size_t)E * H * eng->row_bytes()));
        if (qt != MOE_AWQ) {
            const size_t dk_bytes = (size_t)E * (I / 32) * (H / 32) * sk_slice_bytes(eng);
            CUDA_TRY(cudaMalloc(&eng->dk, dk_bytes));
            CUDA_TRY(cudaMemset(eng->dk, 0, dk_bytes));
        }
    }
    return MOE_OK;
}

// Row records of down -> split-K chunks: one thread per (expert, chunk jb, slice s, row l).
__global__ void pack_down_chunks_kernel(uint8_t* dk, const uint8_t* dn, int64_t E, int64_t H, int64_t I, int64_t rec,
                                        int rs2, int BB, int64_t e0, int64_t e1) {
    const int64_t nb2 = I / 32, nsl = H / 32;
    const int64_t n = (e1 - e0) * nb2 * nsl * 32;
    const int64_t SB = 32 * BB + 64;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int l = (int)(i & 31);
        const int64_t sl = (i >> 5) % nsl, jb = ((i >> 5) / nsl) % nb2, e = e0 + (i >> 5) / (nsl * nb2);
        const uint8_t* src = dn + (e * H + sl * 32 + l) * rec;
        uint8_t* dst = dk + ((e * nb2 + jb) * nsl + sl) * SB;
        const uint4* q = reinterpret_cast<const uint4*>(src + jb * BB);
        uint4* d = reinterpret_cast<uint4*>(dst + (size_t)l * BB);
        d[0] = q[0];
        if (BB == 32) d[1] = q[1];
        reinterpret_cast<uint16_t*>(dst + 32 * BB)[l] = reinterpret_cast<const uint16_t*>(src + rs2)[jb];
    }
}

int build_down_chunks(moe_engine* eng, int64_t e0, int64_t e1, cudaStream_t st) {
    if (!eng->dk) return MOE_OK;
    const int64_t H = eng->cfg.hidden_size, I = eng->cfg.intermediate_size;
    const int BB = eng->cfg.quant_type == MOE_Q4_0 ? 16 : 32;
    pack_down_chunks_kernel<<<eng->num_sms * 8, 256, 0, st>>>(eng->dk, eng->dn, eng->cfg.num_experts, H, I,
                                                               eng->row_bytes(), eng->rs2, BB, e0, e1);
    CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

// AWQ GEMM packing -> records.  qw [E][Kd][N/8] int32, output column n, input row k:
// word n/8, nibble position kAwqPos[n%8].  gate_up (N = 2I): column n < I is gate row
// n of unit n, column I + j is up row j; down (N = H): column n is row n.
__constant__ int kAwqPos[8] = {0, 4, 1, 5, 2, 6, 3, 7};

MOE_DEV int awq_nib(const int32_t* packed, int64_t row, int64_t N, int64_t n) {
    return (int)(((uint32_t)packed[row * (N / 8) + n / 8] >> (4 * kAwqPos[n % 8])) & 0xFu);
}

MOE_DEV uint8_t* awq_record(uint8_t* base, int gate_up, int64_t e, int64_t n, int64_t I, int64_t H, int64_t rec,
                            int64_t rs, int64_t ss, int64_t* roff, int64_t* soff) {
    if (gate_up) {
        const int64_t r = n >= I ? 1 : 0, j = n - r * I;
        *roff = r * rs;
        *soff = 2 * rs + r * ss;
        return base + (e * I + j) * rec;
    }
    *roff = 0;
    *soff = rs;
    return base + (e * H + n) * rec;
}

__global__ void awq_pack_q_kernel(uint8_t* base, const int32_t* qw, int64_t Kd, int64_t N, int gate_up, int64_t I,
                                  int64_t H, int64_t rec, int64_t rs, int64_t ss) {
    const int64_t e = blockIdx.y;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // over n * (Kd/2)
    if (idx >= N * (Kd / 2)) return;
    const int64_t n = idx / (Kd / 2), kb = idx % (Kd / 2);
    const int32_t* q = qw + e * Kd * (N / 8);
    const int lo = awq_nib(q, 2 * kb, N, n), hi = awq_nib(q, 2 * kb + 1, N, n);
    int64_t roff, soff;
    uint8_t* r = awq_record(base, gate_up, e, n, I, H, rec, rs, ss, &roff, &soff);
    r[roff + kb] = (uint8_t)(lo | (hi << 4));
}

__global__ void awq_pack_sz_kernel(uint8_t* base, const uint16_t* sc, const int32_t* qz, int64_t ng, int64_t N,
                                   int gate_up, int64_t I, int64_t H, int64_t rec, int64_t rs, int64_t ss) {
    const int64_t e = blockIdx.y;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // over n * ng
    if (idx >= N * ng) return;
    const int64_t n = idx / ng, g = idx % ng;
    int64_t roff, soff;
    uint8_t* r = awq_record(base, gate_up, e, n, I, H, rec, rs, ss, &roff, &soff);
    reinterpret_cast<uint16_t*>(r + soff)[g] = sc[(e * ng + g) * N + n];
    r[soff + 2 * ng + g] = (uint8_t)awq_nib(qz + e * ng * (N / 8), g, N, n);
}

// Device counters: the grid barrier and the cluster kernel's combine counters in the first
// 256 bytes, the two-pass kernels' row-block counters [H/32] after them.
size_t bar_bytes(const moe_engine* eng) { return 256 + (size_t)(eng->cfg.hidden_size / 32 + 1) * 4; }

int ensure_workspace(moe_engine* eng, int64_t positions) {
    if (!eng->bar) {
        CUDA_TRY(cudaMalloc(&eng->bar, bar_bytes(eng)));
        CUDA_TRY(cudaMemset(eng->bar, 0, bar_bytes(eng)));
    }
    if (!eng->herr) {
        CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&eng->herr), 64, cudaHostAllocMapped));
        *reinterpret_cast<volatile int32_t*>(eng->herr) = 0;
        CUDA_TRY(cudaHostGetDevicePointer(reinterpret_cast<void**>(&eng->err), eng->herr, 0));
    }
    if (positions <= eng->h_cap) return MOE_OK;
    int64_t cap = eng->h_cap ? eng->h_cap : 64;
    while (cap < positions) cap *= 2;
    CUDA_TRY(cudaDeviceSynchronize());  // the old buffers may still be in use by queued work
    if (eng->h_ws) CUDA_TRY(cudaFree(eng->h_ws));
    eng->h_ws = nullptr;
    CUDA_TRY(cudaMalloc(&eng->h_ws, (size_t)cap * eng->cfg.intermediate_size * sizeof(float)));
    eng->h_cap = cap;
    return MOE_OK;
}

// Shared-memory plan of the decode kernel for T tokens; false if it does not fit.
struct DecodePlan {
    DecodeParams p;
    size_t smem;
    int grid;
    bool sk = false;  // split-K kernel (moe_decode_sk_kernel) with layout L
    SkLayout L{};
};

int ensure_part(moe_engine* eng, int64_t tokens) {
    if (tokens <= eng->part_cap) return MOE_OK;
    int64_t cap = eng->part_cap ? eng->part_cap : 8;
    while (cap < tokens) cap *= 2;
    CUDA_TRY(cudaDeviceSynchronize());  // the old buffer may still be in use by queued work
    if (eng->part) CUDA_TRY(cudaFree(eng->part));
    eng->part = nullptr;
    CUDA_TRY(cudaMalloc(&eng->part, (size_t)eng->num_sms * cap * eng->cfg.hidden_size * sizeof(float)));
    eng->part_cap = cap;
    return MOE_OK;
}

// Shared-memory plan of the split-K decode kernel for T tokens; false if it does not fit
// (or the engine cannot use it).
bool plan_decode_sk(const moe_engine* eng, int T, int K, DecodePlan& pl) {
    if (!eng->use_sk || !eng->dk || eng->cfg.quant_type == MOE_AWQ) return false;
    const int E = (int)eng->cfg.num_experts, H = (int)eng->cfg.hidden_size, I = (int)eng->cfg.intermediate_size;
    const int TK = T * K, nb1 = H / 32, nb2 = I / 32, nsl = H / 32;
    const int G = eng->num_sms;
    // with fewer than ~2 chunks per CTA the chunk granularity leaves CTAs with twice the
    // work of others (one token: 8 experts x I/32 chunks); the barrier kernel splits
    // gate_up evenly by rows there
    if ((int64_t)std::min(E, TK) * nb2 < (int64_t)eng->sk_min_chunks_per_cta * G) return false;
    DecodeParams& p = pl.p;
    std::memset(&p, 0, sizeof(p));
    SkLayout& L = pl.L;
    int64_t off = (int64_t)(3 * TK + 5 * E + 4) * 4;
    L.off_tw = (int)off;
    off = round_up(off + (int64_t)TK * 12 + (int64_t)(E + 1) * 4, 128);
    L.off_a = (int)off;
    const int64_t xbytes = (int64_t)T * H + (int64_t)T * nb1 * 8, tile = (int64_t)T * H * 4;
    off += round_up(std::max({xbytes, tile, (int64_t)kThreads * 4}), 128);  // + the reduction's group sums
    L.off_h = (int)off;
    // h slots per CTA: the cost share of one CTA bounds its (chunk, token) pairs
    const int64_t nbmax = (int64_t)std::min(E, TK) * nb2, A = eng->sk_cost_a;
    L.hslots = (int)((nbmax * A + (int64_t)TK * nb2 + G - 1) / G + A + 2 * T + 1);  // + float rounding of the split
    off += round_up((int64_t)L.hslots * 128, 128);
    L.spw = (nsl + kWarps - 1) / kWarps;
    const int64_t SB = sk_slice_bytes(eng);
    const int64_t unit_bytes = eng->unit_bytes(), down_item = L.spw * SB;
    const int64_t avail = (int64_t)eng->max_smem - off - 1024;
    const int64_t per_warp = avail / kWarps;
    int upi = 4;
    while (upi > 1 && 2 * round_up(std::max((int64_t)upi * unit_bytes, down_item), 128) > per_warp) upi >>= 1;
    const int64_t slot = round_up(std::max((int64_t)upi * unit_bytes, down_item), 128);
    const int slots = (int)std::min<int64_t>(6, per_warp / slot);
    if (slots < 2) return false;
    p.units_per_item = upi;
    p.slots = slots;
    p.slot_bytes = (int)slot;
    off = round_up(off + 8 * kWarps * slots, 128);
    p.off_ring = (int)off;
    off += (int64_t)kWarps * slots * slot;
    if (off > eng->max_smem - 1024 - 256) return false;  // static shared memory (1 KB reserved + own)
    p.rs1 = eng->rs1; p.ss1 = eng->ss1; p.rs2 = eng->rs2; p.ss2 = eng->ss2;
    p.E = E; p.e_off = eng->cfg.expert_offset; p.H = H; p.I = I; p.T = T; p.K = K;
    p.emap = eng->emap; p.emap_n = eng->emap_n;
    p.scale_bf16 = eng->scale_bf16;
    p.group = eng->cfg.group_size;
    p.flags = eng->decode_flags;
    p.sk_cost_a = eng->sk_cost_a;
    pl.smem = (size_t)off;
    pl.grid = G;
    pl.sk = true;
    return true;
}

bool plan_decode_lpr(const moe_engine* eng, int T, int K, int lpr0, DecodePlan& pl) {
    const int E = (int)eng->cfg.num_experts, H = (int)eng->cfg.hidden_size, I = (int)eng->cfg.intermediate_size;
    const int TK = T * K, nb1 = H / 32, nb2 = I / 32;
    const int G = eng->num_sms;
    DecodeParams& p = pl.p;
    std::memset(&p, 0, sizeof(p));
    int lpr = lpr0;  // phase 2: lanes per down row (32 / lpr rows per item)
    while (lpr > 1 && nb2 % lpr != 0) lpr >>= 1;
    p.lanes_per_row = lpr;
    const int rpg = 32 / lpr;
    int64_t off = round_up((int64_t)(3 * TK + 5 * E + 4) * 4, 128);
    p.off_x = (int)off;
    const bool awq = eng->cfg.quant_type == MOE_AWQ;
    const int64_t xbytes = awq ? (int64_t)T * H * 2 + (int64_t)T * nb1 * 4
                               : round_up((int64_t)T * H, 16) + (int64_t)T * nb1 * 8;
    const int64_t hbytes = awq ? (int64_t)TK * I * 4 + (int64_t)TK * nb2 * 4
                               : round_up((int64_t)TK * I, 16) + (int64_t)TK * nb2 * 8;
    off += round_up(std::max(xbytes, hbytes), 128);
    p.off_out = (int)off;
    p.rows_max = (H + G - 1) / G;
    off += round_up((int64_t)TK * p.rows_max * 4, 128);
    const int64_t unit_bytes = eng->unit_bytes();
    const int64_t item_bytes = (int64_t)rpg * eng->row_bytes();
    const int64_t avail = (int64_t)eng->max_smem - off - 1024;  // mbarriers + static smem
    const int64_t per_warp = avail / kWarps;
    // phase-1 items of up to 4 units, at least 2 slots per warp
    int upi = 4;
    while (upi > 1 && 2 * round_up(std::max((int64_t)upi * unit_bytes, item_bytes), 128) > per_warp) upi >>= 1;
    const int64_t slot = round_up(std::max((int64_t)upi * unit_bytes, item_bytes), 128);
    int slots = (int)std::min<int64_t>(6, per_warp / slot);
    if (slots < 2) return false;
    p.units_per_item = upi;
    p.slots = slots;
    p.slot_bytes = (int)slot;
    off = round_up(off + 8 * kWarps * slots, 128);
    p.off_ring = (int)off;  // mbarriers sit in the 8*kWarps*slots bytes right before the ring
    off += (int64_t)kWarps * slots * slot;
    if (off > eng->max_smem - 1024 - 256) return false;  // static shared memory (1 KB reserved + own)
    p.rs1 = eng->rs1; p.ss1 = eng->ss1; p.rs2 = eng->rs2; p.ss2 = eng->ss2;
    p.E = E; p.e_off = eng->cfg.expert_offset; p.H = H; p.I = I; p.T = T; p.K = K;
    p.emap = eng->emap; p.emap_n = eng->emap_n;
    p.scale_bf16 = eng->scale_bf16;
    p.group = eng->cfg.group_size;
    p.flags = eng->decode_flags;
    p.dist_min_blocks = eng->dist_min_blocks >= 0 ? eng->dist_min_blocks : 2 * G;
    pl.smem = (size_t)off;
    pl.grid = G;
    return true;
}

// Prefer 4 lanes per down row (8-row items); wider rows (large I) take more lanes per row so
// that two ring slots per warp still fit in shared memory.
bool plan_decode(const moe_engine* eng, int T, int K, DecodePlan& pl) {
    for (int lpr : {4, 8, 16, 32})
        if (plan_decode_lpr(eng, T, K, lpr, pl)) return true;
    return false;
}

template <int FMT>
int launch_decode_sk(const DecodePlan& pl, cudaStream_t st) {
    auto kern = moe_decode_sk_kernel<FMT>;
    static thread_local int smem_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && smem_set[dev] < (int)pl.smem) {
        CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem));
        smem_set[dev] = (int)pl.smem;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // the grid barrier needs every CTA resident
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, pl.p, pl.L));
    return MOE_OK;
}

template <int FMT>
int launch_decode(const DecodePlan& pl, cudaStream_t st) {
    if (pl.sk) return FMT == kQ4 ? launch_decode_sk<kQ4>(pl, st) : launch_decode_sk<kQ8>(pl, st);
    auto kern = moe_decode_kernel<FMT>;
    static thread_local int smem_set[64] = {};  // per device: largest opt-in already applied
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && smem_set[dev] < (int)pl.smem) {
        CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem));
        smem_set[dev] = (int)pl.smem;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, pl.p));
    return MOE_OK;
}

}  // namespace

// ------------------------------------------------------------------ cluster decode path
// AWQ records of the cluster decode kernel, built from the row records: one thread per
// (record, row r, lane column c) writes the 8 bytes lane c of an mma.sync m16n8k16 A
// fragment reads for row r (16 nibbles: word w, nibble position i holds k = 16 (2w + (i%4)/2)
// + 2c + 8 ((i%4)&1) + i/4 of the record's 64 k), and c == 0 the row's scale and zero point.
// gate_up records [E][I/16][2][H/64] of 16 rows (560 B), down records [E][H/32][I/64] of 32
// rows (1120 B).
__global__ void awq_rec_pack_kernel(uint8_t* dst, const uint8_t* src, int64_t nrec, int gate_up, int64_t I, int64_t H,
                                    int64_t G, int64_t rec_bytes, int64_t rs, int64_t ss) {
    const int rows = gate_up ? 16 : 32;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= nrec * rows * 4) return;
    const int64_t R = idx / (rows * 4);
    const int r = (int)((idx >> 2) % rows), c = (int)(idx & 3);
    const int64_t nk = (gate_up ? H : I) / kAwqK, ng = (gate_up ? H : I) / G;
    const int64_t kh = R % nk;
    int64_t t = R / nk;
    const uint8_t* row;
    const uint8_t* sc;
    if (gate_up) {
        const int64_t half = t & 1;
        t >>= 1;
        const int64_t ut = t % (I / 16), e = t / (I / 16);
        const uint8_t* rec = src + (e * I + 16 * ut + r) * rec_bytes;
        row = rec + half * rs;
        sc = rec + 2 * rs + half * ss;
    } else {
        const int64_t rb = t % (H / 32), e = t / (H / 32);
        row = src + (e * H + 32 * rb + r) * rec_bytes;
        sc = row + rs;
    }
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int jw = 0; jw < 2; ++jw)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int pp = i & 3, e2 = i >> 2;
            const int64_t k = kh * kAwqK + 16 * (2 * jw + (pp >> 1)) + 2 * c + 8 * (pp & 1) + e2;
            const uint32_t nib = (row[k >> 1] >> (4 * (k & 1))) & 0xFu;
            w[jw] |= nib << (4 * i);
        }
    const int recb = gate_up ? kAwqGuRec : kAwqDnRec;
    uint8_t* d = dst + R * recb;
    *reinterpret_cast<uint2*>(d + r * 32 + c * 8) = make_uint2(w[0], w[1]);
    if (c == 0) {
        const int64_t grp = kh * kAwqK / G;
        reinterpret_cast<uint16_t*>(d + rows * 32)[r] = reinterpret_cast<const uint16_t*>(sc)[grp];
        d[rows * 34 + r] = sc[2 * ng + grp];
    }
}

// Q8_0 / Q4_0 down row-slice records of the cluster decode kernel: [E][H/32][I/32] slices of
// 32 rows x one 32-column block (32 x BB weight bytes, then 32 scales), from the row records.
__global__ void pack_down_rowslices_kernel(uint8_t* dr, const uint8_t* dn, int64_t e0, int64_t e1, int64_t H,
                                           int64_t I, int64_t rec, int rs2, int BB) {
    const int64_t nb2 = I / 32, nsl = H / 32;
    const int64_t n = (e1 - e0) * nsl * nb2 * 32;
    const int64_t SB = 32 * BB + 64;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int l = (int)(i & 31);
        const int64_t kc = (i >> 5) % nb2, sl = ((i >> 5) / nb2) % nsl, e = e0 + (i >> 5) / (nb2 * nsl);
        const uint8_t* src = dn + (e * H + sl * 32 + l) * rec;
        uint8_t* dst = dr + ((e * nsl + sl) * nb2 + kc) * SB;
        const uint4* q = reinterpret_cast<const uint4*>(src + kc * BB);
        uint4* d = reinterpret_cast<uint4*>(dst + (size_t)l * BB);
        d[0] = q[0];
        if (BB == 32) d[1] = q[1];
        reinterpret_cast<uint16_t*>(dst + 32 * BB)[l] = reinterpret_cast<const uint16_t*>(src + rs2)[kc];
    }
}

bool awq_recs_ok(const moe_engine* eng) {
    const int64_t H = eng->cfg.hidden_size, I = eng->cfg.intermediate_size, G = eng->cfg.group_size;
    return eng->cfg.quant_type == MOE_AWQ && G % kAwqK == 0 && H % G == 0 && I % G == 0 && I % 16 == 0 &&
           H % 32 == 0;
}

// The cluster kernel's weight layouts: AWQ records (from the row records) or the Q8_0 / Q4_0
// down row slices.  Experts [e0, e1) of the row layouts changed.
int build_cl_layout(moe_engine* eng, int64_t e0, int64_t e1, cudaStream_t st) {
    const int64_t E = eng->cfg.num_experts, H = eng->cfg.hidden_size, I = eng->cfg.intermediate_size;
    if (eng->cfg.quant_type == MOE_AWQ) {
        if (!awq_recs_ok(eng)) return MOE_OK;
        const int64_t n1 = E * (I / 16) * 2 * (H / kAwqK), n2 = E * (H / 32) * (I / kAwqK);
        if (!eng->agu) {
            CUDA_TRY(cudaMalloc(&eng->agu, (size_t)n1 * kAwqGuRec));
            CUDA_TRY(cudaMalloc(&eng->adn, (size_t)n2 * kAwqDnRec));
        }
        awq_rec_pack_kernel<<<(unsigned)((n1 * 64 + 255) / 256), 256, 0, st>>>(
            eng->agu, eng->gu, n1, 1, I, H, eng->cfg.group_size, eng->unit_bytes(), eng->rs1, eng->ss1);
        awq_rec_pack_kernel<<<(unsigned)((n2 * 128 + 255) / 256), 256, 0, st>>>(
            eng->adn, eng->dn, n2, 0, I, H, eng->cfg.group_size, eng->row_bytes(), eng->rs2, 0);
        CUDA_TRY(cudaGetLastError());
        return MOE_OK;
    }
    if (H % 32 != 0) return MOE_OK;
    const int BB = eng->cfg.quant_type == MOE_Q4_0 ? 16 : 32;
    const size_t bytes = (size_t)E * (H / 32) * (I / 32) * (32 * BB + 64);
    if (!eng->adn) CUDA_TRY(cudaMalloc(&eng->adn, bytes));
    pack_down_rowslices_kernel<<<eng->num_sms * 8, 256, 0, st>>>(eng->adn, eng->dn, e0, e1, H, I, eng->row_bytes(),
                                                                  eng->rs2, BB);
    CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

struct ClPlan {
    ClParams p;
    size_t smem;
};

// Shared-memory plan of the cluster decode kernel for T tokens; false when it does not apply.
bool plan_decode_cl(const moe_engine* eng, int T, int K, ClPlan& pl) {
    const int qt = eng->cfg.quant_type;
    const int E = (int)eng->cfg.num_experts, H = (int)eng->cfg.hidden_size, I = (int)eng->cfg.intermediate_size;
    const int cs = eng->cl_size;
    if (T < 1 || T > 8 || T > eng->cl_max_tokens || !eng->adn) return false;
    const bool awq = qt == MOE_AWQ;
    if (awq && (!eng->agu || !awq_recs_ok(eng))) return false;
    if (H % (32 * cs) != 0 || H % kClRowBlocks != 0 || 32 % cs != 0) return false;
    // allowed K-splits Q: Q8/Q4 K-ranges of whole 32-blocks and 4-unit CTA slices; AWQ K-ranges
    // of whole 64-k records and 16-unit CTA slices
    int qmask = 0, qmin = 0, qmax = 0;
    for (int lq = 0; (1 << lq) <= kClMaxQ; ++lq) {
        const int q = 1 << lq;
        if (I % q) break;
        const int KR = I / q;
        if (KR % cs) break;
        const int UPC = KR / cs;
        const bool okq = awq ? (KR % kAwqK == 0 && UPC % 16 == 0) : (KR % 32 == 0 && UPC % 4 == 0);
        if (!okq) continue;
        qmask |= 1 << lq;
        if (!qmin) qmin = q;
        qmax = q;
    }
    if (!qmask) return false;
    const int TK = T * K, nb1 = H / 32, cap = T;
    const int KRmax = I / qmin, UPCmax = KRmax / cs, RPC = H / cs;
    ClParams& p = pl.p;
    std::memset(&p, 0, sizeof(p));
    p.qmask = qmask;
    int64_t off = round_up((int64_t)(3 * TK + 5 * E + 4) * 4, 16);
    p.off_wl = (int)off;
    off = round_up(off + (int64_t)TK * qmax * 4, 128);
    p.off_x = (int)off;
    off += round_up(awq ? (int64_t)T * (H + 8) * 2 + (int64_t)T * (H / kAwqK) * 4
                        : (int64_t)T * H + (int64_t)T * nb1 * 8, 128);
    p.off_h = (int)off;
    const int64_t hb = awq ? (int64_t)cap * (KRmax + 8) * 2 : (int64_t)cap * KRmax * 4;
    p.hbuf_bytes = (int)hb;
    off += round_up(hb, 128);
    p.off_hq = (int)off;
    if (awq) {
        int64_t slots_bytes = 0;
        for (int lq = 0; (1 << lq) <= kClMaxQ; ++lq) {
            if (!((qmask >> lq) & 1)) continue;
            const int rtn = 2 * (I >> lq) / cs / 16;  // gate_up row tiles of a CTA
            const int nslot = (kClWarps + rtn - 1) / rtn + 1;
            slots_bytes = std::max(slots_bytes, (int64_t)rtn * nslot * 16 * cap * 4);
        }
        off += round_up(std::max(slots_bytes, (int64_t)cap * (KRmax / kAwqK) * 4), 128);
    } else {
        off += round_up((int64_t)cap * KRmax + (int64_t)cap * (KRmax / 32) * 8, 128);
    }
    p.off_p = (int)off;
    off += round_up((int64_t)cap * UPCmax * (awq ? 2 : 4), 128);
    p.off_out = (int)off;
    off += round_up((int64_t)cap * RPC * 4, 128);
    // ring items of up to ~6 KB
    int64_t maxitem;
    if (awq) {
        p.upi = (int)std::max<int64_t>(1, eng->cl_item_bytes / kAwqGuRec);  // gate_up records per item
        p.kpi = (int)std::max<int64_t>(1, eng->cl_item_bytes / kAwqDnRec);  // down records per item
        maxitem = std::max((int64_t)p.upi * kAwqGuRec, (int64_t)p.kpi * kAwqDnRec);
    } else {
        const int BB = qt == MOE_Q4_0 ? 16 : 32;
        const int64_t ub = eng->unit_bytes(), SBq = 32 * BB + 64;
        p.upi = (int)std::max<int64_t>(1, eng->cl_item_bytes / ub);
        p.kpi = (int)std::max<int64_t>(1, eng->cl_item_bytes / SBq);
        maxitem = std::max((int64_t)p.upi * ub, (int64_t)p.kpi * SBq);
    }
    off = round_up(off + 12 * kClWarps * kClInFlight, 128);  // mbarriers and item offsets
    p.off_ring = (int)off;
    int64_t ring = ((int64_t)eng->max_smem - 1024 - off) / kClWarps / 128 * 128;
    if (const char* v = std::getenv("MOE_CL_RING_KB")) ring = std::min<int64_t>(ring, (int64_t)std::atoi(v) * 1024);
    if (ring < maxitem) return false;
    p.ring_bytes = (int)ring;
    off += ring * kClWarps;
    if (off > eng->max_smem - 1024) return false;
    p.rs1 = eng->rs1; p.ss1 = eng->ss1;
    p.E = E; p.e_off = eng->cfg.expert_offset; p.H = H; p.I = I; p.T = T; p.K = K;
    p.emap = eng->emap; p.emap_n = eng->emap_n;
    p.scale_bf16 = eng->scale_bf16;
    p.flags = eng->decode_flags;
    pl.smem = (size_t)off;
    return true;
}

template <int FMT, bool XBF>
int setup_decode_cl(moe_engine* eng) {
    auto kern = moe_decode_cl_kernel<FMT, XBF, 0>;
    static thread_local bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    // every plan fits in max_smem - 1024 bytes (the static shared memory)
    const int dyn = eng->max_smem - 1024;
    if (dev >= 64 || !attr_set[dev]) {
        CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn));
        CUDA_TRY(cudaFuncSetAttribute(moe_decode_cl_kernel<FMT, XBF, 1>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, dyn));
        if (dev < 64) attr_set[dev] = true;
    }
    int& nc = eng->cl_clusters[FMT];
    if (nc >= 0) return MOE_OK;
    // the kernel holds all registers of an SM, so the count of co-resident clusters does not
    // depend on the plan
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = eng->cl_size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(eng->cl_size * 16);
    cfg.blockDim = dim3(kClThreads);
    cfg.dynamicSmemBytes = (size_t)dyn;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    nc = std::min(n, eng->num_sms / eng->cl_size);
    return MOE_OK;
}

template <int FMT, bool XBF>
int launch_decode_cl(moe_engine* eng, ClPlan& pl, cudaStream_t st) {
    if (int rc = setup_decode_cl<FMT, XBF>(eng)) return rc;
    if (eng->cl_clusters[FMT] < 1) return fail(MOE_ERR_STATE, "no thread-block cluster fits");
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = eng->cl_size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // programmatic dependent launch: the kernel waits (griddepcontrol.wait) for its stream
    // predecessor before reading, so it may be scheduled while that one finishes
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(eng->cl_size * eng->cl_clusters[FMT]);
    cfg.blockDim = dim3(kClThreads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = eng->pdl ? 2 : 1;
    if (pl.p.T == 1) CUDA_TRY(cudaLaunchKernelEx(&cfg, moe_decode_cl_kernel<FMT, XBF, 1>, pl.p));
    else CUDA_TRY(cudaLaunchKernelEx(&cfg, moe_decode_cl_kernel<FMT, XBF, 0>, pl.p));
    if (pl.p.meta) {
        const int n = pl.p.T * pl.p.H;
        cudaLaunchConfig_t c2{};
        c2.gridDim = dim3((n + 255) / 256);
        c2.blockDim = dim3(256);
        c2.stream = st;
        c2.attrs = attr + 1;
        c2.numAttrs = eng->pdl ? 1 : 0;
        CUDA_TRY(cudaLaunchKernelEx(&c2, cl_combine_kernel, (const float*)pl.p.part, (const int32_t*)pl.p.meta,
                                    pl.p.tw, pl.p.T, pl.p.K, pl.p.H, pl.p.y, pl.p.out_kind));
    }
    return MOE_OK;
}

int ensure_clpart(moe_engine* eng, int64_t positions) {
    if (positions <= eng->clpart_cap) return MOE_OK;
    int64_t cap = eng->clpart_cap ? eng->clpart_cap : 64;
    while (cap < positions) cap *= 2;
    CUDA_TRY(cudaDeviceSynchronize());  // the old buffer may still be in use by queued work
    if (eng->clpart) CUDA_TRY(cudaFree(eng->clpart));
    eng->clpart = nullptr;
    CUDA_TRY(cudaMalloc(&eng->clpart, (size_t)cap * eng->cfg.hidden_size * sizeof(float)));
    eng->clpart_cap = cap;
    return MOE_OK;
}

// ------------------------------------------------------------------ grouped-GEMM path
// Large token counts: parallel routing, Q8_0 token rows, two grouped GEMMs on the
// int8 tensor cores, combine.  Only Q8_0 / Q4_0 with H and I multiples of 128.
bool gemm_path_ok(const moe_engine* eng) {
    const int64_t H = eng->cfg.hidden_size, I = eng->cfg.intermediate_size;
    return eng->cfg.quant_type != MOE_AWQ && (2 * I) % gemm::kBN == 0 && H % gemm::kBN == 0 && I % 128 == 0 &&
           H % 128 == 0 && eng->cfg.num_experts <= 1024;
}

struct GemmWs {
    int32_t *blk, *counts, *starts, *mtile, *smap, *tokmap;
    int8_t *xq, *hq;
    float *xd, *hd, *out;
    int32_t *xs, *hs;
    __half *xa, *ha;
};

int gemm_workspace(moe_engine* eng, int64_t T, int64_t K, GemmWs& w) {
    const int64_t E = eng->cfg.num_experts, H = eng->cfg.hidden_size, I = eng->cfg.intermediate_size;
    const int64_t TK = T * K, nblk = (TK + gemm::kChunk - 1) / gemm::kChunk;
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off += (bytes + 255) / 256 * 256; return o; };
    const size_t o_blk = take(nblk * E * 4), o_cnt = take(E * 4), o_st = take((E + 1) * 4), o_mt = take((E + 1) * 4);
    const size_t o_smap = take(TK * 4), o_tok = take(TK * 4);
    const size_t o_xq = take(T * H), o_xd = take(T * (H / 32) * 4), o_xs = take(T * (H / 32) * 4);
    const size_t o_hq = take(TK * I), o_hd = take(TK * (I / 32) * 4), o_hs = take(TK * (I / 32) * 4);
    const size_t o_out = take(TK * H * 4);
    const size_t o_xa = take(T * H * 2), o_ha = take(TK * I * 2);  // fp16 operands of the tcgen05 path
    if (off > eng->gws_bytes) {
        CUDA_TRY(cudaDeviceSynchronize());
        if (eng->gws) CUDA_TRY(cudaFree(eng->gws));
        eng->gws = nullptr;
        size_t cap = std::max(off, eng->gws_bytes * 2);
        CUDA_TRY(cudaMalloc(&eng->gws, cap));
        eng->gws_bytes = cap;
    }
    uint8_t* b = eng->gws;
    w.blk = reinterpret_cast<int32_t*>(b + o_blk);
    w.counts = reinterpret_cast<int32_t*>(b + o_cnt);
    w.starts = reinterpret_cast<int32_t*>(b + o_st);
    w.mtile = reinterpret_cast<int32_t*>(b + o_mt);
    w.smap = reinterpret_cast<int32_t*>(b + o_smap);
    w.tokmap = reinterpret_cast<int32_t*>(b + o_tok);
    w.xq = reinterpret_cast<int8_t*>(b + o_xq);
    w.xd = reinterpret_cast<float*>(b + o_xd);
    w.xs = reinterpret_cast<int32_t*>(b + o_xs);
    w.hq = reinterpret_cast<int8_t*>(b + o_hq);
    w.hd = reinterpret_cast<float*>(b + o_hd);
    w.hs = reinterpret_cast<int32_t*>(b + o_hs);
    w.out = reinterpret_cast<float*>(b + o_out);
    w.xa = reinterpret_cast<__half*>(b + o_xa);
    w.ha = reinterpret_cast<__half*>(b + o_ha);
    return MOE_OK;
}

// GEMM tile kind from the expected tokens per active expert (uniform routing): up to 24,
// the weights-on-M kernel with 8- or 16-token tiles; above, 32- or 64-token M tiles.
// Codes: -8 / -16 weights-on-M, 16 / 32 / 64 tokens-on-M, 128 the tcgen05 bf16 kernels.
int gemm_tile_rows(const moe_engine* eng, int64_t TK) {
    if (eng->gemm_bm) return eng->gemm_bm;
    const int64_t per_expert = TK / std::max<int64_t>(1, std::min<int64_t>(eng->cfg.num_experts, TK));
    if (per_expert >= eng->tc_min_per_expert) return 128;
    return per_expert <= 6 ? -8 : (per_expert <= 24 ? -16 : (per_expert <= 40 ? 32 : 64));
}

// The tcgen05 grouped GEMMs of one layer.  WF: 0 Q8_0, 1 Q4_0 (A = fp16(q_a d_a) rows from
// quant_rows_f16_kernel), 2 AWQ (A = the 16-bit hidden rows themselves, W4A16).
template <int WF>
int launch_gemms_tc(moe_engine* eng, const GemmWs& w, const void* x, int act_bf16, int64_t T, int64_t K,
                    cudaStream_t st) {
    const int E = (int)eng->cfg.num_experts, H = (int)eng->cfg.hidden_size, I = (int)eng->cfg.intermediate_size;
    const int64_t TK = T * K;
    const __half* a1 = static_cast<const __half*>(x);  // AWQ: the caller's rows (bf16 or fp16 bits)
    if (WF != 2) {
        const int nb = (int)(T * (H / 32));
        gemm::quant_rows_f16_kernel<<<std::min((nb + 255) / 256, eng->num_sms * 8), 256, 0, st>>>(
            static_cast<const uint8_t*>(x), act_bf16, (int)T, H, w.xa, eng->err);
        CUDA_TRY(cudaGetLastError());
        a1 = w.xa;
    }
    const int smem = gemm::kStagesTc * gemm::StageTc<WF != 0>::kBytes + 1024;
    static thread_local int smem_set[2][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    auto k1 = gemm::grouped_gemm_tc_kernel<WF, true>;
    auto k2 = gemm::grouped_gemm_tc_kernel<WF, false>;
    if (dev < 64 && smem_set[1][dev] < smem) {
        CUDA_TRY(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        smem_set[1][dev] = smem;
    }
    if (dev < 64 && smem_set[0][dev] < smem) {
        CUDA_TRY(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        smem_set[0][dev] = smem;
    }
    const int64_t mt_bound = (TK + gemm::kTcM - 1) / gemm::kTcM + std::min<int64_t>(E, TK);
    gemm::TcParams tp{};
    tp.scale_bf16 = eng->scale_bf16;
    tp.counts = w.counts;
    tp.starts = w.starts;
    tp.mtile_start = w.mtile;
    tp.tokmap = w.tokmap;
    tp.topk = (int)K;
    tp.E = E;
    tp.err = eng->err;
    tp.group = eng->cfg.group_size;
    tp.bf16ops = (WF == 2 && act_bf16) ? 1 : 0;
    gemm::TcParams t1 = tp;  // gate_up: A = token rows, B = unit records (2 rows each)
    t1.a = a1;
    t1.wbase = eng->gu; t1.rec = eng->unit_bytes(); t1.rows_per_rec = 2; t1.rs = eng->rs1;
    t1.sc_off = 2 * eng->rs1; t1.ss = eng->ss1; t1.nrec = I; t1.K = H; t1.N = 2 * I;
    t1.ngk = H / std::max(1, tp.group);
    t1.ha = w.ha;
    k1<<<(unsigned)(mt_bound * (2 * I / gemm::kTcN)), gemm::kTcThreads, smem, st>>>(t1);
    CUDA_TRY(cudaGetLastError());
    gemm::TcParams t2 = tp;  // down: A = h rows, B = down row records
    t2.a = w.ha;
    t2.wbase = eng->dn; t2.rec = eng->row_bytes(); t2.rows_per_rec = 1; t2.rs = eng->rs2;
    t2.sc_off = eng->rs2; t2.ss = eng->ss2; t2.nrec = H; t2.K = I; t2.N = H;
    t2.ngk = I / std::max(1, tp.group);
    t2.out = w.out;
    k2<<<(unsigned)(mt_bound * (H / gemm::kTcN)), gemm::kTcThreads, smem, st>>>(t2);
    CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

// AWQ (W4A16) layers with many tokens: routing, the tcgen05 GEMMs on the 16-bit hidden rows,
// combine.  The per-expert tiles hold 128 tokens, so this pays off from ~24 tokens per call.
int forward_gemm_awq(moe_engine* eng, const void* x, void* y, const int32_t* ids, const float* tw, int64_t T,
                     int64_t K, int act_bf16, int out_kind, cudaStream_t st) {
    const int E = (int)eng->cfg.num_experts, H = (int)eng->cfg.hidden_size;
    const int TK = (int)(T * K);
    GemmWs w;
    if (int rc = gemm_workspace(eng, T, K, w)) return rc;
    const int nblk = (TK + gemm::kChunk - 1) / gemm::kChunk;
    const int eoff = eng->cfg.expert_offset;
    gemm::route_count_kernel<<<nblk, 256, E * 4, st>>>(ids, TK, (int)K, E, eoff, eng->emap, eng->emap_n, w.blk);
    gemm::route_scan_kernel<<<1, std::max(32, (E + 31) / 32 * 32), 2 * E * 4, st>>>(w.blk, nblk, E, w.counts, w.starts,
                                                                                  w.mtile, gemm::kTcM);
    gemm::route_place_kernel<<<nblk, 256, E * 4, st>>>(ids, TK, (int)K, E, eoff, eng->emap, eng->emap_n, w.blk, w.starts,
                                                       w.smap, w.tokmap);
    CUDA_TRY(cudaGetLastError());
    if (int rc = launch_gemms_tc<2>(eng, w, x, act_bf16, T, K, st)) return rc;
    const int64_t total = T * (H / 4);
    gemm::combine_kernel<<<(unsigned)std::min<int64_t>((total + 255) / 256, eng->num_sms * 16), 256, 0, st>>>(
        w.out, w.smap, tw, (int)T, (int)K, H, y, out_kind);
    CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

bool awq_gemm_ok(const moe_engine* eng) {
    const int64_t H = eng->cfg.hidden_size, I = eng->cfg.intermediate_size;
    return eng->cfg.quant_type == MOE_AWQ && H % 128 == 0 && I % 128 == 0 && eng->cfg.num_experts <= 1024;
}

template <bool Q4, int BT>
int launch_gemms_wm(moe_engine* eng, const gemm::GemmParams& g1, const gemm::GemmParams& g2, int64_t TK,
                    cudaStream_t st) {
    using S = gemm::StageW<Q4, BT>;
    const int smem = std::max(gemm::kStages * S::kBytes, BT * (gemm::kBN / 2 + 1) * 4);
    static thread_local int smem_set[2][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const int E = (int)eng->cfg.num_experts, H = (int)eng->cfg.hidden_size, I = (int)eng->cfg.intermediate_size;
    const int64_t mt_bound = (TK + BT - 1) / BT + std::min<int64_t>(E, TK);
    auto k1 = gemm::grouped_gemm_wm_kernel<Q4, true, BT>;
    auto k2 = gemm::grouped_gemm_wm_kernel<Q4, false, BT>;
    if (dev < 64 && smem_set[1][dev] < smem) {
        CUDA_TRY(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        smem_set[1][dev] = smem;
    }
    if (dev < 64 && smem_set[0][dev] < smem) {
        CUDA_TRY(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        smem_set[0][dev] = smem;
    }
    k1<<<(unsigned)(mt_bound * (2 * I / gemm::kBN)), gemm::kThreads, smem, st>>>(g1);
    CUDA_TRY(cudaGetLastError());
    k2<<<(unsigned)(mt_bound * (H / gemm::kBN)), gemm::kThreads, smem, st>>>(g2);
    CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

template <bool Q4, int BM>
int launch_gemms(moe_engine* eng, const gemm::GemmParams& g1, const gemm::GemmParams& g2, int64_t TK,
                 cudaStream_t st) {
    using S = gemm::Stage<Q4, BM>;
    const int smem = std::max(gemm::kStages * S::kBytes, BM * (gemm::kBN / 2 + 1) * 4);
    static thread_local int smem_set[2][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const int E = (int)eng->cfg.num_experts, H = (int)eng->cfg.hidden_size, I = (int)eng->cfg.intermediate_size;
    const int64_t mt_bound = (TK + BM - 1) / BM + std::min<int64_t>(E, TK);
    auto k1 = gemm::grouped_gemm_kernel<Q4, true, BM>;
    auto k2 = gemm::grouped_gemm_kernel<Q4, false, BM>;
    if (dev < 64 && smem_set[1][dev] < smem) {
        CUDA_TRY(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        smem_set[1][dev] = smem;
    }
    if (dev < 64 && smem_set[0][dev] < smem) {
        CUDA_TRY(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        smem_set[0][dev] = smem;
    }
    k1<<<(unsigned)(mt_bound * (2 * I / gemm::kBN)), gemm::kThreads, smem, st>>>(g1);
    CUDA_TRY(cudaGetLastError());
    k2<<<(unsigned)(mt_bound * (H / gemm::kBN)), gemm::kThreads, smem, st>>>(g2);
    CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

template <bool Q4>
int forward_gemm_t(moe_engine* eng, const void* x, void* y, const int32_t* ids, const float* tw, int64_t T, int64_t K,
                   int act_bf16, int out_kind, cudaStream_t st) {
    const int E = (int)eng->cfg.num_experts, H = (int)eng->cfg.hidden_size, I = (int)eng->cfg.intermediate_size;
    const int TK = (int)(T * K);
    GemmWs w;
    if (int rc = gemm_workspace(eng, T, K, w)) return rc;
    const int nblk = (TK + gemm::kChunk - 1) / gemm::kChunk;
    const int eoff = eng->cfg.expert_offset;
    gemm::route_count_kernel<<<nblk, 256, E * 4, st>>>(ids, TK, (int)K, E, eoff, eng->emap, eng->emap_n, w.blk);
    gemm::route_scan_kernel<<<1, std::max(32, (E + 31) / 32 * 32), 2 * E * 4, st>>>(w.blk, nblk, E, w.counts, w.starts,
                                                                                  w.mtile, std::abs(gemm_tile_rows(eng, TK)));
    gemm::route_place_kernel<<<nblk, 256, E * 4, st>>>(ids, TK, (int)K, E, eoff, eng->emap, eng->emap_n, w.blk, w.starts,
                                                       w.smap, w.tokmap);
    const int bm = gemm_tile_rows(eng, TK);
    if (bm == 128) {
        if (int rc = launch_gemms_tc<Q4 ? 1 : 0>(eng, w, x, act_bf16, T, K, st)) return rc;
    } else {
    {
        const int nb = (int)(T * (H / 32));
        gemm::quant_rows_kernel<Q4><<<std::min((nb + 255) / 256, eng->num_sms * 8), 256, 0, st>>>(
            static_cast<const uint8_t*>(x), act_bf16, (int)T, H, w.xq, w.xd, w.xs);
    }
    CUDA_TRY(cudaGetLastError());
    gemm::GemmParams gp{};
    gp.scale_bf16 = eng->scale_bf16;
    gp.counts = w.counts;
    gp.starts = w.starts;
    gp.mtile_start = w.mtile;
    gp.tokmap = w.tokmap;
    gp.topk = (int)K;
    gp.E = E;
    gemm::GemmParams g1 = gp;  // gate_up: A = token rows, B = unit records (2 rows each)
    g1.aq = w.xq; g1.ad = w.xd; g1.as = w.xs;
    g1.wbase = eng->gu; g1.rec = eng->unit_bytes(); g1.rows_per_rec = 2; g1.rs = eng->rs1;
    g1.sc_off = 2 * eng->rs1; g1.ss = eng->ss1; g1.nrec = I; g1.K = H; g1.N = 2 * I;
    g1.hq = w.hq; g1.hd = w.hd; g1.hs = w.hs;
    gemm::GemmParams g2 = gp;  // down: A = requantised h rows, B = down row records
    g2.aq = w.hq; g2.ad = w.hd; g2.as = w.hs;
    g2.wbase = eng->dn; g2.rec = eng->row_bytes(); g2.rows_per_rec = 1; g2.rs = eng->rs2;
    g2.sc_off = eng->rs2; g2.ss = eng->ss2; g2.nrec = H; g2.K = I; g2.N = H;
    g2.out = w.out;
    int rc;
    switch (bm) {
        case -8: rc = launch_gemms_wm<Q4, 8>(eng, g1, g2, TK, st); break;
        case -16: rc = launch_gemms_wm<Q4, 16>(eng, g1, g2, TK, st); break;
        case 16: rc = launch_gemms<Q4, 16>(eng, g1, g2, TK, st); break;
        case 32: rc = launch_gemms<Q4, 32>(eng, g1, g2, TK, st); break;
        default: rc = launch_gemms<Q4, 64>(eng, g1, g2, TK, st); break;
    }
    if (rc) return rc;
    }
    {
        const int64_t total = T * (H / 4);
        gemm::combine_kernel<<<(unsigned)std::min<int64_t>((total + 255) / 256, eng->num_sms * 16), 256, 0, st>>>(
            w.out, w.smap, tw, (int)T, (int)K, H, y, out_kind);
        CUDA_TRY(cudaGetLastError());
    }
    return MOE_OK;
}

// The placement map on the device: emap_n entries, then the replica split (world, rank).
int upload_expert_map(moe_engine* eng) {
    DeviceGuard g(eng->cfg.device);
    CUDA_TRY(cudaDeviceSynchronize());  // the old map may still be read by queued work
    if (eng->emap) CUDA_TRY(cudaFree(eng->emap));
    eng->emap = nullptr;
    std::vector<int32_t> m(eng->emap_host);
    m.push_back(eng->rep_world);
    m.push_back(eng->rep_rank);
    CUDA_TRY(cudaMalloc(&eng->emap, m.size() * sizeof(int32_t)));
    CUDA_TRY(cudaMemcpy(eng->emap, m.data(), m.size() * sizeof(int32_t), cudaMemcpyHostToDevice));
    eng->emap_n = (int32_t)eng->emap_host.size();
    return MOE_OK;
}

// Meaning of a device error code (ErrCode in common.cuh).
const char* device_error_meaning(int32_t c) {
    switch (c) {
        case kErrGridBarrier: return "grid barrier wait expired";
        case kErrFullWait: return "wait for weight data expired";
        case kErrEmptyWait: return "wait for a free pipeline stage expired";
        case kErrPeerWait: return "a peer rank did not arrive at the combine";
        case kErrRange: return "an activation block exceeds the float16 range of the tcgen05 GEMM path";
        default: return "unknown device error";
    }
}

// Errors that kernels recorded are reported at the entry of the next call on the engine,
// as the reference's TORCH_CHECKs would have raised: the host reads the mapped error word
// (no synchronisation in the common case).  On an error the engine waits for the device,
// clears the word and the barrier state so that later calls work, and fails this call.
int check_sticky_error(moe_engine* eng, cudaStream_t st) {
    if (!eng->herr) return MOE_OK;
    const int32_t v = *reinterpret_cast<volatile int32_t*>(eng->herr);
    if (v == 0) return MOE_OK;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cap) == cudaSuccess && cap == cudaStreamCaptureStatusNone) {
        CUDA_TRY(cudaDeviceSynchronize());
        *reinterpret_cast<volatile int32_t*>(eng->herr) = 0;
        CUDA_TRY(cudaMemset(eng->bar, 0, bar_bytes(eng)));
    }
    return fail(MOE_ERR_DEVICE, std::string("an earlier launch on this engine failed on the device: error ") +
                                    std::to_string(v) + " (" + device_error_meaning(v) +
                                    "); its output is invalid; the engine state has been reset");
}

// =================================================================== C ABI
extern "C" int moe_engine_create(const moe_config* cfg, moe_engine** out) {
    if (!cfg || !out) return fail(MOE_ERR_INVALID, "null argument");
    *out = nullptr;
    const int64_t E = cfg->num_experts, H = cfg->hidden_size, I = cfg->intermediate_size;
    if (E <= 0 || H <= 0 || I <= 0) return fail(MOE_ERR_INVALID, "E, H, I must be positive");
    if (H % 32 != 0) return fail(MOE_ERR_INVALID, "hidden_size must be multiple of 32");
    if (I % 32 != 0) return fail(MOE_ERR_INVALID, "intermediate_size must be multiple of 32");
    if (cfg->quant_type < MOE_Q8_0 || cfg->quant_type > MOE_AWQ)
        return fail(MOE_ERR_INVALID, "quant_type must be 0 (Q8_0), 1 (Q4_0) or 2 (AWQ)");
    if (cfg->quant_type == MOE_AWQ) {
        const int g = cfg->group_size;
        if (g <= 0 || g % 32 != 0 || H % g != 0 || I % g != 0)
            return fail(MOE_ERR_INVALID, "AWQ group_size must be a multiple of 32 dividing H and I");
    }
    int ndev = 0;
    CUDA_TRY(cudaGetDeviceCount(&ndev));
    if (cfg->device < 0 || cfg->device >= ndev) return fail(MOE_ERR_INVALID, "device ordinal out of range");
    DeviceGuard g(cfg->device);
    auto* eng = new moe_engine();
    eng->cfg = *cfg;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, cfg->device) != cudaSuccess) {
        delete eng;
        return fail(MOE_ERR_CUDA, "cudaGetDeviceProperties failed");
    }
    eng->num_sms = prop.multiProcessorCount;
    if (const char* v = std::getenv("MOE_GEMM_MIN_TOKENS")) eng->gemm_min_tokens = std::atoll(v);
    if (const char* v = std::getenv("MOE_DIST_REQUANT_MIN")) eng->dist_min_blocks = std::atoi(v);
    if (const char* v = std::getenv("MOE_DECODE_FLAGS")) eng->decode_flags = std::atoi(v);
    if (const char* v = std::getenv("MOE_TC_MIN_PER_EXPERT")) eng->tc_min_per_expert = std::atoll(v);
    if (const char* v = std::getenv("MOE_AWQ_GEMM_MIN_TOKENS")) eng->awq_gemm_min_tokens = std::atoll(v);
    if (const char* v = std::getenv("MOE_GEMM_BM")) {  // "w8" / "w16" weights-on-M, "16" / "32" / "64"
        const bool wm = v[0] == 'w';
        const int bm = std::atoi(wm ? v + 1 : v);
        if (wm && (bm == 8 || bm == 16)) eng->gemm_bm = -bm;
        else if (!wm && (bm == 16 || bm == 32 || bm == 64 || bm == 128)) eng->gemm_bm = bm;
    }
    if (const char* v = std::getenv("MOE_DECODE_SK")) eng->use_sk = std::atoi(v) != 0;
    if (const char* v = std::getenv("MOE_CL_MAX_TOKENS")) eng->cl_max_tokens = std::atoi(v);
    if (const char* v = std::getenv("MOE_PDL")) eng->pdl = std::atoi(v) != 0;
    if (const char* v = std::getenv("MOE_CL_COMBINE")) eng->cl_combine = std::strcmp(v, "kernel") == 0 ? 1 : 0;
    if (const char* v = std::getenv("MOE_CL_ITEM_BYTES")) eng->cl_item_bytes = std::max(512, std::atoi(v));
    if (const char* v = std::getenv("MOE_CL_SIZE")) {
        const int c = std::atoi(v);
        if (c == 1 || c == 2 || c == 4 || c == 8) eng->cl_size = c;
    }
    if (const char* v = std::getenv("MOE_SK_COST_A")) eng->sk_cost_a = std::max(0, std::atoi(v));
    if (const char* v = std::getenv("MOE_SK_MIN_CHUNKS")) eng->sk_min_chunks_per_cta = std::max(0, std::atoi(v));
    eng->max_smem = (int)prop.sharedMemPerBlockOptin;
    if (eng->cl_max_tokens < 0) eng->cl_max_tokens = cfg->quant_type == MOE_AWQ ? 8 : 1;  // where it is faster
    if (const char* v = std::getenv("MOE_TP_MAX_TOKENS")) eng->tp_max_tokens = std::atoi(v);
    if (eng->tp_max_tokens < 0) eng->tp_max_tokens = cfg->quant_type == MOE_AWQ ? 8 : 4;  // where it is faster
    if (const char* v = std::getenv("MOE_TP_SLICE_MAX")) eng->tp_slice_max = std::atoi(v);
    if (eng->tp_slice_max < 0) eng->tp_slice_max = cfg->quant_type == MOE_AWQ ? 32 : 0;  // measured crossover
    int rc = MOE_OK;
    rc = alloc_q_layout(eng);
    if (rc == MOE_OK) rc = ensure_workspace(eng, 64);
    if (rc == MOE_OK && (cudaEventCreate(&eng->ev0) != cudaSuccess || cudaEventCreate(&eng->ev1) != cudaSuccess))
        rc = fail(MOE_ERR_CUDA, "cudaEventCreate failed");
    if (rc != MOE_OK) {
        moe_engine_destroy(eng);
        return rc;
    }
    *out = eng;
    return MOE_OK;
}

extern "C" int moe_engine_destroy(moe_engine* eng) {
    if (!eng) return MOE_OK;
    DeviceGuard g(eng->cfg.device);
    cudaFree(eng->gu);
    cudaFree(eng->dn);
    cudaFree(eng->dk);
    cudaFree(eng->agu);
    cudaFree(eng->adn);
    cudaFree(eng->clpart);
    cudaFree(eng->dense_ids);
    cudaFree(eng->clmeta);
    cudaFree(eng->emap);
    cudaFree(eng->part);
    for (int q = 0; q < kMaxPeers; ++q)
        if (eng->peer_base[q]) cudaIpcCloseMemHandle(eng->peer_base[q]);
    cudaFree(eng->mbox);
    cudaFree(eng->h_ws);
    cudaFree(eng->bar);
    if (eng->herr) cudaFreeHost(eng->herr);
    cudaFree(eng->timeline);
    cudaFree(eng->gws);
    if (eng->ev0) cudaEventDestroy(eng->ev0);
    if (eng->ev1) cudaEventDestroy(eng->ev1);
    delete eng;
    return MOE_OK;
}

extern "C" int moe_engine_load_quantized(moe_engine* eng, const void* gu_qs, const void* gu_d, const void* dn_qs,
                                         const void* dn_d, int32_t scale_dtype, int32_t src_on_device,
                                         void* stream) {
    if (int rc = check_engine(eng)) return rc;
    if (eng->cfg.quant_type == MOE_AWQ) return fail(MOE_ERR_STATE, "AWQ engine: use moe_engine_load_awq");
    if (!gu_qs || !gu_d || !dn_qs || !dn_d) return fail(MOE_ERR_INVALID, "null weight pointer");
    if (scale_dtype != MOE_F16 && scale_dtype != MOE_BF16)
        return fail(MOE_ERR_INVALID, "scales must be float16 or bfloat16");
    DeviceGuard g(eng->cfg.device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t E = eng->cfg.num_experts, H = eng->cfg.hidden_size, I = eng->cfg.intermediate_size;
    const bool q4 = eng->cfg.quant_type == MOE_Q4_0;
    const int64_t gu_row = q4 ? H / 2 : H, dn_row = q4 ? I / 2 : I;
    struct Piece { const void* src; int64_t rows, row_bytes; uint8_t* dst; int64_t rec, base, part; int map; };
    const int64_t U1 = eng->unit_bytes(), R2 = eng->row_bytes();
    Piece pieces[4] = {
        {gu_qs, E * 2 * I, gu_row, eng->gu, U1, 0, eng->rs1, kGateUp},
        {gu_d, E * 2 * I, (H / 32) * 2, eng->gu, U1, 2 * (int64_t)eng->rs1, eng->ss1, kGateUp},
        {dn_qs, E * H, dn_row, eng->dn, R2, 0, 0, kDown},
        {dn_d, E * H, (I / 32) * 2, eng->dn, R2, eng->rs2, 0, kDown},
    };
    for (auto& pc : pieces) {
        const uint8_t* src = nullptr;
        uint8_t* owned = nullptr;
        if (int rc = stage_to_device(pc.src, (size_t)pc.rows * pc.row_bytes, src_on_device, st, &src, &owned)) return rc;
        pack_rows_kernel<<<(unsigned)pc.rows, 128, 0, st>>>(pc.dst, src, pc.rows, pc.row_bytes, pc.rec, pc.base,
                                                             pc.part, pc.map, I);
        CUDA_TRY(cudaGetLastError());
        if (owned) CUDA_TRY(cudaFreeAsync(owned, st));
    }
    if (int rc = build_down_chunks(eng, 0, E, st)) return rc;
    if (int rc = build_cl_layout(eng, 0, E, st)) return rc;
    CUDA_TRY(cudaStreamSynchronize(st));
    eng->scale_bf16 = scale_dtype == MOE_BF16;
    eng->loaded = true;
    return MOE_OK;
}

extern "C" int moe_engine_quantize_store_expert(moe_engine* eng, int64_t expert, int32_t proj, const void* w,
                                                int32_t w_dtype, int32_t src_on_device, void* stream) {
    if (int rc = check_engine(eng)) return rc;
    if (eng->cfg.quant_type != MOE_Q8_0)
        return fail(MOE_ERR_STATE, "online quantization is Q8_0 only; use store_quantized_repack()");
    if (!w) return fail(MOE_ERR_INVALID, "null weight");
    if (w_dtype != MOE_F32 && w_dtype != MOE_F16 && w_dtype != MOE_BF16)
        return fail(MOE_ERR_INVALID, "weight must be float32, float16 or bfloat16");
    const int64_t E = eng->cfg.num_experts, H = eng->cfg.hidden_size, I = eng->cfg.intermediate_size;
    if (expert < 0 || expert >= E) return fail(MOE_ERR_INVALID, "expert index out of range");
    if (proj < 0 || proj > 2) return fail(MOE_ERR_INVALID, "Unknown proj_name");
    if (eng->loaded && eng->scale_bf16) return fail(MOE_ERR_STATE, "engine holds bfloat16 scales");
    DeviceGuard g(eng->cfg.device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t rows = proj == 2 ? H : I, cols = proj == 2 ? I : H;
    const size_t esz = w_dtype == MOE_F32 ? 4 : 2;
    const uint8_t* src = nullptr;
    uint8_t* owned = nullptr;
    if (int rc = stage_to_device(w, (size_t)rows * cols * esz, src_on_device, st, &src, &owned)) return rc;
    uint8_t *qb, *sb;
    int64_t stride;
    if (proj == 2) {
        qb = eng->dn + (size_t)expert * H * eng->row_bytes();
        sb = qb + eng->rs2;
        stride = eng->row_bytes();
    } else {
        qb = eng->gu + (size_t)expert * I * eng->unit_bytes() + (size_t)proj * eng->rs1;
        sb = eng->gu + (size_t)expert * I * eng->unit_bytes() + 2 * (size_t)eng->rs1 + (size_t)proj * eng->ss1;
        stride = eng->unit_bytes();
    }
    const int64_t warps = rows * (cols / 32);
    quantize_weight_rows_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(src, w_dtype, rows, cols, qb,
                                                                                       sb, stride);
    CUDA_TRY(cudaGetLastError());
    if (owned) CUDA_TRY(cudaFreeAsync(owned, st));
    if (proj == 2) {
        if (int rc = build_down_chunks(eng, expert, expert + 1, st)) return rc;
        if (int rc = build_cl_layout(eng, expert, expert + 1, st)) return rc;
    }
    CUDA_TRY(cudaStreamSynchronize(st));
    eng->scale_bf16 = 0;
    eng->loaded = true;
    return MOE_OK;
}

extern "C" int moe_engine_load_awq(moe_engine* eng, const void* w13_qw, const void* w13_sc, const void* w13_qz,
                                   const void* w2_qw, const void* w2_sc, const void* w2_qz, int32_t src_on_device,
                                   void* stream) {
    if (int rc = check_engine(eng)) return rc;
    if (eng->cfg.quant_type != MOE_AWQ) return fail(MOE_ERR_STATE, "not an AWQ engine");
    if (!w13_qw || !w13_sc || !w13_qz || !w2_qw || !w2_sc || !w2_qz) return fail(MOE_ERR_INVALID, "null weight");
    DeviceGuard g(eng->cfg.device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t E = eng->cfg.num_experts, H = eng->cfg.hidden_size, I = eng->cfg.intermediate_size;
    const int64_t G = eng->cfg.group_size;
    const void* srcs[6] = {w13_qw, w13_sc, w13_qz, w2_qw, w2_sc, w2_qz};
    const size_t sizes[6] = {(size_t)E * H * (2 * I / 8) * 4, (size_t)E * (H / G) * 2 * I * 2,
                             (size_t)E * (H / G) * (2 * I / 8) * 4, (size_t)E * I * (H / 8) * 4,
                             (size_t)E * (I / G) * H * 2, (size_t)E * (I / G) * (H / 8) * 4};
    const uint8_t* dev[6];
    uint8_t* owned[6] = {};
    for (int i = 0; i < 6; ++i)
        if (int rc = stage_to_device(srcs[i], sizes[i], src_on_device, st, &dev[i], &owned[i])) return rc;
    const int64_t U1 = eng->unit_bytes(), R2 = eng->row_bytes();
    {   // gate_up: Kd = H, N = 2I
        const int64_t N = 2 * I, n1 = N * (H / 2), n2 = N * (H / G);
        awq_pack_q_kernel<<<dim3((unsigned)((n1 + 255) / 256), (unsigned)E), 256, 0, st>>>(
            eng->gu, reinterpret_cast<const int32_t*>(dev[0]), H, N, 1, I, H, U1, eng->rs1, eng->ss1);
        awq_pack_sz_kernel<<<dim3((unsigned)((n2 + 255) / 256), (unsigned)E), 256, 0, st>>>(
            eng->gu, reinterpret_cast<const uint16_t*>(dev[1]), reinterpret_cast<const int32_t*>(dev[2]), H / G, N, 1,
            I, H, U1, eng->rs1, eng->ss1);
    }
    {   // down: Kd = I, N = H
        const int64_t N = H, n1 = N * (I / 2), n2 = N * (I / G);
        awq_pack_q_kernel<<<dim3((unsigned)((n1 + 255) / 256), (unsigned)E), 256, 0, st>>>(
            eng->dn, reinterpret_cast<const int32_t*>(dev[3]), I, N, 0, I, H, R2, eng->rs2, eng->ss2);
        awq_pack_sz_kernel<<<dim3((unsigned)((n2 + 255) / 256), (unsigned)E), 256, 0, st>>>(
            eng->dn, reinterpret_cast<const uint16_t*>(dev[4]), reinterpret_cast<const int32_t*>(dev[5]), I / G, N, 0,
            I, H, R2, eng->rs2, eng->ss2);
    }
    CUDA_TRY(cudaGetLastError());
    if (int rc = build_cl_layout(eng, 0, E, st)) return rc;
    for (int i = 0; i < 6; ++i)
        if (owned[i]) CUDA_TRY(cudaFreeAsync(owned[i], st));
    CUDA_TRY(cudaStreamSynchronize(st));
    eng->loaded = true;
    return MOE_OK;
}

// ============================================================ two-pass decode
struct TpPlan {
    TpParams p;
    size_t smem1, smem2;
};

// Plan of the two-pass kernels for T tokens; false when they do not apply.
bool plan_decode_tp(moe_engine* eng, int T, int K, TpPlan& pl) {
    const int qt = eng->cfg.quant_type;
    if (T < 1 || T > eng->tp_max_tokens || T * K > kTpMaxPairs || !eng->adn) return false;
    const int H = (int)eng->cfg.hidden_size, I = (int)eng->cfg.intermediate_size;
    const bool awq = qt == MOE_AWQ;
    if (awq && (!eng->agu || !awq_recs_ok(eng) || H % kAwqK || I % kAwqK)) return false;
    if (!awq && (H % 64 || I % 32)) return false;
    TpParams& p = pl.p;
    std::memset(&p, 0, sizeof(p));
    p.E = (int)eng->cfg.num_experts; p.e_off = (int)eng->cfg.expert_offset; p.H = H; p.I = I; p.T = T; p.K = K;
    p.emap = eng->emap; p.emap_n = eng->emap_n;
    p.flags = eng->decode_flags;
    p.rs1 = eng->rs1; p.ss1 = eng->ss1;
    p.scale_bf16 = eng->scale_bf16;
    p.ncol = std::min(T, kTpCols);
    if (awq) {
        pl.smem1 = (size_t)2 * (H / kAwqK) * kAwqGuRec + (size_t)T * (H + 8) * 2 + (size_t)T * (H / kAwqK) * 4;
        pl.smem2 = (size_t)(I / kAwqK) * kAwqDnRec + (size_t)p.ncol * (I + 8) * 2 + (size_t)p.ncol * (I / kAwqK) * 4;
    } else {
        const int64_t SB = 32 * (qt == MOE_Q4_0 ? 16 : 32) + 64;
        pl.smem1 = (size_t)kTpUnitsQ * eng->unit_bytes() + (size_t)T * H + (size_t)T * (H / 32) * 8;
        pl.smem2 = (size_t)(I / 32) * SB + (size_t)p.ncol * I + (size_t)p.ncol * (I / 32) * 8;
    }
    const size_t lim = (size_t)eng->max_smem - 16384;  // static shared memory of the kernels (< 16 KB)
    return pl.smem1 <= lim && pl.smem2 <= lim;
}

// Largest dynamic shared memory next to the kernel's static share, and the full carveout, so
// that pass 2's CTAs can start on SMs that still run pass 1's (a different carveout waits for
// the SM to drain).  Once per kernel and device.
int tp_kernel_attrs(const void* fn, int max_smem) {
    static std::mutex mu;
    static std::vector<std::pair<const void*, int>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    for (auto& d : done)
        if (d.first == fn && d.second == dev) return MOE_OK;
    cudaFuncAttributes fa{};
    CUDA_TRY(cudaFuncGetAttributes(&fa, fn));
    CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem - (int)fa.sharedSizeBytes));
    CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    done.emplace_back(fn, dev);
    return MOE_OK;
}

int launch_decode_tp(moe_engine* eng, TpPlan& pl, bool act_bf16, cudaStream_t st) {
    const TpParams& p = pl.p;
    const int qt = eng->cfg.quant_type;
    void (*k1)(TpParams);
    void (*k2)(TpParams);
    dim3 g1;
    if (qt == MOE_AWQ) {
        k1 = act_bf16 ? tp_gate_up_kernel<true> : tp_gate_up_kernel<false>;
        k2 = act_bf16 ? tp_down_kernel<true> : tp_down_kernel<false>;
        g1 = dim3(p.I / 16, p.T * p.K);
    } else {
        k1 = qt == MOE_Q4_0 ? tp_gate_up_q_kernel<true> : tp_gate_up_q_kernel<false>;
        k2 = qt == MOE_Q4_0 ? tp_down_q_kernel<true> : tp_down_q_kernel<false>;
        g1 = dim3((p.I + kTpUnitsQ - 1) / kTpUnitsQ, p.T * p.K);
    }
    if (int rc = tp_kernel_attrs(reinterpret_cast<const void*>(k1), eng->max_smem)) return rc;
    if (int rc = tp_kernel_attrs(reinterpret_cast<const void*>(k2), eng->max_smem)) return rc;
    cudaLaunchAttribute attr[1];
    // programmatic dependent launch: each kernel waits (griddepcontrol.wait) for its stream
    // predecessor before it reads that one's output
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(kTpWarpsA * 32);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = eng->pdl ? 1 : 0;
    cfg.gridDim = g1;
    cfg.dynamicSmemBytes = pl.smem1;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, k1, p));
    cfg.gridDim = dim3(p.H / 32, p.T * p.K);
    cfg.blockDim = dim3((qt == MOE_AWQ ? kTpWarpsB : kTpWarpsBQ) * 32);
    cfg.dynamicSmemBytes = pl.smem2;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, k2, p));
    return MOE_OK;
}

extern "C" int moe_engine_reserve(moe_engine* eng, int64_t max_tokens, int64_t top_k) {
    if (int rc = check_engine(eng)) return rc;
    if (max_tokens < 0 || top_k <= 0) return fail(MOE_ERR_INVALID, "bad reserve size");
    DeviceGuard g(eng->cfg.device);
    if ((max_tokens > eng->gemm_min_tokens && gemm_path_ok(eng)) ||
        (max_tokens > eng->awq_gemm_min_tokens && awq_gemm_ok(eng))) {  // the grouped-GEMM path's workspace
        GemmWs w;
        if (int rc = gemm_workspace(eng, max_tokens, top_k, w)) return rc;
    }
    if (eng->dk)
        if (int rc = ensure_part(eng, std::min<int64_t>(max_tokens, 64))) return rc;
    if (int rc = ensure_clpart(eng, std::min<int64_t>(max_tokens, 8) * top_k * kClMaxQ)) return rc;
    if (eng->cl_combine != 0 && 1 + std::min<int64_t>(max_tokens, 8) * top_k > eng->clmeta_cap) {
        cudaFree(eng->clmeta);
        eng->clmeta = nullptr;
        eng->clmeta_cap = 1 + std::min<int64_t>(max_tokens, 8) * top_k;
        CUDA_TRY(cudaMalloc(&eng->clmeta, (size_t)eng->clmeta_cap * 4));
    }
    return ensure_workspace(eng, std::min<int64_t>(max_tokens, 64) * top_k);
}

extern "C" int moe_engine_p2p_covers(moe_engine* eng, int64_t num_tokens);

// Peer-combine parameters of a decode launch.
void fill_peer_combine(moe_engine* eng, PeerCombine& pc) {
    std::memset(&pc, 0, sizeof(pc));
    pc.rank = eng->p2p_rank;
    pc.world = eng->p2p_world;
    pc.tcap = eng->p2p_tcap;
    for (int q = 0; q < eng->p2p_world; ++q) {
        uint8_t* base = q == eng->p2p_rank ? eng->mbox : static_cast<uint8_t*>(eng->peer_base[q]);
        pc.data[q] = reinterpret_cast<float*>(base);
        pc.flag[q] = reinterpret_cast<unsigned long long*>(base + eng->mbox_data_bytes);
    }
}

extern "C" int moe_engine_forward(moe_engine* eng, const void* x, void* y, const int32_t* topk_ids,
                                  const float* topk_w, int64_t T, int64_t K, int32_t act_dtype, int32_t out_dtype,
                                  void* stream) {
    if (int rc = check_engine(eng)) return rc;
    if (!eng->loaded) return fail(MOE_ERR_STATE, "no weights loaded");
    if (T < 0 || K <= 0 || K > 64) return fail(MOE_ERR_INVALID, "num_tokens must be >= 0 and 1 <= top_k <= 64");
    if (act_dtype != MOE_F16 && act_dtype != MOE_BF16) return fail(MOE_ERR_INVALID, "hidden must be f16 or bf16");
    if (out_dtype != MOE_F16 && out_dtype != MOE_BF16 && out_dtype != MOE_F32)
        return fail(MOE_ERR_INVALID, "bad output dtype");
    if (T > 0 && (!x || !y || !topk_ids || !topk_w)) return fail(MOE_ERR_INVALID, "null tensor pointer");
    DeviceGuard g(eng->cfg.device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (int rc = check_sticky_error(eng, st)) return rc;
    if (T == 0) return MOE_OK;
    const int64_t H = eng->cfg.hidden_size;
    const size_t xe = 2, ye = out_dtype == MOE_F32 ? 4 : 2;
    if (eng->p2p_active && !moe_engine_p2p_covers(eng, T))
        return fail(MOE_ERR_STATE, "peer combine covers decode-size calls only; use the fp32 partial and an all-reduce");
    // decode sizes: the two-pass kernels, in token slices of at most tp_max_tokens up to
    // tp_slice_max tokens (each slice's pass 1 waits for the previous slice's pass 2)
    if (!eng->p2p_active && (T <= eng->tp_max_tokens || T <= eng->tp_slice_max) && eng->tp_max_tokens > 0) {
        const int64_t S = std::min<int64_t>(T, eng->tp_max_tokens);
        TpPlan tp;
        if (plan_decode_tp(eng, (int)S, (int)K, tp)) {
            if (int rc = ensure_clpart(eng, S * K)) return rc;   // part [S K][H]
            if (int rc = ensure_workspace(eng, S * K)) return rc;  // h, counters, error word
            cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
            CUDA_TRY(cudaStreamIsCapturing(st, &cap));
            const bool timed = cap == cudaStreamCaptureStatusNone;
            if (timed) CUDA_TRY(cudaEventRecord(eng->ev0, st));
            const size_t ye = out_dtype == MOE_F32 ? 4 : 2;
            for (int64_t t0 = 0; t0 < T; t0 += S) {
                const int64_t n = std::min(S, T - t0);
                if (n != S && !plan_decode_tp(eng, (int)n, (int)K, tp)) return fail(MOE_ERR_INVALID, "plan failed");
                TpParams& p = tp.p;
                p.out_kind = out_dtype == MOE_F32 ? 2 : (out_dtype == MOE_BF16 ? 1 : 0);
                p.act_bf16 = act_dtype == MOE_BF16;
                p.x = static_cast<const uint8_t*>(x) + (size_t)t0 * H * 2;
                p.y = static_cast<uint8_t*>(y) + (size_t)t0 * H * ye;
                p.ids = topk_ids + t0 * K;
                p.tw = topk_w + t0 * K;
                p.gu = eng->cfg.quant_type == MOE_AWQ ? eng->agu : eng->gu;
                p.dn = eng->adn;
                p.h = eng->h_ws;
                p.part = eng->clpart;
                p.cnt = reinterpret_cast<unsigned int*>(reinterpret_cast<uint8_t*>(eng->bar) + 256);
                p.err = eng->err;
                p.dbg = eng->timeline_ctas >= (int)(std::max<int64_t>(H / 32, p.I / 16) * n * K) ? eng->timeline : nullptr;
                if (int rc = launch_decode_tp(eng, tp, act_dtype == MOE_BF16, st)) return rc;
            }
            if (timed) {
                CUDA_TRY(cudaEventRecord(eng->ev1, st));
                eng->timed = true;
            }
            return MOE_OK;
        }
    }
    if (T > eng->awq_gemm_min_tokens && awq_gemm_ok(eng)) {  // AWQ: the tcgen05 GEMMs on the 16-bit rows
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        CUDA_TRY(cudaStreamIsCapturing(st, &cap));
        const bool timed = cap == cudaStreamCaptureStatusNone;
        if (timed) CUDA_TRY(cudaEventRecord(eng->ev0, st));
        const int okind = out_dtype == MOE_F32 ? 2 : (out_dtype == MOE_BF16 ? 1 : 0);
        if (int rc = forward_gemm_awq(eng, x, y, topk_ids, topk_w, T, K, act_dtype == MOE_BF16, okind, st)) return rc;
        if (timed) {
            CUDA_TRY(cudaEventRecord(eng->ev1, st));
            eng->timed = true;
        }
        return MOE_OK;
    }
    if (T > eng->gemm_min_tokens && gemm_path_ok(eng)) {  // dense enough for the grouped GEMMs
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        CUDA_TRY(cudaStreamIsCapturing(st, &cap));
        const bool timed = cap == cudaStreamCaptureStatusNone;
        if (timed) CUDA_TRY(cudaEventRecord(eng->ev0, st));
        const int okind = out_dtype == MOE_F32 ? 2 : (out_dtype == MOE_BF16 ? 1 : 0);
        const int rc = eng->cfg.quant_type == MOE_Q4_0
                           ? forward_gemm_t<true>(eng, x, y, topk_ids, topk_w, T, K, act_dtype == MOE_BF16, okind, st)
                           : forward_gemm_t<false>(eng, x, y, topk_ids, topk_w, T, K, act_dtype == MOE_BF16, okind, st);
        if (rc) return rc;
        if (timed) {
            CUDA_TRY(cudaEventRecord(eng->ev1, st));
            eng->timed = true;
        }
        return MOE_OK;
    }
    // decode sizes: the cluster kernel when it applies
    if (!eng->p2p_active && T <= eng->cl_max_tokens) {
        ClPlan cp;
        const int qt = eng->cfg.quant_type;
        const int fmt = qt == MOE_Q4_0 ? kQ4 : (qt == MOE_AWQ ? kAWQ : kQ8);
        bool use = plan_decode_cl(eng, (int)T, (int)K, cp);
        if (use) {
            const bool xbf = act_dtype == MOE_BF16;
            const int rc = fmt == kQ4 ? setup_decode_cl<kQ4, true>(eng)
                                      : (fmt == kAWQ ? (xbf ? setup_decode_cl<kAWQ, true>(eng)
                                                            : setup_decode_cl<kAWQ, false>(eng))
                                                     : setup_decode_cl<kQ8, true>(eng));
            if (rc) return rc;
            use = eng->cl_clusters[fmt] >= 1;
        }
        if (use) {
            if (int rc = ensure_clpart(eng, T * K * kClMaxQ)) return rc;
            if (int rc = ensure_workspace(eng, 1)) return rc;  // combine counters and error word
            cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
            CUDA_TRY(cudaStreamIsCapturing(st, &cap));
            const bool timed = cap == cudaStreamCaptureStatusNone;
            if (timed) CUDA_TRY(cudaEventRecord(eng->ev0, st));
            ClParams& p = cp.p;
            p.act_bf16 = act_dtype == MOE_BF16;
            p.out_kind = out_dtype == MOE_F32 ? 2 : (out_dtype == MOE_BF16 ? 1 : 0);
            p.x = x; p.y = y; p.ids = topk_ids; p.tw = topk_w;
            p.gu = qt == MOE_AWQ ? eng->agu : eng->gu;
            p.dn = eng->adn;
            p.part = eng->clpart;
            p.cnt = reinterpret_cast<unsigned int*>(reinterpret_cast<uint8_t*>(eng->bar) + 128);
            if (eng->cl_combine == 1 || (eng->cl_combine < 0 && T > 1)) {
                if (1 + T * K > eng->clmeta_cap) {
                    CUDA_TRY(cudaDeviceSynchronize());
                    cudaFree(eng->clmeta);
                    eng->clmeta = nullptr;
                    eng->clmeta_cap = std::max<int64_t>(1 + T * K, 1 + 8 * 64);
                    CUDA_TRY(cudaMalloc(&eng->clmeta, (size_t)eng->clmeta_cap * 4));
                }
                p.meta = eng->clmeta;
            }
            p.err = eng->err;
            p.dbg = eng->timeline;
            const int rc = qt == MOE_Q4_0 ? launch_decode_cl<kQ4, true>(eng, cp, st)
                           : qt == MOE_AWQ ? (p.act_bf16 ? launch_decode_cl<kAWQ, true>(eng, cp, st)
                                                         : launch_decode_cl<kAWQ, false>(eng, cp, st))
                                           : launch_decode_cl<kQ8, true>(eng, cp, st);
            if (rc) return rc;
            if (timed) {
                CUDA_TRY(cudaEventRecord(eng->ev1, st));
                eng->timed = true;
            }
            return MOE_OK;
        }
    }
    // token slice that fits the decode kernel's shared-memory plan
    // (the split-K kernel when its plan fits)
    auto plan = [&](int n, DecodePlan& pl) {
        return plan_decode_sk(eng, n, (int)K, pl) || plan_decode(eng, n, (int)K, pl);
    };
    int64_t slice = T;
    DecodePlan pl;
    while (slice > 0 && !plan((int)slice, pl)) slice = slice > 8 ? slice / 2 : slice - 1;
    if (slice == 0) return fail(MOE_ERR_INVALID, "shapes exceed the decode kernel's shared memory");
    if (pl.sk) {
        if (int rc = ensure_part(eng, slice)) return rc;
    } else if (int rc = ensure_workspace(eng, slice * K)) {
        return rc;
    }
    if (int rc = ensure_workspace(eng, 1)) return rc;  // barrier counter and error word
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    CUDA_TRY(cudaStreamIsCapturing(st, &cap));
    const bool timed = cap == cudaStreamCaptureStatusNone;
    if (timed) CUDA_TRY(cudaEventRecord(eng->ev0, st));
    for (int64_t t0 = 0; t0 < T; t0 += slice) {
        const int64_t n = std::min(slice, T - t0);
        if (n != slice && !plan((int)n, pl)) return fail(MOE_ERR_INVALID, "plan failed");
        DecodeParams& p = pl.p;
        p.T = (int)n;
        p.act_bf16 = act_dtype == MOE_BF16;
        p.out_kind = out_dtype == MOE_F32 ? 2 : (out_dtype == MOE_BF16 ? 1 : 0);
        p.x = static_cast<const uint8_t*>(x) + (size_t)t0 * H * xe;
        p.y = static_cast<uint8_t*>(y) + (size_t)t0 * H * ye;
        p.ids = topk_ids + t0 * K;
        p.tw = topk_w + t0 * K;
        p.gu = eng->gu; p.dn = eng->dn;
        p.h_ws = eng->h_ws; p.bar = reinterpret_cast<unsigned long long*>(eng->bar); p.err = eng->err;
        p.dk = eng->dk; p.part = eng->part;
        if (eng->p2p_active) {
            if (n > eng->p2p_tcap) return fail(MOE_ERR_INVALID, "tokens per decode launch exceed the mailbox capacity");
            fill_peer_combine(eng, p.pc);
        }
        p.dbg = eng->timeline;
        const int qt = eng->cfg.quant_type;
        const int rc = qt == MOE_Q4_0 ? launch_decode<kQ4>(pl, st)
                                      : (qt == MOE_AWQ ? launch_decode<kAWQ>(pl, st) : launch_decode<kQ8>(pl, st));
        if (rc) return rc;
    }
    if (timed) {
        CUDA_TRY(cudaEventRecord(eng->ev1, st));
        eng->timed = true;
    }
    return MOE_OK;
}

// Dense MLP through the same fused kernels: every token routed to one expert with weight 1.
__global__ void fill_dense_route_kernel(int32_t* ids, float* w, int64_t n, int32_t expert) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        ids[i] = expert;
        w[i] = 1.0f;
    }
}

extern "C" int moe_engine_forward_dense(moe_engine* eng, int64_t expert, const void* x, void* y, int64_t T,
                                        int32_t act_dtype, int32_t out_dtype, void* stream) {
    if (int rc = check_engine(eng)) return rc;
    if (expert < 0 || expert >= eng->cfg.num_experts) return fail(MOE_ERR_INVALID, "expert index out of range");
    if (T < 0) return fail(MOE_ERR_INVALID, "num_tokens must be >= 0");
    if (T == 0) return MOE_OK;
    DeviceGuard g(eng->cfg.device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (T > eng->dense_cap) {
        CUDA_TRY(cudaDeviceSynchronize());  // the old buffers may still be in use by queued work
        cudaFree(eng->dense_ids);
    cudaFree(eng->clmeta);
        eng->dense_ids = nullptr;
        int64_t cap = std::max<int64_t>(64, eng->dense_cap);
        while (cap < T) cap *= 2;
        CUDA_TRY(cudaMalloc(&eng->dense_ids, (size_t)cap * 8));
        eng->dense_cap = cap;
        eng->dense_expert = -1;
    }
    int32_t* ids = reinterpret_cast<int32_t*>(eng->dense_ids);
    float* w = reinterpret_cast<float*>(ids + eng->dense_cap);
    // global id of the expert for the routing (placement map or contiguous block)
    int32_t gid = (int32_t)(expert + eng->cfg.expert_offset);
    if (!eng->emap_host.empty()) {
        gid = -1;
        for (size_t gg = 0; gg < eng->emap_host.size(); ++gg)
            if (eng->emap_host[gg] >= 0 && (eng->emap_host[gg] & ~kReplicaFlag) == expert) gid = (int32_t)gg;
        if (gid < 0) return fail(MOE_ERR_INVALID, "expert is not in this engine's placement map");
    }
    if (eng->dense_expert != gid) {  // (re)fill on the stream; stays valid for later calls
        fill_dense_route_kernel<<<(unsigned)((eng->dense_cap + 255) / 256), 256, 0, st>>>(ids, w, eng->dense_cap, gid);
        CUDA_TRY(cudaGetLastError());
        eng->dense_expert = gid;
    }
    return moe_engine_forward(eng, x, y, ids, w, T, 1, act_dtype, out_dtype, stream);
}

extern "C" int moe_engine_last_time_ms(moe_engine* eng, double* ms) {
    if (int rc = check_engine(eng)) return rc;
    if (!ms) return fail(MOE_ERR_INVALID, "null output");
    *ms = 0.0;
    if (!eng->timed) return MOE_OK;
    DeviceGuard g(eng->cfg.device);
    CUDA_TRY(cudaEventSynchronize(eng->ev1));
    float f = 0.f;
    CUDA_TRY(cudaEventElapsedTime(&f, eng->ev0, eng->ev1));
    *ms = f;
    return MOE_OK;
}

extern "C" int moe_engine_device_error(moe_engine* eng, int32_t* code) {
    if (int rc = check_engine(eng)) return rc;
    if (!code) return fail(MOE_ERR_INVALID, "null output");
    DeviceGuard g(eng->cfg.device);
    CUDA_TRY(cudaDeviceSynchronize());
    const int32_t v = eng->herr ? *reinterpret_cast<volatile int32_t*>(eng->herr) : 0;
    *code = v;
    if (v != 0) {  // clear the error word and the barrier state
        *reinterpret_cast<volatile int32_t*>(eng->herr) = 0;
        CUDA_TRY(cudaMemset(eng->bar, 0, bar_bytes(eng)));
    }
    return MOE_OK;
}

extern "C" int moe_engine_export_expert(moe_engine* eng, int64_t expert, int32_t which, void* qs_out,
                                        void* d_out) {
    if (int rc = check_engine(eng)) return rc;
    const int64_t E = eng->cfg.num_experts, H = eng->cfg.hidden_size, I = eng->cfg.intermediate_size;
    if (expert < 0 || expert >= E || (which != 0 && which != 1) || !qs_out || !d_out)
        return fail(MOE_ERR_INVALID, "bad export argument");
    DeviceGuard g(eng->cfg.device);
    const bool awq = eng->cfg.quant_type == MOE_AWQ;
    const bool q4 = eng->cfg.quant_type == MOE_Q4_0 || awq;
    const int64_t rows = which == 0 ? 2 * I : H;
    const int64_t kd = which == 0 ? H : I;
    const int64_t qrow = q4 ? kd / 2 : kd;
    const int64_t ng = awq ? kd / eng->cfg.group_size : kd / 32;
    const int64_t srow = awq ? ng * 3 : ng * 2;  // AWQ: bf16 scales then u8 zeros
    const int map = which == 0 ? kGateUp : kDown;
    const uint8_t* base = which == 0 ? eng->gu + (size_t)expert * I * eng->unit_bytes()
                                     : eng->dn + (size_t)expert * H * eng->row_bytes();
    const int64_t rec = which == 0 ? eng->unit_bytes() : eng->row_bytes();
    uint8_t *dq = nullptr, *ds = nullptr;
    CUDA_TRY(cudaMalloc(&dq, rows * qrow));
    CUDA_TRY(cudaMalloc(&ds, rows * srow));
    unpack_rows_kernel<<<(unsigned)rows, 128>>>(dq, base, rows, qrow, rec, 0, which == 0 ? eng->rs1 : 0, map, I);
    unpack_rows_kernel<<<(unsigned)rows, 128>>>(ds, base, rows, srow, rec, which == 0 ? 2 * (int64_t)eng->rs1 : eng->rs2,
                                                which == 0 ? eng->ss1 : 0, map, I);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaMemcpy(qs_out, dq, rows * qrow, cudaMemcpyDeviceToHost));
    CUDA_TRY(cudaMemcpy(d_out, ds, rows * srow, cudaMemcpyDeviceToHost));
    cudaFree(dq);
    cudaFree(ds);
    return MOE_OK;
}

extern "C" int moe_route_topk(const float* logits, int64_t T, int64_t E, int64_t K, int32_t renorm, int32_t* ids,
                              float* w, void* stream) {
    if (T < 0 || E <= 0 || K <= 0 || K > 16 || K > E) return fail(MOE_ERR_INVALID, "need 1 <= top_k <= min(16, E)");
    if (E > 4096) return fail(MOE_ERR_INVALID, "num_experts > 4096");
    if (T == 0) return MOE_OK;
    if (!logits || !ids || !w) return fail(MOE_ERR_INVALID, "null pointer");
    const int wpb = 4;
    const size_t smem = (size_t)wpb * ((E + 31) / 32) * 4;
    route_topk_kernel<<<(unsigned)((T + wpb - 1) / wpb), wpb * 32, smem, static_cast<cudaStream_t>(stream)>>>(
        logits, (int)T, (int)E, (int)K, renorm, ids, w);
    CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

extern "C" int moe_route_gemm_topk(const void* hidden, int32_t act_dtype, const void* router_w, int32_t w_dtype,
                                   int64_t T, int64_t H, int64_t E, int64_t K, int32_t renorm, int32_t* ids,
                                   float* topk_w, float* logits, void* stream) {
    if (T < 0 || H <= 0 || E <= 0 || K <= 0 || K > 16 || K > E) return fail(MOE_ERR_INVALID, "need 1 <= top_k <= min(16, E)");
    if (act_dtype != MOE_F16 && act_dtype != MOE_BF16) return fail(MOE_ERR_INVALID, "hidden must be f16 or bf16");
    if (w_dtype != MOE_F16 && w_dtype != MOE_BF16 && w_dtype != MOE_F32)
        return fail(MOE_ERR_INVALID, "router weight must be f16, bf16 or f32");
    if (H % 8 != 0) return fail(MOE_ERR_INVALID, "hidden_size must be a multiple of 8");
    const size_t smem = ((size_t)H + E + (E + 31) / 32) * 4;
    if (smem > 200 * 1024) return fail(MOE_ERR_INVALID, "hidden_size + num_experts too large for the router kernel");
    if (T == 0) return MOE_OK;
    if (!hidden || !router_w || !ids || !topk_w) return fail(MOE_ERR_INVALID, "null pointer");
    if (smem > 48 * 1024)
        CUDA_TRY(cudaFuncSetAttribute(route_gemm_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    route_gemm_topk_kernel<<<(unsigned)T, kRgWarps * 32, smem, static_cast<cudaStream_t>(stream)>>>(
        hidden, act_dtype == MOE_BF16, router_w, w_dtype, (int)H, (int)E, (int)K, renorm, ids, topk_w, logits);
    CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

extern "C" int moe_route_permute(const int32_t* ids, int64_t T, int64_t K, int64_t E, int32_t* counts, int32_t* starts,
                                 int32_t* token_map, int32_t* scatter_map, void* stream) {
    if (T < 0 || K <= 0 || E <= 0) return fail(MOE_ERR_INVALID, "bad sizes");
    if (!counts || !starts || (T > 0 && (!ids || !token_map || !scatter_map)))
        return fail(MOE_ERR_INVALID, "null pointer");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int TK = (int)(T * K);
    int32_t* tmp = nullptr;
    CUDA_TRY(cudaMallocAsync(&tmp, (size_t)std::max(TK, 1) * 4, st));
    route_permute_kernel<<<1, 32, 0, st>>>(ids, TK, (int)E, counts, starts, token_map, scatter_map, tmp);
    CUDA_TRY(cudaGetLastError());
    if (TK > 0) {
        token_map_kernel<<<(TK + 255) / 256, 256, 0, st>>>(scatter_map, TK, (int)K, token_map);
        CUDA_TRY(cudaGetLastError());
    }
    CUDA_TRY(cudaFreeAsync(tmp, st));
    return MOE_OK;
}

extern "C" int moe_quantize_rows_q8_0(const void* x, int32_t dtype, int64_t rows, int64_t cols, int8_t* qs, float* d,
                                      void* stream) {
    if (rows < 0 || cols <= 0 || cols % 32 != 0) return fail(MOE_ERR_INVALID, "cols must be a positive multiple of 32");
    if (dtype != MOE_F16 && dtype != MOE_BF16 && dtype != MOE_F32) return fail(MOE_ERR_INVALID, "bad dtype");
    if (rows == 0) return MOE_OK;
    if (!x || !qs || !d) return fail(MOE_ERR_INVALID, "null pointer");
    const int64_t warps = rows * (cols / 32);
    quantize_rows_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, dtype, rows, cols, qs, d);
    CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

extern "C" int moe_engine_debug_timeline(moe_engine* eng, int32_t enable, uint64_t* out, int32_t max_entries,
                                         int32_t* n_entries) {
    if (int rc = check_engine(eng)) return rc;
    DeviceGuard g(eng->cfg.device);
    if (enable && !eng->timeline) {
        // one row per CTA: the persistent kernels use num_sms rows, the two-pass kernels up to
        // (row tiles x pieces) rows
        const int rows = std::max(eng->num_sms, 1024);
        CUDA_TRY(cudaMalloc(&eng->timeline, (size_t)rows * kStamps * sizeof(unsigned long long)));
        CUDA_TRY(cudaMemset(eng->timeline, 0, (size_t)rows * kStamps * sizeof(unsigned long long)));
        eng->timeline_ctas = rows;
    }
    if (!enable && eng->timeline) {
        CUDA_TRY(cudaDeviceSynchronize());
        cudaFree(eng->timeline);
        eng->timeline = nullptr;
        eng->timeline_ctas = 0;
    }
    if (n_entries) *n_entries = eng->timeline_ctas * kStamps;
    if (out && eng->timeline) {
        CUDA_TRY(cudaDeviceSynchronize());
        const int n = std::min(max_entries, eng->timeline_ctas * kStamps);
        CUDA_TRY(cudaMemcpy(out, eng->timeline, (size_t)n * 8, cudaMemcpyDeviceToHost));
    }
    return MOE_OK;
}

// ============================================================ no-allocation forward
// Some callers cannot call cudaMalloc at the moment they run the layer: serving
// runtimes that reserve all device memory up front and forbid allocations
// afterwards, or latency-critical paths where an allocation (which may
// synchronise the device) is not acceptable.  moe_engine_forward_noalloc runs the
// fused decode kernel with the grid barrier between gate_up and down (the one
// moe_engine_forward uses for AWQ) but takes its scratch (the h workspace, the
// grid-barrier counter) from the fixed device array below instead of the engine's workspace, so it
// allocates nothing.  The array lives in every GPU that loads this library until
// the process exits.
constexpr size_t kNoAllocScratchBytes = 512 * 1024;
constexpr size_t kNoAllocHeader = 256;  // grid-barrier counter at 0; h from byte 256
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[128] = {};

// Device address of g_noalloc_scratch on `dev` (current).  In host code the array's
// name only stands in for the symbol, so its address must be asked for once per device.
int noalloc_scratch(int dev, unsigned char** out) {
    if (dev < 0 || dev >= 128) return fail(MOE_ERR_INVALID, "device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return fail(MOE_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        g_noalloc_ptr[dev] = p;
    }
    *out = static_cast<unsigned char*>(g_noalloc_ptr[dev]);
    return MOE_OK;
}
}  // namespace

extern "C" int moe_engine_forward_noalloc(moe_engine* eng, const void* x, void* y, const int32_t* topk_ids,
                                          const float* topk_w, int64_t T, int64_t K, int32_t act_dtype,
                                          int32_t out_dtype, void* stream) {
    if (int rc = check_engine(eng)) return rc;
    if (!eng->loaded) return fail(MOE_ERR_STATE, "no weights loaded");
    if (T < 0 || K <= 0 || K > 64) return fail(MOE_ERR_INVALID, "num_tokens must be >= 0 and 1 <= top_k <= 64");
    if (act_dtype != MOE_F16 && act_dtype != MOE_BF16) return fail(MOE_ERR_INVALID, "hidden must be f16 or bf16");
    if (out_dtype != MOE_F16 && out_dtype != MOE_BF16 && out_dtype != MOE_F32)
        return fail(MOE_ERR_INVALID, "bad output dtype");
    if (T > 0 && (!x || !y || !topk_ids || !topk_w)) return fail(MOE_ERR_INVALID, "null tensor pointer");
    if (eng->p2p_active) return fail(MOE_ERR_STATE, "the no-allocation forward does not run the peer combine");
    const int64_t I = eng->cfg.intermediate_size;
    const int64_t P = T * K;
    const size_t need = kNoAllocHeader + (size_t)P * I * 4;  // h is requantised in place
    if (need > kNoAllocScratchBytes)
        return fail(MOE_ERR_INVALID, "num_tokens x top_k x intermediate_size needs " + std::to_string(need) +
                                         " bytes of scratch; moe_engine_forward_noalloc holds at most " +
                                         std::to_string(kNoAllocScratchBytes));
    DeviceGuard g(eng->cfg.device);
    if (T == 0) return MOE_OK;
    DecodePlan pl;  // the barrier-in-the-middle kernel: its scratch does not grow with the grid
    if (!plan_decode(eng, (int)T, (int)K, pl))
        return fail(MOE_ERR_INVALID, "num_tokens x top_k too large for one decode launch; use moe_engine_forward");
    unsigned char* base = nullptr;
    if (int rc = noalloc_scratch(eng->cfg.device, &base)) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (int rc = check_sticky_error(eng, st)) return rc;
    // every call reuses the array: clear the barrier counter (it must start at zero), leave
    // h to be overwritten
    CUDA_TRY(cudaMemsetAsync(base, 0, kNoAllocHeader, st));
    DecodeParams& p = pl.p;
    p.act_bf16 = act_dtype == MOE_BF16;
    p.out_kind = out_dtype == MOE_F32 ? 2 : (out_dtype == MOE_BF16 ? 1 : 0);
    p.x = x;
    p.y = y;
    p.ids = topk_ids;
    p.tw = topk_w;
    p.gu = eng->gu;
    p.dn = eng->dn;
    p.bar = reinterpret_cast<unsigned long long*>(base);
    p.err = eng->err;  // the engine's mapped error word: reported like moe_engine_forward's
    p.h_ws = reinterpret_cast<float*>(base + kNoAllocHeader);
    p.dbg = nullptr;
    const int qt = eng->cfg.quant_type;
    return qt == MOE_Q4_0 ? launch_decode<kQ4>(pl, st)
                          : (qt == MOE_AWQ ? launch_decode<kAWQ>(pl, st) : launch_decode<kQ8>(pl, st));
}

// =================================================================== peer combine (expert parallel)
extern "C" int moe_engine_p2p_covers(moe_engine* eng, int64_t num_tokens) {
    if (!eng) return 0;
    return !(num_tokens > eng->gemm_min_tokens && gemm_path_ok(eng)) &&
           !(num_tokens > eng->awq_gemm_min_tokens && awq_gemm_ok(eng)) && num_tokens <= std::max<int64_t>(eng->p2p_tcap, 8);
}

extern "C" int moe_engine_p2p_mailbox(moe_engine* eng, int32_t world, int64_t max_tokens, void* ipc_handle_out) {
    if (int rc = check_engine(eng)) return rc;
    if (world < 2 || world > kMaxPeers || max_tokens <= 0 || !ipc_handle_out)
        return fail(MOE_ERR_INVALID, "peer combine needs 2..8 ranks, max_tokens > 0 and a handle buffer");
    if (eng->mbox) return fail(MOE_ERR_STATE, "mailbox already created");
    DeviceGuard g(eng->cfg.device);
    const int64_t tcap = std::min<int64_t>(max_tokens, 64);
    const size_t data = (size_t)2 * world * tcap * eng->cfg.hidden_size * sizeof(float);
    const size_t flags = (size_t)world * eng->num_sms * sizeof(unsigned long long);
    CUDA_TRY(cudaMalloc(&eng->mbox, data + flags));
    CUDA_TRY(cudaMemset(eng->mbox, 0, data + flags));
    eng->mbox_data_bytes = (int64_t)data;
    eng->p2p_tcap = (int)tcap;
    cudaIpcMemHandle_t h;
    CUDA_TRY(cudaIpcGetMemHandle(&h, eng->mbox));
    std::memcpy(ipc_handle_out, &h, sizeof(h));
    return MOE_OK;
}

extern "C" int moe_engine_p2p_connect(moe_engine* eng, int32_t rank, int32_t world, const void* ipc_handles) {
    if (int rc = check_engine(eng)) return rc;
    if (!eng->mbox) return fail(MOE_ERR_STATE, "create the mailbox first (moe_engine_p2p_mailbox)");
    if (world < 2 || world > kMaxPeers || rank < 0 || rank >= world || !ipc_handles)
        return fail(MOE_ERR_INVALID, "bad rank / world / handles");
    if (eng->mbox_data_bytes != (int64_t)2 * world * eng->p2p_tcap * eng->cfg.hidden_size * (int64_t)sizeof(float))
        return fail(MOE_ERR_INVALID, "world differs from the mailbox's");
    DeviceGuard g(eng->cfg.device);
    const auto* hs = static_cast<const cudaIpcMemHandle_t*>(ipc_handles);
    for (int q = 0; q < world; ++q) {
        if (q == rank) continue;
        void* ptr = nullptr;
        CUDA_TRY(cudaIpcOpenMemHandle(&ptr, hs[q], cudaIpcMemLazyEnablePeerAccess));
        eng->peer_base[q] = ptr;
    }
    eng->p2p_rank = rank;
    eng->p2p_world = world;
    eng->p2p_active = true;
    return MOE_OK;
}

extern "C" int moe_engine_p2p_enable(moe_engine* eng, int32_t on) {
    if (int rc = check_engine(eng)) return rc;
    if (on && eng->p2p_world < 2) return fail(MOE_ERR_STATE, "not connected (moe_engine_p2p_connect)");
    eng->p2p_active = on != 0;
    return MOE_OK;
}

// =================================================================== packed-layout files
// A file of an engine's device-resident layouts, so that a later process loads them with
// plain copies instead of repacking from the quantised tensors.  Little-endian:
//   "MOEB200\0" | u32 version | u32 section count | config (E, H, I as i64; quant type,
//   group size, scale dtype, rs1, ss1, rs2, ss2 as i32) | per section: u32 id, u32 0,
//   u64 bytes, u64 file offset, u64 FNV-1a checksum | data (4 KiB-aligned sections).
namespace {
constexpr char kFileMagic[8] = {'M', 'O', 'E', 'B', '2', '0', '0', '\0'};
constexpr uint32_t kFileVersion = 1;
struct FileConfig {
    int64_t E, H, I;
    int32_t quant_type, group_size, scale_bf16, rs1, ss1, rs2, ss2, pad;
};
struct FileSection {
    uint32_t id, zero;
    uint64_t bytes, offset, checksum;
};

uint64_t fnv1a(const uint8_t* p, size_t n, uint64_t h = 1469598103934665603ull) {
    for (size_t i = 0; i < n; ++i) h = (h ^ p[i]) * 1099511628211ull;
    return h;
}

// The engine's device buffers that a file holds: (id, pointer, bytes).
struct Buf {
    uint32_t id;
    uint8_t** ptr;
    size_t bytes;
};
std::vector<Buf> engine_buffers(moe_engine* eng) {
    const int64_t E = eng->cfg.num_experts, H = eng->cfg.hidden_size, I = eng->cfg.intermediate_size;
    std::vector<Buf> v;
    v.push_back({1, &eng->gu, (size_t)E * I * eng->unit_bytes()});
    v.push_back({2, &eng->dn, (size_t)E * H * eng->row_bytes()});
    if (eng->dk) v.push_back({3, &eng->dk, (size_t)E * (I / 32) * (H / 32) * sk_slice_bytes(eng)});
    if (eng->cfg.quant_type == MOE_AWQ) {
        if (eng->agu) v.push_back({4, &eng->agu, (size_t)E * (I / 16) * 2 * (H / kAwqK) * kAwqGuRec});
        if (eng->adn) v.push_back({5, &eng->adn, (size_t)E * (H / 32) * (I / kAwqK) * kAwqDnRec});
    } else if (eng->adn) {
        const int BB = eng->cfg.quant_type == MOE_Q4_0 ? 16 : 32;
        v.push_back({5, &eng->adn, (size_t)E * (H / 32) * (I / 32) * (32 * BB + 64)});
    }
    return v;
}
}  // namespace

extern "C" int moe_engine_save(moe_engine* eng, const char* path) {
    if (int rc = check_engine(eng)) return rc;
    if (!path) return fail(MOE_ERR_INVALID, "null path");
    if (!eng->loaded) return fail(MOE_ERR_STATE, "no weights loaded");
    DeviceGuard g(eng->cfg.device);
    CUDA_TRY(cudaDeviceSynchronize());
    std::vector<Buf> bufs = engine_buffers(eng);
    FileConfig fc{eng->cfg.num_experts, eng->cfg.hidden_size, eng->cfg.intermediate_size, eng->cfg.quant_type,
                  eng->cfg.group_size, eng->scale_bf16, eng->rs1, eng->ss1, eng->rs2, eng->ss2, 0};
    std::vector<FileSection> secs(bufs.size());
    uint64_t off = round_up(sizeof(kFileMagic) + 8 + sizeof(FileConfig) + bufs.size() * sizeof(FileSection), 4096);
    std::vector<std::vector<uint8_t>> host(bufs.size());
    for (size_t i = 0; i < bufs.size(); ++i) {
        host[i].resize(bufs[i].bytes);
        CUDA_TRY(cudaMemcpy(host[i].data(), *bufs[i].ptr, bufs[i].bytes, cudaMemcpyDeviceToHost));
        secs[i] = {bufs[i].id, 0, bufs[i].bytes, off, fnv1a(host[i].data(), bufs[i].bytes)};
        off = round_up(off + bufs[i].bytes, 4096);
    }
    FILE* f = std::fopen(path, "wb");
    if (!f) return fail(MOE_ERR_INVALID, std::string("cannot open ") + path + " for writing");
    const uint32_t hdr[2] = {kFileVersion, (uint32_t)bufs.size()};
    bool ok = std::fwrite(kFileMagic, 1, 8, f) == 8 && std::fwrite(hdr, 4, 2, f) == 2 &&
              std::fwrite(&fc, sizeof(fc), 1, f) == 1 &&
              std::fwrite(secs.data(), sizeof(FileSection), secs.size(), f) == secs.size();
    for (size_t i = 0; ok && i < bufs.size(); ++i)
        ok = std::fseek(f, (long)secs[i].offset, SEEK_SET) == 0 &&
             std::fwrite(host[i].data(), 1, host[i].size(), f) == host[i].size();
    ok = (std::fclose(f) == 0) && ok;
    if (!ok) return fail(MOE_ERR_INVALID, std::string("write to ") + path + " failed");
    return MOE_OK;
}

extern "C" int moe_engine_load_file(moe_engine* eng, const char* path) {
    if (int rc = check_engine(eng)) return rc;
    if (!path) return fail(MOE_ERR_INVALID, "null path");
    FILE* f = std::fopen(path, "rb");
    if (!f) return fail(MOE_ERR_INVALID, std::string("cannot open ") + path);
    struct Closer {
        FILE* f;
        ~Closer() { std::fclose(f); }
    } closer{f};
    char magic[8];
    uint32_t hdr[2];
    FileConfig fc;
    if (std::fread(magic, 1, 8, f) != 8 || std::memcmp(magic, kFileMagic, 8) != 0)
        return fail(MOE_ERR_INVALID, "not a packed-layout file (bad magic)");
    if (std::fread(hdr, 4, 2, f) != 2 || hdr[0] != kFileVersion || hdr[1] == 0 || hdr[1] > 16)
        return fail(MOE_ERR_INVALID, "unsupported packed-layout file version or section count");
    if (std::fread(&fc, sizeof(fc), 1, f) != 1) return fail(MOE_ERR_INVALID, "truncated header");
    if (fc.E != eng->cfg.num_experts || fc.H != eng->cfg.hidden_size || fc.I != eng->cfg.intermediate_size ||
        fc.quant_type != eng->cfg.quant_type || (fc.quant_type == MOE_AWQ && fc.group_size != eng->cfg.group_size))
        return fail(MOE_ERR_INVALID, "the file's shape or quantisation differs from the engine's");
    std::vector<FileSection> secs(hdr[1]);
    if (std::fread(secs.data(), sizeof(FileSection), secs.size(), f) != secs.size())
        return fail(MOE_ERR_INVALID, "truncated section table");
    DeviceGuard g(eng->cfg.device);
    if (int rc = alloc_q_layout(eng)) return rc;  // the row layouts (and the split-K chunks)
    if (fc.rs1 != eng->rs1 || fc.ss1 != eng->ss1 || fc.rs2 != eng->rs2 || fc.ss2 != eng->ss2)
        return fail(MOE_ERR_INVALID, "the file's record layout differs from this build's");
    const int64_t E = eng->cfg.num_experts, H = eng->cfg.hidden_size, I = eng->cfg.intermediate_size;
    // the cluster kernel's layouts are allocated on demand, as build_cl_layout does
    for (const FileSection& sc : secs) {
        if (sc.id == 4 && !eng->agu) CUDA_TRY(cudaMalloc(&eng->agu, sc.bytes));
        if (sc.id == 5 && !eng->adn) CUDA_TRY(cudaMalloc(&eng->adn, sc.bytes));
    }
    (void)E; (void)H; (void)I;
    std::vector<Buf> bufs = engine_buffers(eng);
    std::vector<uint8_t> host;
    for (const FileSection& sc : secs) {
        const Buf* b = nullptr;
        for (const Buf& x : bufs)
            if (x.id == sc.id) b = &x;
        if (!b || b->bytes != sc.bytes) return fail(MOE_ERR_INVALID, "section " + std::to_string(sc.id) + " does not fit the engine");
        host.resize(sc.bytes);
        if (std::fseek(f, (long)sc.offset, SEEK_SET) != 0 || std::fread(host.data(), 1, sc.bytes, f) != sc.bytes)
            return fail(MOE_ERR_INVALID, "truncated section " + std::to_string(sc.id));
        if (fnv1a(host.data(), sc.bytes) != sc.checksum)
            return fail(MOE_ERR_INVALID, "checksum mismatch in section " + std::to_string(sc.id));
        CUDA_TRY(cudaMemcpy(*b->ptr, host.data(), sc.bytes, cudaMemcpyHostToDevice));
    }
    eng->scale_bf16 = fc.scale_bf16;
    eng->loaded = true;
    return MOE_OK;
}

// =================================================================== expert placement
extern "C" int moe_engine_set_expert_map(moe_engine* eng, const int32_t* local_of_global, int64_t num_global) {
    if (int rc = check_engine(eng)) return rc;
    if (!local_of_global || num_global <= 0 || num_global > (1 << 20)) return fail(MOE_ERR_INVALID, "bad expert map");
    const int64_t E = eng->cfg.num_experts;
    std::vector<int> seen(E, 0);
    for (int64_t g = 0; g < num_global; ++g) {
        const int32_t v = local_of_global[g];
        if (v == -1) continue;
        const int32_t l = v & ~kReplicaFlag;
        if (v < 0 || l >= E || seen[l]++) return fail(MOE_ERR_INVALID, "expert map must send each local expert id once");
    }
    eng->emap_host.assign(local_of_global, local_of_global + num_global);
    return upload_expert_map(eng);
}

extern "C" int moe_engine_set_replica_split(moe_engine* eng, int32_t rank, int32_t world) {
    if (int rc = check_engine(eng)) return rc;
    if (world < 1 || rank < 0 || rank >= world) return fail(MOE_ERR_INVALID, "bad replica split rank / world");
    eng->rep_rank = rank;
    eng->rep_world = world;
    if (eng->emap_host.empty()) return MOE_OK;  // applied when the map is set
    return upload_expert_map(eng);
}
