// Shared device helpers: element conversions, the SiLU of the reference,
// mbarrier / bulk-copy PTX wrappers and bounded waits.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define MOE_DEV __device__ __forceinline__

namespace moe {

// Iteration budget of every spin-wait (mbarrier, grid barrier).  With the
// nanosleep back-off this is on the order of a second; an expired wait sets
// the workspace error word and the kernel leaves without hanging the GPU.
constexpr uint32_t kSpinLimit = 1u << 22;

enum ErrCode : int32_t { kErrNone = 0, kErrGridBarrier = 1, kErrFullWait = 2, kErrEmptyWait = 3, kErrPeerWait = 4,
                         kErrRange = 5 };

// Record a device error.  `err` is the engine's error word in mapped pinned host memory
// (cudaHostAllocMapped), so the host reads it at the entry of the next call without a
// device synchronisation: a plain system-scope store, made visible before the kernel
// goes on.  The code is sticky until the host clears it.
MOE_DEV void set_err(int32_t* err, int32_t code) {
    if (!err) return;
    *reinterpret_cast<volatile int32_t*>(err) = code;
    __threadfence_system();
}

// Global expert id -> this engine's local id, or -1 for experts it does not hold: through
// the placement map when one is set (local_of_global[gid]), else the contiguous block
// [e_off, e_off + E).  Invalid ids are skipped like in the reference (moe_common.cpp:158).
// A map entry with kReplicaFlag marks a hot expert replicated on every rank: this engine
// takes the pair only when (token + gid) % world == rank, with world and rank stored after
// the map's emap_n entries, so that every pair is computed by exactly one rank.
constexpr int32_t kReplicaFlag = 1 << 30;
MOE_DEV int local_expert(int gid, int e_off, int E, const int32_t* emap, int emap_n, int pair, int K) {
    if (emap) {
        if (gid < 0 || gid >= emap_n) return -1;
        const int v = emap[gid];
        if (v >= 0 && (v & kReplicaFlag)) {
            const int world = emap[emap_n], rank = emap[emap_n + 1];
            return ((pair / K + gid) % world == rank) ? (v & ~kReplicaFlag) : -1;
        }
        return v;
    }
    const int g = gid - e_off;
    return (g >= 0 && g < E) ? g : -1;
}

MOE_DEV float act_to_f32(const void* p, int64_t i, int is_bf16) {
    if (is_bf16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

MOE_DEV float scale_to_f32(uint16_t bits, int is_bf16) {
    if (is_bf16) return __uint_as_float(static_cast<uint32_t>(bits) << 16);
    return __half2float(__ushort_as_half(bits));
}

// exp(x) as the reference's vectorised SiLU computes it: the range-reduced
// polynomial of Int8-gemm/vec_simd.h:9-33, per lane with fused multiply-adds,
// so that the intermediate activations track the reference bit for bit.
MOE_DEV float ref_expf(float x) {
    const float r = 0x1.8p23f;
    const float z = __fmaf_rn(x, 0x1.715476p+0f, r);
    const float n = z - r;
    const float b = __fmaf_rn(-n, 0x1.7f7d1cp-20f, __fmaf_rn(-n, 0x1.62e4p-1f, x));
    const uint32_t e = __float_as_uint(z) << 23;
    const float k = __uint_as_float(e + 0x3f800000u);
    const float u = __fmul_rn(b, b);
    const float j = __fmaf_rn(__fmaf_rn(__fmaf_rn(0x1.0e4020p-7f, b, 0x1.573e2ep-5f), u,
                                        __fmaf_rn(0x1.555e66p-3f, b, 0x1.fffdb6p-2f)),
                              u, __fmul_rn(0x1.ffffecp-1f, b));
    if (!(fabsf(n) > 126.0f)) return __fmaf_rn(k, j, k);
    const uint32_t d = (n <= 0.0f) ? 0x82000000u : 0u;
    const float s1 = __uint_as_float(d + 0x7f000000u);
    const float s2 = __uint_as_float(e - d);
    if (fabsf(n) > 192.0f) return __fmul_rn(s1, s1);
    return __fmul_rn(__fmaf_rn(s2, j, s2), s1);
}

// SiLU(gate) * up with IEEE division, as Int8-gemm/vec_simd.h:36-64.
MOE_DEV float silu_mul(float g, float up) {
    const float act = __fdiv_rn(g, __fadd_rn(1.0f, ref_expf(-g)));
    return __fmul_rn(up, act);
}

// One Q8_0 block scale as the reference binary computes it: d = amax * (1/127)
// (Int8-gemm/gemm_kernels.cpp:43 under -ffast-math), id = d ? 1/d : 0.
MOE_DEV float q8_scale(float amax) { return __fmul_rn(amax, 1.0f / 127.0f); }
// __frcp_rn is the correctly rounded reciprocal, i.e. the IEEE quotient 1/d.
MOE_DEV float q8_inv(float d) { return d != 0.0f ? __frcp_rn(d) : 0.0f; }
MOE_DEV int q8_quant(float v, float id) {
    int q = __float2int_rn(__fmul_rn(v, id));  // round to nearest even
    return q > 127 ? 127 : (q < -128 ? -128 : q);
}

// ------------------------------------------------------------------ PTX
MOE_DEV uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

MOE_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

MOE_DEV void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

MOE_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

MOE_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

MOE_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on a phase of an mbarrier; false when the budget ran out.  try_wait itself
// suspends the thread for a while; a back-off sleep only starts after many polls, since a
// sleeping warp wakes up late and the weight copies it waits for are on the critical path.
MOE_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
    for (uint32_t it = 0; it < kSpinLimit; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if (it > 8192) __nanosleep(128);
    }
    return false;
}

// 1-D bulk copy global -> shared, completion counted on `bar` (plain, one destination CTA).
// dst, src and bytes must be multiples of 16.
MOE_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same copy with an L2 cache-policy operand (e.g. evict-first for data read once).
MOE_DEV void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// L2 policy: lines filled by the accesses that carry it are the first to be evicted.
MOE_DEV uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

MOE_DEV void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

MOE_DEV uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

MOE_DEV unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

MOE_DEV unsigned long long atom_add_release_gpu_u64(unsigned long long* p, unsigned long long v) {
    unsigned long long old;
    asm volatile("atom.add.release.gpu.global.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
    return old;
}

// Grid barrier over `nblocks` co-resident CTAs (cooperative launch), one thread
// per CTA.  `ctr` counts arrivals monotonically over all launches; launch n
// (0-based, read by barrier_launch_index at its start) is released once the
// counter reaches (n+1)*nblocks.  The arrival is a gpu-scope fence (orders this
// CTA's earlier global writes before it) and a fire-and-forget reduction, then acquire
// polling.  Returns false (and sets *err) when the wait budget ran out.
MOE_DEV bool grid_barrier(unsigned long long* ctr, uint32_t nblocks, unsigned long long target, int32_t* err,
                          unsigned long long* stamps = nullptr) {
    (void)nblocks;
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    if (stamps) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(stamps[0]));
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(ctr), "l"(1ull) : "memory");
    for (uint32_t it = 0; it < kSpinLimit; ++it) {
        if (ld_acquire_gpu_u64(ctr) >= target) {
            if (stamps) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(stamps[1]));
            return true;
        }
        if (it > 4096) __nanosleep(256);  // hot spin first: the barrier is on the critical path
    }
    set_err(err, kErrGridBarrier);
    return false;
}

// Index of the current launch on this barrier counter (valid before this CTA arrives).
MOE_DEV unsigned long long barrier_launch_index(const unsigned long long* ctr, uint32_t nblocks) {
    return ld_acquire_gpu_u64(ctr) / nblocks;
}

}  // namespace moe
