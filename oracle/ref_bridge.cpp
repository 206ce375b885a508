// TEST INFRASTRUCTURE ONLY -- never linked into the product library.
//
// extern "C" entry points into the reference CPU engine's own objects
// (compiled unmodified from Int8-gemm/{q8_gemm,moe_infer,moe_common,gemm_kernels}.cpp
// by oracle/Makefile), so that the parity tests can call the reference's
// internal routines and its engine from ctypes in the same process as the
// product library, without registering the reference's `nanovllm` torch
// namespace (Int8-gemm/nanovllm_ops.cpp is left out of this bridge).
//
//   ref_route_preprocess  -> moe::preprocess_moe_routing     (moe_common.cpp:186-216)
//   ref_quantize_block    -> gemm::quantize_block_q8_0<float> (gemm_kernels.cpp:25-58)
//   ref_quantize_weight   -> quantize_weight_only             (q8_gemm.cpp:219-260)
//   ref_engine_*          -> MoEInfer                         (moe_infer.cpp:18-456)
#include <torch/torch.h>
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "moe_common.h"
#include "moe_infer.h"
#include "q8_gemm.h"

static thread_local std::string g_err;
extern "C" void ref_pool_warmup(void);

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

int ref_route_preprocess(int E, int K, int T, const int32_t* ids, int32_t* counts,
                         int32_t* starts, int32_t* token_map, int32_t* scatter_map) {
    try {
        std::vector<int> c, s;
        std::vector<moe::MoETokenInfo> tm;
        std::vector<int32_t> sm;
        moe::preprocess_moe_routing(E, K, T, ids, c, s, tm, sm);
        for (int e = 0; e < E; ++e) counts[e] = c[e];
        for (int e = 0; e <= E; ++e) starts[e] = s[e];
        for (size_t p = 0; p < tm.size(); ++p) {
            token_map[2 * p] = tm[p].token_id;
            token_map[2 * p + 1] = tm[p].expert_idx_in_tok;
        }
        for (int i = 0; i < T * K; ++i) scatter_map[i] = sm[i];
        return (int)tm.size();
    } catch (const std::exception& ex) {
        g_err = ex.what();
        return -1;
    }
}

// One Q8_0 block with an fp32 scale (the activation path).
float ref_quantize_block(const float* x, int8_t* qs) {
    float d = 0.0f;
    gemm::quantize_block_q8_0<float>(x, &d, qs);
    return d;
}

// Weight quantiser: fp32 [N,K] -> int8 [N,K] + fp16 bits [N,K/32].
int ref_quantize_weight(const float* w, int64_t N, int64_t K, int8_t* qs, uint16_t* d) {
    try {
        auto t = torch::from_blob(const_cast<float*>(w), {N, K}, torch::kFloat32);
        auto q = quantize_weight_only(t);
        std::memcpy(qs, q[0].data_ptr(), (size_t)N * K);
        std::memcpy(d, q[1].data_ptr(), (size_t)N * (K / 32) * 2);
        return 0;
    } catch (const std::exception& ex) {
        g_err = ex.what();
        return -1;
    }
}

void* ref_engine_create(int64_t E, int64_t H, int64_t I, int quant_type) {
    try {
        ref_pool_warmup();
        return new MoEInfer(E, H, I, static_cast<quant::QuantType>(quant_type));
    } catch (const std::exception& ex) {
        g_err = ex.what();
        return nullptr;
    }
}

void ref_engine_destroy(void* h) { delete static_cast<MoEInfer*>(h); }

// Pre-quantised weights in the row-major input contract; scale_is_bf16 picks
// the scale dtype; qs are int8 (Q8_0) or packed uint32 words (Q4_0).
int ref_engine_store_repack(void* h, int quant_type, int scale_is_bf16,
                            const void* gu_qs, const uint16_t* gu_d,
                            const void* dn_qs, const uint16_t* dn_d) {
    try {
        auto* m = static_cast<MoEInfer*>(h);
        const int64_t E = m->num_experts(), H = m->hidden_size(), I = m->intermediate_size();
        auto sdt = scale_is_bf16 ? torch::kBFloat16 : torch::kFloat16;
        torch::Tensor gq, dq;
        if (quant_type == 0) {
            gq = torch::from_blob(const_cast<void*>(gu_qs), {E, 2 * I, H}, torch::kInt8);
            dq = torch::from_blob(const_cast<void*>(dn_qs), {E, H, I}, torch::kInt8);
        } else {
            gq = torch::from_blob(const_cast<void*>(gu_qs), {E, 2 * I, H / 8}, torch::kInt32);
            dq = torch::from_blob(const_cast<void*>(dn_qs), {E, H, I / 8}, torch::kInt32);
        }
        auto gd = torch::from_blob(const_cast<uint16_t*>(gu_d), {E, 2 * I, H / 32}, sdt);
        auto dd = torch::from_blob(const_cast<uint16_t*>(dn_d), {E, H, I / 32}, sdt);
        m->store_quantized_weights_repack(gq, gd, dq, dd);
        return 0;
    } catch (const std::exception& ex) {
        g_err = ex.what();
        return -1;
    }
}

int ref_engine_quantize_store(void* h, int64_t e, const char* proj, const float* w, int64_t rows,
                              int64_t cols) {
    try {
        auto t = torch::from_blob(const_cast<float*>(w), {rows, cols}, torch::kFloat32);
        static_cast<MoEInfer*>(h)->quantize_and_store_expert(e, proj, t);
        return 0;
    } catch (const std::exception& ex) {
        g_err = ex.what();
        return -1;
    }
}

// act_is_bf16: hidden / output dtype (bf16 when 1, fp16 when 0).
int ref_engine_forward(void* h, const void* x, void* y, const int32_t* ids, const float* w,
                       int64_t T, int64_t K, int act_is_bf16) {
    try {
        static_cast<MoEInfer*>(h)->execute_on_cpu_routed_from_pointers(
            x, y, ids, w, T, K, act_is_bf16 ? at::kBFloat16 : at::kHalf);
        return 0;
    } catch (const std::exception& ex) {
        g_err = ex.what();
        return -1;
    }
}

double ref_engine_last_ms(void* h) { return static_cast<MoEInfer*>(h)->get_last_run_time_ms(); }

}  // extern "C"
