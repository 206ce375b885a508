// AWQ W4A16 path: device layout, load-time packing and forward.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace moe {

struct AwqWeights {
    int64_t E = 0, H = 0, I = 0, G = 0;
    uint8_t* buf = nullptr;
};

int awq_alloc(AwqWeights& w, int64_t E, int64_t H, int64_t I, int64_t G);
void awq_free(AwqWeights& w);
int awq_pack(AwqWeights& w, const uint8_t* const src[6], cudaStream_t st);
int awq_forward(const AwqWeights& w, int num_sms, int max_smem, int e_off, const void* x, void* y,
                const int32_t* ids, const float* tw, int T, int K, int act_bf16, int out_dtype, float* h_ws,
                uint32_t* bar, int32_t* err, cudaStream_t st);

}  // namespace moe
