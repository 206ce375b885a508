// AWQ W4A16 path (placeholder until the tensor-core GEMV lands).
#include "awq.cuh"

namespace moe {
int awq_alloc(AwqWeights& w, int64_t E, int64_t H, int64_t I, int64_t G) {
    w.E = E; w.H = H; w.I = I; w.G = G;
    return 0;
}
void awq_free(AwqWeights& w) { cudaFree(w.buf); w.buf = nullptr; }
int awq_pack(AwqWeights&, const uint8_t* const*, cudaStream_t) { return -1; }
int awq_forward(const AwqWeights&, int, int, int, const void*, void*, const int32_t*, const float*, int, int, int,
                int, float*, uint32_t*, int32_t*, cudaStream_t) {
    return -1;
}
}  // namespace moe
