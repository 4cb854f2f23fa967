// kvstore.cu -- fp32 k/v rows into the fp16 KV cache with the engine's rounding.
//
// Reference: engine.c:1068-1072 (CPU store through f32_to_f16, platform.c:340-379)
// and cuda_kernels.cu:494-528 (GPU store through __float2half_rn).  The two
// disagree on ties and on f32 subnormals; this store follows the engine so the
// device cache holds the same bytes as the CPU engine's cache.
#include "common.cuh"

#include <algorithm>

namespace yattn {
namespace {

// Grid-stride over the B*kv_dim values; input row r lands at cache row pos_start + r.
__global__ void k_store_kv(uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, const float* __restrict__ k,
                           const float* __restrict__ v, uint32_t pos_start, uint32_t B, uint32_t kv_dim) {
    const size_t n = static_cast<size_t>(B) * kv_dim;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t row = i / kv_dim, col = i % kv_dim;
        const size_t dst = (static_cast<size_t>(pos_start) + row) * kv_dim + col;
        kc[dst] = engine_f32_to_f16(k[i]);
        vc[dst] = engine_f32_to_f16(v[i]);
    }
}

int store_kv(uint16_t* kc, uint16_t* vc, const float* k, const float* v, uint32_t pos_start, uint32_t B,
             uint32_t kv_dim, cudaStream_t st, char* err, size_t errlen) {
    if (!kc || !vc || !k || !v || kv_dim == 0) {
        set_err(err, errlen, "store_kv: bad arguments");
        return -1;
    }
    if (B == 0) return 0;
    const size_t n = static_cast<size_t>(B) * kv_dim;
    const uint32_t blocks = static_cast<uint32_t>(std::min<size_t>((n + 255) / 256, 148u * 16u));
    k_store_kv<<<blocks, 256, 0, st>>>(kc, vc, k, v, pos_start, B, kv_dim);
    YATTN_CHECK_LAUNCH(err, errlen, "store_kv");
    return 0;
}

}  // namespace
}  // namespace yattn

using namespace yattn;

extern "C" int yattn_store_kv(uint16_t* kcache, uint16_t* vcache, const float* k, const float* v,
                              uint32_t pos_start, uint32_t B, uint32_t kv_dim, void* stream, char* err,
                              size_t errlen) {
    return store_kv(kcache, vcache, k, v, pos_start, B, kv_dim, static_cast<cudaStream_t>(stream), err, errlen);
}

extern "C" void cuda_k_store_kv(uint16_t* kcache, uint16_t* vcache, const float* k, const float* v, uint32_t pos,
                                uint32_t kv_dim) {
    char err[256];
    err[0] = 0;
    if (store_kv(kcache, vcache, k, v, pos, 1, kv_dim, nullptr, err, sizeof(err)) != 0) set_last_error(err);
}

extern "C" void cuda_k_store_kv_batch(uint16_t* kcache, uint16_t* vcache, const float* k, const float* v,
                                      uint32_t pos_start, uint32_t B, uint32_t kv_dim) {
    char err[256];
    err[0] = 0;
    if (store_kv(kcache, vcache, k, v, pos_start, B, kv_dim, nullptr, err, sizeof(err)) != 0) set_last_error(err);
}
