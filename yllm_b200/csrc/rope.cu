// rope.cu -- one decode step's RoPE and KV store, fused, for many sequences.
//
// Reference: per sequence, engine.c:1052-1072 on the CPU (rope_inplace /
// rope_inplace_qwen on every q and k head, matvec.c:890-921, then the fp32 ->
// fp16 store of k and v through f32_to_f16, platform.c:340-379) and
// cuda_fwd.c:136-147 on the GPU (cuda_k_rope_{llama,qwen}_heads on q, on k,
// then cuda_k_store_kv: three launches per sequence and layer).  qwen35's
// M-RoPE (rope_inplace_mrope, matvec.c:924-939: the first n_dims dims only) is
// the third kind.
//
// One launch covers every item (sequence) of a layer: q is rotated in place
// (the attention reads it next), k is rotated on the way into the cache, v is
// stored as is.  The arithmetic follows the reference's fp32 operation order:
// the inverse frequencies are computed on the host with the same powf
// expression (so they are the reference's own values), the angle is one fp32
// multiply, and a*c - b*s / a*s + b*c are evaluated without FMA contraction.
// The only difference left is the device's sinf/cosf against the host
// library's (a few ulps), which moves a stored fp16 value by one ulp rarely.
//
// With QK-norm (qwen3, engine.c:1036-1045; qwen35, engine.c:915-919) every q
// head and every k head is first normalised by rmsnorm (matvec.c:152-165) with
// the layer's shared head_dim weights, then rotated.  That launch runs one CTA
// per head: the sum of squares goes in index order through one thread, as the
// reference's loop does, and y = (x * w) * inv keeps its operation order.
#include "common.cuh"

#include <algorithm>
#include <cmath>

namespace yattn {
namespace {

constexpr int kMaxPairs = 128;   // head_dim <= 256

struct RopeParams {
    const YattnRopeItem* items;      // NULL: the batch form below
    const void* q_norm_w;            // QK-norm weights [hd] (fp32, or fp16 bits if norm_f16); NULL: no norm
    const void* k_norm_w;
    uint32_t norm_f16;
    float norm_eps;
    YattnRopeItem batch;             // row 0 of a token batch: row b at q + b*q_stride, k/v + b*kv_dim, pos + b
    uint32_t q_stride;
    uint32_t n_items, n_heads, n_kv, hd, kv_dim;
    uint32_t kind;                   // 0 llama (2j, 2j+1), 1 qwen (j, j + hd/2), 2 mrope (j, j + n_dims/2), j < n_dims/2
    uint32_t n_dims;                 // rotated dims (hd for kinds 0 and 1)
    float inv_freq[kMaxPairs];       // theta^(-2j/n_dims), the reference's powf values
};

// Row `blockIdx.y` of the launch: the item, or row b of the batch form.
__device__ __forceinline__ YattnRopeItem item_of(const RopeParams& p) {
    YattnRopeItem it;
    if (p.items) {
        it = p.items[blockIdx.y];
    } else {
        it = p.batch;
        it.q += static_cast<size_t>(blockIdx.y) * p.q_stride;
        it.k += static_cast<size_t>(blockIdx.y) * p.kv_dim;
        it.v += static_cast<size_t>(blockIdx.y) * p.kv_dim;
        it.pos += blockIdx.y;
    }
    return it;
}

// blockIdx.y = item.  Work of an item, grid-strided over blockIdx.x:
//   [0, nq)            q pairs (head, j), rotated in place
//   [nq, nq + nk)      k pairs, rotated and stored (engine rounding)
//   [.., + nr)         k elements outside the rotated dims (mrope), stored as is
//   [.., + kv_dim)     v elements, stored
__global__ void __launch_bounds__(256) k_rope_store(const RopeParams p) {
    const YattnRopeItem it = item_of(p);
    const uint32_t pairs = p.n_dims / 2;
    // staged in shared memory: a warp's threads index different pairs, and a divergent index into the
    // kernel's parameter bank would serialise
    __shared__ float s_freq[kMaxPairs];
    for (uint32_t j = threadIdx.x; j < pairs; j += blockDim.x) s_freq[j] = p.inv_freq[j];
    __syncthreads();
    const uint32_t nq = p.n_heads * pairs, nk = p.n_kv * pairs, nr = p.n_kv * (p.hd - p.n_dims);
    const uint32_t total = nq + nk + nr + p.kv_dim;
    uint16_t* krow = it.kcache + static_cast<size_t>(it.pos) * p.kv_dim;
    uint16_t* vrow = it.vcache + static_cast<size_t>(it.pos) * p.kv_dim;
    for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u < total; u += gridDim.x * blockDim.x) {
        if (u < nq) {
            const uint32_t h = u / pairs, j = u % pairs;
            uint32_t e0, e1;
            rope_pair(p.kind, p.hd, p.n_dims, j, e0, e1);
            float* qh = it.q + static_cast<size_t>(h) * p.hd;
            float a = qh[e0], b = qh[e1];
            rope_rotate(a, b, s_freq[j], it.pos);
            qh[e0] = a;
            qh[e1] = b;
        } else if (u < nq + nk) {
            const uint32_t w = u - nq, h = w / pairs, j = w % pairs;
            uint32_t e0, e1;
            rope_pair(p.kind, p.hd, p.n_dims, j, e0, e1);
            const float* kh = it.k + static_cast<size_t>(h) * p.hd;
            float a = kh[e0], b = kh[e1];
            rope_rotate(a, b, s_freq[j], it.pos);
            krow[h * p.hd + e0] = engine_f32_to_f16(a);
            krow[h * p.hd + e1] = engine_f32_to_f16(b);
        } else if (u < nq + nk + nr) {
            const uint32_t w = u - nq - nk, h = w / (p.hd - p.n_dims), e = p.n_dims + w % (p.hd - p.n_dims);
            krow[h * p.hd + e] = engine_f32_to_f16(it.k[static_cast<size_t>(h) * p.hd + e]);
        } else {
            const uint32_t e = u - nq - nk - nr;
            vrow[e] = engine_f32_to_f16(it.v[e]);
        }
    }
}

// QK-norm + RoPE + store.  blockIdx.x: q head [0, n_heads), k head [n_heads,
// n_heads + n_kv), then v blocks of 128 elements.  128 threads; head_dim <= 256.
__global__ void __launch_bounds__(128) k_qknorm_rope_store(const RopeParams p) {
    const YattnRopeItem it = item_of(p);
    const uint32_t hd = p.hd, t = threadIdx.x;
    const uint32_t nh = p.n_heads + p.n_kv;
    if (blockIdx.x >= nh) {   // v elements, stored as they are
        const uint32_t e = (blockIdx.x - nh) * 128 + t;
        if (e < p.kv_dim)
            it.vcache[static_cast<size_t>(it.pos) * p.kv_dim + e] = engine_f32_to_f16(it.v[e]);
        return;
    }
    const bool is_q = blockIdx.x < p.n_heads;
    const uint32_t h = is_q ? blockIdx.x : blockIdx.x - p.n_heads;
    const float* src = is_q ? it.q + static_cast<size_t>(h) * hd : it.k + static_cast<size_t>(h) * hd;
    const void* wv = is_q ? p.q_norm_w : p.k_norm_w;
    __shared__ float s_freq[kMaxPairs];
    __shared__ float s_x[2 * kMaxPairs];
    __shared__ float s_inv;
    for (uint32_t j = t; j < p.n_dims / 2; j += 128) s_freq[j] = p.inv_freq[j];
    for (uint32_t e = t; e < hd; e += 128) s_x[e] = src[e];
    __syncthreads();
    if (t == 0) {   // matvec.c:154-157: s += x*x in index order, inv = 1 / sqrt(s/n + eps)
        float sum = 0.0f;
        for (uint32_t i = 0; i < hd; ++i) sum = __fadd_rn(sum, __fmul_rn(s_x[i], s_x[i]));
        s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, static_cast<float>(hd)), p.norm_eps)));
    }
    __syncthreads();
    const float inv = s_inv;
    float y[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {   // matvec.c:160/163: y = x * w * inv, left to right
        const uint32_t e = t + 128 * i;
        if (e < hd) {
            const float w = p.norm_f16 ? h2f(static_cast<const uint16_t*>(wv)[e]) : static_cast<const float*>(wv)[e];
            y[i] = __fmul_rn(__fmul_rn(s_x[e], w), inv);
        }
    }
    __syncthreads();   // every x read before the normalised values replace them
#pragma unroll
    for (int i = 0; i < 2; ++i)
        if (t + 128 * i < hd) s_x[t + 128 * i] = y[i];
    __syncthreads();
    float* qh = is_q ? it.q + static_cast<size_t>(h) * hd : nullptr;
    uint16_t* krow = it.kcache + static_cast<size_t>(it.pos) * p.kv_dim + static_cast<size_t>(h) * hd;
    const uint32_t pairs = p.n_dims / 2;
    for (uint32_t u = t; u < pairs + (hd - p.n_dims); u += 128) {
        if (u < pairs) {
            uint32_t e0, e1;
            rope_pair(p.kind, hd, p.n_dims, u, e0, e1);
            float a = s_x[e0], b = s_x[e1];
            rope_rotate(a, b, s_freq[u], it.pos);
            if (is_q) {
                qh[e0] = a;
                qh[e1] = b;
            } else {
                krow[e0] = engine_f32_to_f16(a);
                krow[e1] = engine_f32_to_f16(b);
            }
        } else {   // dims past the rotated ones (M-RoPE): normalised only
            const uint32_t e = p.n_dims + (u - pairs);
            if (is_q)
                qh[e] = s_x[e];
            else
                krow[e] = engine_f32_to_f16(s_x[e]);
        }
    }
}

}  // namespace
}  // namespace yattn

using namespace yattn;

namespace {

// Checks the geometry and launches; p.items or p.batch already set.
int launch_rope(RopeParams& p, uint32_t n_items, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                uint32_t kv_dim, int rope_kind, uint32_t n_rope_dims, float theta, const YattnQkNorm* qk_norm,
                void* stream, char* err, size_t errlen, const char* who) {
    if (n_heads == 0 || n_kv_heads == 0 || n_kv_heads > n_heads || head_dim == 0 || head_dim > 2 * kMaxPairs ||
        (head_dim & 1) || kv_dim < n_kv_heads * head_dim) {
        set_err(err, errlen, "%s: bad geometry n_heads=%u n_kv_heads=%u head_dim=%u kv_dim=%u", who, n_heads,
                n_kv_heads, head_dim, kv_dim);
        return -1;
    }
    if (rope_kind < 0 || rope_kind > 2) {
        set_err(err, errlen, "%s: rope_kind %d (0 llama, 1 qwen, 2 mrope)", who, rope_kind);
        return -1;
    }
    const uint32_t n_dims = rope_kind == 2 ? n_rope_dims : head_dim;
    if (n_dims == 0 || (n_dims & 1) || n_dims > head_dim) {
        set_err(err, errlen, "%s: %u rotated dims for head_dim %u", who, n_dims, head_dim);
        return -1;
    }
    if (n_items > 65535) {
        set_err(err, errlen, "%s: %u rows (max 65535 per launch)", who, n_items);
        return -1;
    }
    if (qk_norm) {
        if (!qk_norm->q_w || !qk_norm->k_w) {
            set_err(err, errlen, "%s: QK-norm needs both the q and the k weights", who);
            return -1;
        }
        if ((reinterpret_cast<uintptr_t>(qk_norm->q_w) | reinterpret_cast<uintptr_t>(qk_norm->k_w)) &
            (qk_norm->w_f16 ? 1u : 3u)) {
            set_err(err, errlen, "%s: QK-norm weights must be aligned to their element size", who);
            return -1;
        }
        if (n_heads + n_kv_heads + (kv_dim + 127) / 128 > 0x7fffffffu) {
            set_err(err, errlen, "%s: too many heads", who);
            return -1;
        }
        p.q_norm_w = qk_norm->q_w;
        p.k_norm_w = qk_norm->k_w;
        p.norm_f16 = qk_norm->w_f16 ? 1u : 0u;
        p.norm_eps = qk_norm->eps;
    }
    p.n_items = n_items;
    p.n_heads = n_heads;
    p.n_kv = n_kv_heads;
    p.hd = head_dim;
    p.kv_dim = kv_dim;
    p.kind = static_cast<uint32_t>(rope_kind);
    p.n_dims = n_dims;
    // the reference's expression, in the same fp32 operation order (matvec.c:895, 912, 929)
    for (uint32_t j = 0; j < n_dims / 2; ++j)
        p.inv_freq[j] = powf(theta, -2.0f * static_cast<float>(j) / static_cast<float>(n_dims));
    if (p.q_norm_w) {
        k_qknorm_rope_store<<<dim3(n_heads + n_kv_heads + (kv_dim + 127) / 128, n_items), 128, 0,
                              static_cast<cudaStream_t>(stream)>>>(p);
        YATTN_CHECK_LAUNCH(err, errlen, who);
        return 0;
    }
    const uint32_t work = n_heads * (n_dims / 2) + n_kv_heads * (n_dims / 2) + n_kv_heads * (head_dim - n_dims) + kv_dim;
    // one work unit per thread up to 32 blocks per item: the loop body is a chain of dependent memory
    // round trips (item, inputs, stores), so a second pass through it would double the kernel time
    const uint32_t bx = std::max(1u, std::min((work + 255) / 256, 32u));
    k_rope_store<<<dim3(bx, n_items), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
    YATTN_CHECK_LAUNCH(err, errlen, who);
    return 0;
}

}  // namespace

extern "C" int yattn_rope_store_kv(const YattnRopeItem* items_dev, uint32_t n_items, uint32_t n_heads,
                                   uint32_t n_kv_heads, uint32_t head_dim, uint32_t kv_dim, int rope_kind,
                                   uint32_t n_rope_dims, float theta, const YattnQkNorm* qk_norm, void* stream,
                                   char* err, size_t errlen) {
    if (n_items == 0) return 0;
    if (!items_dev) {
        set_err(err, errlen, "rope_store_kv: null items");
        return -1;
    }
    RopeParams p{};
    p.items = items_dev;
    return launch_rope(p, n_items, n_heads, n_kv_heads, head_dim, kv_dim, rope_kind, n_rope_dims, theta, qk_norm,
                       stream, err, errlen, "rope_store_kv");
}

extern "C" int yattn_rope_store_kv_batch(float* q, const float* k, const float* v, uint16_t* kcache,
                                         uint16_t* vcache, uint32_t pos_start, uint32_t B, uint32_t q_stride,
                                         uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, uint32_t kv_dim,
                                         int rope_kind, uint32_t n_rope_dims, float theta,
                                         const YattnQkNorm* qk_norm, void* stream, char* err, size_t errlen) {
    if (B == 0) return 0;
    if (!q || !k || !v || !kcache || !vcache) {
        set_err(err, errlen, "rope_store_kv_batch: null pointer");
        return -1;
    }
    if (q_stride < n_heads * head_dim) {
        set_err(err, errlen, "rope_store_kv_batch: q_stride %u < n_heads*head_dim %u", q_stride, n_heads * head_dim);
        return -1;
    }
    if (static_cast<uint64_t>(pos_start) + B > 0xFFFFFFFFull) {
        set_err(err, errlen, "rope_store_kv_batch: positions overflow");
        return -1;
    }
    RopeParams p{};
    p.items = nullptr;
    p.batch.q = q;
    p.batch.k = k;
    p.batch.v = v;
    p.batch.kcache = kcache;
    p.batch.vcache = vcache;
    p.batch.pos = pos_start;
    p.q_stride = q_stride;
    return launch_rope(p, B, n_heads, n_kv_heads, head_dim, kv_dim, rope_kind, n_rope_dims, theta, qk_norm, stream,
                       err, errlen, "rope_store_kv_batch");
}
