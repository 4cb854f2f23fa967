// gdn.cu -- Qwen3.5 Gated DeltaNet recurrent state update (sm_100a).
//
// Reference semantics: gdn_state_update (inference/core/matvec.c:975-1004) and
// its caller (engine.c:826-852).  Per v-head h (k-head h % num_k_heads), state
// row j (the v index; row stride hv, hk columns):
//     S_j *= e^gate[h];  d = (v_j - S_j.k) * beta[h];  S_j += d * k;
//     out_j = (S_j.q) / sqrt(hv)
// then optionally the per-v-head epilogue rmsnorm_gated (matvec.c:1007-1021):
//     y_j = out_j * w_j / sqrt(mean(out^2) + eps) * silu(z_j).
// All arithmetic fp32.  Rows evolve independently given (k, q, v_j, gate,
// beta), which is what both kernels exploit:
//   k_gdn_decode   one token per sequence; CTA = (v-head, sequence) streams
//                  the 64 KB fp32 state (HBM-bound), epilogue fused.
//   k_gdn_prefill  T tokens of one or more sequences token by token, as the
//                  engine's qwen35 prefill does (engine.c:723-734); CTA = 16
//                  state rows of one v-head kept in registers for the whole
//                  sequence, 16 threads per row, token inputs staged in smem.
//                  yattn_gdn_prefill runs the chunked tensor-core form
//                  (gdn_chunk.cu); this kernel backs yattn_gdn_prefill_recurrent.
#include "common.cuh"

#include <algorithm>

namespace yattn {
namespace {

constexpr int kGdnD = 128;          // head dim (hk == hv) handled by these kernels

struct GdnParams {
    float* S;                       // [n_seq][n_vheads][hv][hk]
    float* out;                     // [n_seq][T][n_vheads*hv]
    const float* q;                 // [n_seq][T][num_k_heads*hk]
    const float* k;
    const float* v;                 // [n_seq][T][n_vheads*hv]
    const float* gate;              // [n_seq][T][n_vheads]
    const float* beta;
    const float* norm_w;            // [hv] or nullptr
    const float* z;                 // [n_seq][T][n_vheads*hv] or nullptr
    uint32_t T, num_k_heads, n_vheads;
    float eps;
};

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// ------------------------------------------------------------------ decode
// 256 threads = 8 warps x 16 rows; lane owns 4 columns.
__global__ void __launch_bounds__(256) k_gdn_decode(const GdnParams p) {
    constexpr int D = kGdnD;
    const uint32_t h = blockIdx.x, sq = blockIdx.y;
    const uint32_t kh = h % p.num_k_heads;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ float s_o[D];
    __shared__ float s_red[8];

    const size_t qk_row = static_cast<size_t>(p.num_k_heads) * D;
    const size_t v_row = static_cast<size_t>(p.n_vheads) * D;
    const float* qh = p.q + sq * qk_row + kh * D;
    const float* kk = p.k + sq * qk_row + kh * D;
    const float* vh = p.v + sq * v_row + static_cast<size_t>(h) * D;
    float* Sh = p.S + (static_cast<size_t>(sq) * p.n_vheads + h) * D * D;
    const float g = expf(p.gate[static_cast<size_t>(sq) * p.n_vheads + h]);
    const float b = p.beta[static_cast<size_t>(sq) * p.n_vheads + h];
    const float scale = 1.0f / sqrtf(static_cast<float>(D));

    const float4 k4 = *reinterpret_cast<const float4*>(kk + lane * 4);
    const float4 q4 = *reinterpret_cast<const float4*>(qh + lane * 4);
    // all 16 rows of this warp in flight at once
    float4 rows[16];
#pragma unroll
    for (int r = 0; r < 16; ++r)
        rows[r] = __ldcs(reinterpret_cast<const float4*>(Sh + static_cast<size_t>(warp * 16 + r) * D + lane * 4));
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        const int j = warp * 16 + r;
        float4 s = rows[r];
        s.x *= g; s.y *= g; s.z *= g; s.w *= g;
        float dot = s.x * k4.x + s.y * k4.y + s.z * k4.z + s.w * k4.w;
        dot = warp_sum(dot);
        const float del = (vh[j] - dot) * b;
        s.x += k4.x * del; s.y += k4.y * del; s.z += k4.z * del; s.w += k4.w * del;
        float o = s.x * q4.x + s.y * q4.y + s.z * q4.z + s.w * q4.w;
        o = warp_sum(o);
        __stcs(reinterpret_cast<float4*>(Sh + static_cast<size_t>(j) * D + lane * 4), s);
        if (lane == 0) s_o[j] = o * scale;
    }
    __syncthreads();
    float* oh = p.out + sq * v_row + static_cast<size_t>(h) * D;
    if (p.norm_w) {
        const int t = threadIdx.x;
        float x = (t < D) ? s_o[t] : 0.f;
        float ss = warp_sum(x * x);
        if (lane == 0) s_red[warp] = ss;
        __syncthreads();
        if (t < D) {
            float tot = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) tot += s_red[w];
            const float inv = 1.0f / sqrtf(tot / static_cast<float>(D) + p.eps);
            const float zg = p.z[sq * v_row + static_cast<size_t>(h) * D + t];
            oh[t] = x * p.norm_w[t] * inv * (zg / (1.0f + expf(-zg)));
        }
    } else if (threadIdx.x < D) {
        oh[threadIdx.x] = s_o[threadIdx.x];
    }
}

// ------------------------------------------------------------------ prefill
constexpr int kRows = 16;           // state rows per CTA
constexpr int kTC = 32;             // tokens staged per chunk

__global__ void __launch_bounds__(256) k_gdn_prefill(const GdnParams p) {
    constexpr int D = kGdnD;
    const uint32_t rb = blockIdx.x, h = blockIdx.y, sq = blockIdx.z;
    const uint32_t kh = h % p.num_k_heads;
    const int tid = threadIdx.x;
    const int rl = tid >> 4;                 // local row 0..15
    const int cg = tid & 15;                 // columns cg*4..cg*4+3 and 64+cg*4..64+cg*4+3 (bank-conflict free)
    const int j = rb * kRows + rl;           // state row (v index)

    __shared__ __align__(16) float s_k[kTC][D];
    __shared__ __align__(16) float s_q[kTC][D];
    __shared__ float s_v[kTC][kRows];
    __shared__ float s_g[kTC], s_b[kTC];

    const size_t qk_row = static_cast<size_t>(p.num_k_heads) * D;
    const size_t v_row = static_cast<size_t>(p.n_vheads) * D;
    const size_t tok0 = static_cast<size_t>(sq) * p.T;
    float* Sh = p.S + (static_cast<size_t>(sq) * p.n_vheads + h) * D * D;
    float st[8];
    {
        const float* src = Sh + static_cast<size_t>(j) * D + cg * 4;
        float4 a = *reinterpret_cast<const float4*>(src), c = *reinterpret_cast<const float4*>(src + 64);
        st[0] = a.x; st[1] = a.y; st[2] = a.z; st[3] = a.w;
        st[4] = c.x; st[5] = c.y; st[6] = c.z; st[7] = c.w;
    }
    const float scale = 1.0f / sqrtf(static_cast<float>(D));

    for (uint32_t t0 = 0; t0 < p.T; t0 += kTC) {
        const int nt = min(static_cast<uint32_t>(kTC), p.T - t0);
        __syncthreads();   // previous chunk fully consumed
        for (int i = tid; i < nt * (D / 4); i += 256) {
            const int tt = i / (D / 4), c4 = (i % (D / 4)) * 4;
            const size_t row = (tok0 + t0 + tt);
            *reinterpret_cast<float4*>(&s_k[tt][c4]) =
                *reinterpret_cast<const float4*>(p.k + row * qk_row + kh * D + c4);
            *reinterpret_cast<float4*>(&s_q[tt][c4]) =
                *reinterpret_cast<const float4*>(p.q + row * qk_row + kh * D + c4);
        }
        for (int i = tid; i < nt * kRows; i += 256) {
            const int tt = i / kRows, r = i % kRows;
            s_v[tt][r] = p.v[(tok0 + t0 + tt) * v_row + static_cast<size_t>(h) * D + rb * kRows + r];
        }
        if (tid < nt) {
            const size_t gi = (tok0 + t0 + tid) * p.n_vheads + h;
            s_g[tid] = expf(p.gate[gi]);
            s_b[tid] = p.beta[gi];
        }
        __syncthreads();
        for (int tt = 0; tt < nt; ++tt) {
            const float4 ka = *reinterpret_cast<const float4*>(&s_k[tt][cg * 4]);
            const float4 kb = *reinterpret_cast<const float4*>(&s_k[tt][cg * 4 + 64]);
            const float kv[8] = {ka.x, ka.y, ka.z, ka.w, kb.x, kb.y, kb.z, kb.w};
            const float g = s_g[tt];
            float dot = 0.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                st[c] *= g;
                dot += st[c] * kv[c];
            }
#pragma unroll
            for (int o = 8; o >= 1; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            const float del = (s_v[tt][rl] - dot) * s_b[tt];
            const float4 qa = *reinterpret_cast<const float4*>(&s_q[tt][cg * 4]);
            const float4 qb = *reinterpret_cast<const float4*>(&s_q[tt][cg * 4 + 64]);
            const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
            float o = 0.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                st[c] += kv[c] * del;
                o += st[c] * qv[c];
            }
#pragma unroll
            for (int s = 8; s >= 1; s >>= 1) o += __shfl_xor_sync(0xffffffffu, o, s);
            if (cg == 0) p.out[(tok0 + t0 + tt) * v_row + static_cast<size_t>(h) * D + j] = o * scale;
        }
    }
    float* dst = Sh + static_cast<size_t>(j) * D + cg * 4;
    *reinterpret_cast<float4*>(dst) = make_float4(st[0], st[1], st[2], st[3]);
    *reinterpret_cast<float4*>(dst + 64) = make_float4(st[4], st[5], st[6], st[7]);
}

// y = x * w / sqrt(mean(x^2) + eps) * silu(z), one warp per (row, v-head) vector of 128.
__global__ void k_rmsnorm_gated(float* y, const float* x, const float* w, const float* z, size_t n_vec,
                                float eps) {
    constexpr int D = kGdnD;
    const size_t vec = blockIdx.x * static_cast<size_t>(blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (vec >= n_vec) return;
    const float4 xv = *reinterpret_cast<const float4*>(x + vec * D + lane * 4);
    float ss = warp_sum(xv.x * xv.x + xv.y * xv.y + xv.z * xv.z + xv.w * xv.w);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
    const float4 wv = *reinterpret_cast<const float4*>(w + lane * 4);
    const float4 zv = *reinterpret_cast<const float4*>(z + vec * D + lane * 4);
    float4 r;
    r.x = xv.x * wv.x * inv * (zv.x / (1.0f + expf(-zv.x)));
    r.y = xv.y * wv.y * inv * (zv.y / (1.0f + expf(-zv.y)));
    r.z = xv.z * wv.z * inv * (zv.z / (1.0f + expf(-zv.z)));
    r.w = xv.w * wv.w * inv * (zv.w / (1.0f + expf(-zv.w)));
    *reinterpret_cast<float4*>(y + vec * D + lane * 4) = r;
}

int check_gdn(const float* S, const float* out, const float* q, const float* k, const float* v, const float* gate,
              const float* beta, uint32_t num_k_heads, uint32_t hk, uint32_t n_vheads, uint32_t hv,
              const float* norm_w, const float* z, char* err, size_t errlen) {
    if (!S || !out || !q || !k || !v || !gate || !beta) {
        set_err(err, errlen, "gdn: null pointer argument");
        return -1;
    }
    if (hk != kGdnD || hv != kGdnD) {
        set_err(err, errlen, "gdn: head dims hk=%u hv=%u not supported (128/128)", hk, hv);
        return -1;
    }
    if (num_k_heads == 0 || n_vheads == 0) {
        set_err(err, errlen, "gdn: bad head counts");
        return -1;
    }
    if ((norm_w == nullptr) != (z == nullptr)) {
        set_err(err, errlen, "gdn: norm_w and z go together");
        return -1;
    }
    const uintptr_t a = reinterpret_cast<uintptr_t>(S) | reinterpret_cast<uintptr_t>(q) |
                        reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(out) |
                        reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(norm_w) |
                        reinterpret_cast<uintptr_t>(z);
    if (a & 15u) {
        set_err(err, errlen, "gdn: S, q, k, v, out, norm_w, z must be 16-byte aligned");
        return -1;
    }
    return 0;
}

}  // namespace

int gdn_decode(float* S, float* out, const float* q, const float* k, const float* v, const float* gate,
               const float* beta, uint32_t n_seqs, uint32_t num_k_heads, uint32_t hk, uint32_t n_vheads, uint32_t hv,
               const float* norm_w, const float* z, float eps, cudaStream_t st, char* err, size_t errlen) {
    if (check_gdn(S, out, q, k, v, gate, beta, num_k_heads, hk, n_vheads, hv, norm_w, z, err, errlen)) return -1;
    if (n_seqs == 0) return 0;
    GdnParams p{S, out, q, k, v, gate, beta, norm_w, z, 1, num_k_heads, n_vheads, eps};
    k_gdn_decode<<<dim3(n_vheads, n_seqs), 256, 0, st>>>(p);
    YATTN_CHECK_LAUNCH(err, errlen, "gdn_decode");
    return 0;
}

size_t gdn_chunk_scratch_bytes(uint32_t n_seqs, uint32_t T, uint32_t num_k_heads, uint32_t n_vheads);
int gdn_prefill_chunked(float* S, float* out, const float* q, const float* k, const float* v, const float* gate,
                        const float* beta, uint32_t n_seqs, uint32_t T, uint32_t num_k_heads, uint32_t n_vheads,
                        void* scratch, cudaStream_t st, char* err, size_t errlen);

// chunked = true: the chunked tensor-core form (gdn_chunk.cu, scratch grown on
// the device context); false: the token-by-token kernel above.
int gdn_prefill(float* S, float* out, const float* q, const float* k, const float* v, const float* gate,
                const float* beta, uint32_t n_seqs, uint32_t T, uint32_t num_k_heads, uint32_t hk, uint32_t n_vheads,
                uint32_t hv, const float* norm_w, const float* z, float eps, bool chunked, cudaStream_t st, char* err,
                size_t errlen) {
    if (check_gdn(S, out, q, k, v, gate, beta, num_k_heads, hk, n_vheads, hv, norm_w, z, err, errlen)) return -1;
    if (n_seqs == 0 || T == 0) return 0;
    if (n_seqs > 65535 || n_vheads > 65535) {
        set_err(err, errlen, "gdn_prefill: too many sequences/heads");
        return -1;
    }
    if (chunked) {
        DevCtx* ctx = dev_ctx(err, errlen);
        if (!ctx) return -1;
        const size_t need = gdn_chunk_scratch_bytes(n_seqs, T, num_k_heads, n_vheads);
        if (ctx->gdn_ws_bytes < need) {
            if (ctx->gdn_ws) cudaFree(ctx->gdn_ws);
            ctx->gdn_ws = nullptr;
            ctx->gdn_ws_bytes = 0;
            if (cudaMalloc(&ctx->gdn_ws, need) != cudaSuccess) {
                set_err(err, errlen, "gdn_prefill: cudaMalloc(%zu) of the chunk scratch failed", need);
                return -1;
            }
            ctx->gdn_ws_bytes = need;
        }
        if (gdn_prefill_chunked(S, out, q, k, v, gate, beta, n_seqs, T, num_k_heads, n_vheads, ctx->gdn_ws, st, err,
                                errlen))
            return -1;
    } else {
        GdnParams p{S, out, q, k, v, gate, beta, norm_w, z, T, num_k_heads, n_vheads, eps};
        k_gdn_prefill<<<dim3(kGdnD / kRows, n_vheads, n_seqs), 256, 0, st>>>(p);
        YATTN_CHECK_LAUNCH(err, errlen, "gdn_prefill");
    }
    if (norm_w) {
        const size_t n_vec = static_cast<size_t>(n_seqs) * T * n_vheads;
        const uint32_t blocks = static_cast<uint32_t>((n_vec + 7) / 8);
        k_rmsnorm_gated<<<blocks, 256, 0, st>>>(out, out, norm_w, z, n_vec, eps);
        YATTN_CHECK_LAUNCH(err, errlen, "gdn_prefill epilogue");
    }
    return 0;
}

}  // namespace yattn

using namespace yattn;

extern "C" void cuda_k_gdn_state_update(float* S, float* out, const float* q, const float* k, const float* v,
                                        const float* gate, const float* beta, uint32_t num_k_heads, uint32_t hk,
                                        uint32_t n_vheads, uint32_t hv) {
    char err[256];
    err[0] = 0;
    if (gdn_decode(S, out, q, k, v, gate, beta, 1, num_k_heads, hk, n_vheads, hv, nullptr, nullptr, 0.f, nullptr,
                   err, sizeof(err)) != 0)
        set_last_error(err);
}

extern "C" int yattn_gdn_decode(float* S, float* out, const float* q, const float* k, const float* v,
                                const float* gate, const float* beta, uint32_t n_seqs, uint32_t num_k_heads,
                                uint32_t hk, uint32_t n_vheads, uint32_t hv, const float* norm_w, const float* z,
                                float eps, void* stream, char* err, size_t errlen) {
    return gdn_decode(S, out, q, k, v, gate, beta, n_seqs, num_k_heads, hk, n_vheads, hv, norm_w, z, eps,
                      static_cast<cudaStream_t>(stream), err, errlen);
}

extern "C" int yattn_gdn_prefill(float* S, float* out, const float* q, const float* k, const float* v,
                                 const float* gate, const float* beta, uint32_t n_seqs, uint32_t T,
                                 uint32_t num_k_heads, uint32_t hk, uint32_t n_vheads, uint32_t hv,
                                 const float* norm_w, const float* z, float eps, void* stream, char* err,
                                 size_t errlen) {
    return gdn_prefill(S, out, q, k, v, gate, beta, n_seqs, T, num_k_heads, hk, n_vheads, hv, norm_w, z, eps, true,
                       static_cast<cudaStream_t>(stream), err, errlen);
}

extern "C" int yattn_gdn_prefill_recurrent(float* S, float* out, const float* q, const float* k, const float* v,
                                           const float* gate, const float* beta, uint32_t n_seqs, uint32_t T,
                                           uint32_t num_k_heads, uint32_t hk, uint32_t n_vheads, uint32_t hv,
                                           const float* norm_w, const float* z, float eps, void* stream, char* err,
                                           size_t errlen) {
    return gdn_prefill(S, out, q, k, v, gate, beta, n_seqs, T, num_k_heads, hk, n_vheads, hv, norm_w, z, eps, false,
                       static_cast<cudaStream_t>(stream), err, errlen);
}
