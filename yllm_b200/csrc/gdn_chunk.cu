// gdn_chunk.cu -- chunked Gated DeltaNet prefill on tensor cores (sm_100a).
//
// Semantics: the token-by-token recurrence of gdn_state_update
// (inference/core/matvec.c:975-1004), run once per token by the qwen35
// prefill (engine.c:723-734).  Per v-head h (k-head h % num_k_heads), with
// the state S (hv x hk, row j = v index) and per token t:
//     S <- e^{a_t} S;   u_t = beta_t (v_t - S k_t);   S <- S + u_t k_t^T;
//     o_t = S q_t / sqrt(hv)
// (a_t = gate, beta_t = beta).  Over a chunk of C = 64 tokens with start
// state S0, let Gamma_t = a_0 + ... + a_t (inclusive) and gamma_t = e^Gamma_t.
// Unrolling the recurrence gives S_t = gamma_t S0 + sum_{i<=t}
// e^{Gamma_t - Gamma_i} u_i k_i^T, and the u_t solve a unit lower-triangular
// system (the WY / UT form of the delta rule: Yang et al. 2024, "Parallelizing
// Linear Transformers with the Delta Rule over Sequence Length"; gating as in
// "Gated Delta Networks"):
//     A[t][i] = beta_t e^{Gamma_t - Gamma_i} (k_t . k_i)      (i < t)
//     T = (I + A)^-1
//     U = T (diag(beta) V - diag(beta gamma) K S0^T)          [C x hv]
//     O = (diag(gamma) Q S0^T + P U) / sqrt(hv),  P[t][i] = e^{Gamma_t - Gamma_i} (q_t . k_i) (i <= t)
//     S_C = gamma_{C-1} S0 + U^T diag(e^{Gamma_{C-1} - Gamma_i}) K
// A partial last chunk is padded with k = q = v = 0, a = 0, beta = 0, which
// leaves every formula exact for the real tokens.
//
// Gamma is a prefix sum in double.  In fp32, |Gamma| reaches tens within a
// chunk, and the difference Gamma_t - Gamma_i of two rounded prefix sums loses
// about ulp(Gamma) (4e-6 at |Gamma| ~ 45) in the exponent of every decay: that
// alone made the chunked state several times noisier than the engine's fp32
// token-by-token products of expf(a_t).  The decays are expf of the
// double-precision difference, e^Gamma and e^(Gamma_63 - Gamma) exp in double.
//
// Two kernels:
//   k_gdn_chunk_prep   (chunk, k-head, seq): everything that does not depend on
//                      S -- Gamma, T and P of each v-head on the k-head -- plus
//                      fp16 hi/lo copies of K and Q.  Fully parallel.
//   k_gdn_chunk_state  (32 state rows, v-head, seq): walks the chunks in order
//                      with its 32 x 128 slice of S in fp32 registers; every
//                      contraction is mma.sync m16n8k16 with both operands split
//                      into fp16 hi + lo (3 products: hi.hi + hi.lo + lo.hi,
//                      about 22 significant bits, fp32 accumulate).
// The optional rmsnorm_gated epilogue runs after, as for the recurrent kernel.
#include "common.cuh"

#include <algorithm>

namespace yattn {
namespace {

constexpr int kC = 64;          // tokens per chunk
constexpr int kD = 128;         // head dim (hk == hv)
constexpr int kR = 32;          // state rows (v index) per CTA of the state kernel
constexpr int LDH = kD + 8;     // smem row stride (halves) of 128-wide fp16 tiles: 272 B, ldmatrix conflict-free
constexpr int LDC = kC + 8;     // smem row stride (halves) of 64-wide fp16 tiles: 144 B
constexpr int LA = kC + 4;      // fp32 row stride of 64 x 64 tiles in the prep kernel (16-B rows)

// Scratch, per (sequence, chunk) sc = seq * n_chunks + chunk:
//   kq[(sc * num_k_heads + kh)]: K_hi, K_lo, Q_hi, Q_lo   fp16 [64][128] each
//   tp[(sc * n_vheads + h)]:     T_hi, T_lo, P_hi, P_lo   fp16 [64][64] each
//   gam[(sc * n_vheads + h)]:    Gamma, e^Gamma, e^(Gamma_63 - Gamma)   fp32 [3][64]
constexpr size_t kKqHalves = 4ull * kC * kD;
constexpr size_t kTpHalves = 4ull * kC * kC;
constexpr size_t kGamFloats = 3ull * kC;

struct ChunkParams {
    const float* q;                 // [n_seq][T][num_k_heads*128]
    const float* k;
    const float* v;                 // [n_seq][T][n_vheads*128]
    const float* gate;              // [n_seq][T][n_vheads]
    const float* beta;
    float* S;                       // [n_seq][n_vheads][128][128]
    float* out;                     // [n_seq][T][n_vheads*128]
    __half* kq;
    __half* tp;
    float* gam;
    uint32_t T, n_chunks, num_k_heads, n_vheads;
};

// ------------------------------------------------------------- mma helpers

__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col)
__device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// d += (ah + al)(bh + bl) without the lo.lo term
__device__ __forceinline__ void mma3(float (&d)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4], uint32_t bh0,
                                     uint32_t bh1, uint32_t bl0, uint32_t bl1) {
    mma(d, ah, bh0, bh1);
    mma(d, ah, bl0, bl1);
    mma(d, al, bh0, bh1);
}
// ldmatrix lane addresses (bytes), row-major halves arrays with row stride ld:
//   A tile 16x16 at (m0, k0)                            -> a0..a3
__device__ __forceinline__ uint32_t a_addr(uint32_t base, int m0, int k0, int ld, int lane) {
    return base + 2u * static_cast<uint32_t>((m0 + (lane & 15)) * ld + k0 + ((lane >> 4) << 3));
}
//   B tiles (k16 x n8) for n-tiles n0, n0+8 of an [n][k] array, non-trans -> b0,b1 | b0,b1
__device__ __forceinline__ uint32_t bnk_addr(uint32_t base, int n0, int k0, int ld, int lane) {
    return base + 2u * static_cast<uint32_t>((n0 + (lane & 7) + ((lane >> 4) << 3)) * ld + k0 +
                                             (((lane >> 3) & 1) << 3));
}
//   B tiles for n-tiles n0, n0+8 of a [k][n] array, trans        -> b0,b1 | b0,b1
__device__ __forceinline__ uint32_t bkn_addr(uint32_t base, int k0, int n0, int ld, int lane) {
    return base + 2u * static_cast<uint32_t>((k0 + (lane & 7) + (((lane >> 3) & 1) << 3)) * ld + n0 +
                                             ((lane >> 4) << 3));
}

// x = hi + lo, hi = fp16(x), lo = fp16(x - hi)
__device__ __forceinline__ void split2(float a, float b, __half2& hi, __half2& lo) {
    hi = __floats2half2_rn(a, b);
    const float2 f = __half22float2(hi);
    lo = __floats2half2_rn(a - f.x, b - f.y);
}
__device__ __forceinline__ void split1(float a, __half& hi, __half& lo) {
    hi = __float2half_rn(a);
    lo = __float2half_rn(a - __half2float(hi));
}

__device__ __forceinline__ void cp16(void* dst_smem, const void* src, bool valid) {
    // zero-fills the 16 bytes when !valid (src-size 0); src stays a valid address
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst_smem)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}

// ------------------------------------------------------------------ prep
// One CTA per (chunk, k-head, sequence).  K K^T and Q K^T depend only on the
// k-head, so they are contracted once, lower triangles only (10 of the 16
// 16x16 output tiles each), and every v-head that reads this k-head
// (h = kh, kh + num_k_heads, ...) then applies its own gates and betas.
// smem: Kh Kl Qh Ql [64][LDH] halves, raw K K^T and Q K^T [64][LA] fp32,
// then per half of the CTA: Gamma [64] double, beta [64] fp32.  Once the
// contractions are done, the two halves (128 threads each) take the v-heads
// in turn, each half with its own A, T [64][LA] and block scratch [3][16][16]
// in the space of the consumed K/Q tiles (grown to fit both halves).
constexpr int kPrepHalfFloats = 2 * kC * LA + 3 * 256;
constexpr int kPrepAlias = std::max(4 * kC * LDH * 2, 2 * kPrepHalfFloats * 4);
constexpr int kPrepSmem = kPrepAlias + 2 * kC * LA * 4 + 2 * kC * 8 + 2 * kC * 4;
static_assert(2 * (kPrepSmem + 1024) <= 233472, "two prep CTAs per SM");

// lower-triangular 16x16 output tile r (0..9) -> (m-tile, n-tile)
__device__ __forceinline__ void tri_tile(int r, int& mt, int& nt) {
    mt = r >= 6 ? 3 : r >= 3 ? 2 : r >= 1 ? 1 : 0;
    nt = r - mt * (mt + 1) / 2;
}

__global__ void __launch_bounds__(256, 2) k_gdn_chunk_prep(const ChunkParams p) {
    extern __shared__ __align__(16) uint8_t smp[];
    __half* Kh = reinterpret_cast<__half*>(smp);
    __half* Kl = Kh + kC * LDH;
    __half* Qh = Kl + kC * LDH;
    __half* Ql = Qh + kC * LDH;
    float* KK = reinterpret_cast<float*>(smp + kPrepAlias);   // raw k_t . k_i   (i <= t)
    float* QK = KK + kC * LA;                              // raw q_t . k_i   (i <= t)

    const uint32_t ch = blockIdx.x, kh = blockIdx.y, sq = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t t0 = ch * kC;
    const uint32_t nvalid = min(static_cast<uint32_t>(kC), p.T - t0);
    const size_t qk_row = static_cast<size_t>(p.num_k_heads) * kD;
    const size_t tok0 = static_cast<size_t>(sq) * p.T + t0;
    const size_t sc = static_cast<size_t>(sq) * p.n_chunks + ch;

    // ---- K, Q -> fp16 hi/lo (all 16 float4 loads of a thread in flight) ----
    constexpr int NL = kC * kD / 4 / 256;   // float4 of K (and of Q) per thread
    float4 kvs[NL], qvs[NL];
#pragma unroll
    for (int j = 0; j < NL; ++j) {
        const int i = tid + 256 * j, t = i / (kD / 4), c = (i % (kD / 4)) * 4;
        kvs[j] = qvs[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (static_cast<uint32_t>(t) < nvalid) {
            kvs[j] = __ldcs(reinterpret_cast<const float4*>(p.k + (tok0 + t) * qk_row + kh * kD + c));
            qvs[j] = __ldcs(reinterpret_cast<const float4*>(p.q + (tok0 + t) * qk_row + kh * kD + c));
        }
    }
#pragma unroll
    for (int j = 0; j < NL; ++j) {
        const int i = tid + 256 * j, t = i / (kD / 4), c = (i % (kD / 4)) * 4;
        const float4 kv = kvs[j], qv = qvs[j];
        __half2 h0, l0, h1, l1;
        split2(kv.x, kv.y, h0, l0);
        split2(kv.z, kv.w, h1, l1);
        *reinterpret_cast<__half2*>(Kh + t * LDH + c) = h0;
        *reinterpret_cast<__half2*>(Kh + t * LDH + c + 2) = h1;
        *reinterpret_cast<__half2*>(Kl + t * LDH + c) = l0;
        *reinterpret_cast<__half2*>(Kl + t * LDH + c + 2) = l1;
        split2(qv.x, qv.y, h0, l0);
        split2(qv.z, qv.w, h1, l1);
        *reinterpret_cast<__half2*>(Qh + t * LDH + c) = h0;
        *reinterpret_cast<__half2*>(Qh + t * LDH + c + 2) = h1;
        *reinterpret_cast<__half2*>(Ql + t * LDH + c) = l0;
        *reinterpret_cast<__half2*>(Ql + t * LDH + c + 2) = l1;
    }
    __syncthreads();
    {   // K/Q hi/lo to the scratch (Kh, Kl, Qh, Ql are consecutive [64][LDH] arrays)
        __half* dst = p.kq + (sc * p.num_k_heads + kh) * kKqHalves;
#pragma unroll 4
        for (int i = tid; i < 4 * kC * (kD / 8); i += 256) {
            const int ar = i / (kD / 8), c = (i % (kD / 8)) * 8;   // ar = array * 64 + row
            *reinterpret_cast<uint4*>(dst + static_cast<size_t>(ar) * kD + c) =
                *reinterpret_cast<const uint4*>(Kh + ar * LDH + c);
        }
    }

    // ---- K K^T and Q K^T, lower-triangular tiles: 20 tiles of 16x16 over the 8 warps ----
    {
        const uint32_t bh_b = smem_u32(Kh), bl_b = smem_u32(Kl);
        const int g = lane >> 2, tq = lane & 3;
#pragma unroll 1
        for (int u = warp; u < 20; u += 8) {
            const int which = u >= 10;
            int mt, nt;
            tri_tile(u - 10 * which, mt, nt);
            const uint32_t ah_b = smem_u32(which ? Qh : Kh), al_b = smem_u32(which ? Ql : Kl);
            float acc[2][4];
#pragma unroll
            for (int n = 0; n < 2; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < kD / 16; ++ks) {
                uint32_t ah[4], al[4], bh[4], bl[4];
                ldsm4(a_addr(ah_b, 16 * mt, 16 * ks, LDH, lane), ah);
                ldsm4(a_addr(al_b, 16 * mt, 16 * ks, LDH, lane), al);
                ldsm4(bnk_addr(bh_b, 16 * nt, 16 * ks, LDH, lane), bh);
                ldsm4(bnk_addr(bl_b, 16 * nt, 16 * ks, LDH, lane), bl);
                mma3(acc[0], ah, al, bh[0], bh[1], bl[0], bl[1]);
                mma3(acc[1], ah, al, bh[2], bh[3], bl[2], bl[3]);
            }
            float* dst = which ? QK : KK;
#pragma unroll
            for (int n = 0; n < 2; ++n) {
                const int t = 16 * mt + g, i = 16 * nt + 8 * n + 2 * tq;
                *reinterpret_cast<float2*>(dst + t * LA + i) = make_float2(acc[n][0], acc[n][1]);
                *reinterpret_cast<float2*>(dst + (t + 8) * LA + i) = make_float2(acc[n][2], acc[n][3]);
            }
        }
    }
    __syncthreads();   // K/Q consumed: the halves' A, T and scratch may overwrite them

    // ---- per v-head: half hf of the CTA takes h = kh + hf * nk, kh + 3 * nk, ... (named barrier 1 + hf) ----
    const int hf = tid >> 7, th = tid & 127, hw = th >> 5;
    double* G = reinterpret_cast<double*>(QK + kC * LA) + hf * kC;   // 8-byte aligned: every array above is
    float* Bt = reinterpret_cast<float*>(reinterpret_cast<double*>(QK + kC * LA) + 2 * kC) + hf * kC;
    float* Am = reinterpret_cast<float*>(smp) + hf * kPrepHalfFloats;   // [64][LA]
    float* Tm = Am + kC * LA;                                           // [64][LA]
    float* Xs = Tm + kC * LA;                                           // [3][16][16]
    auto half_sync = [&]() {
        if (hf == 0)
            asm volatile("bar.sync 1, 128;" ::: "memory");
        else
            asm volatile("bar.sync 2, 128;" ::: "memory");
    };
#pragma unroll 1
    for (uint32_t h = kh + hf * p.num_k_heads; h < p.n_vheads; h += 2 * p.num_k_heads) {
        // Gamma: inclusive prefix sum of the gates in double (warp 0 of the half), published for the state
        // kernel; the betas by warp 1
        if (hw == 0) {
            const bool ok0 = static_cast<uint32_t>(lane) < nvalid, ok1 = static_cast<uint32_t>(32 + lane) < nvalid;
            double x0 = ok0 ? p.gate[(tok0 + lane) * p.n_vheads + h] : 0.f;
            double x1 = ok1 ? p.gate[(tok0 + 32 + lane) * p.n_vheads + h] : 0.f;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const double y0 = __shfl_up_sync(0xffffffffu, x0, o), y1 = __shfl_up_sync(0xffffffffu, x1, o);
                if (lane >= o) {
                    x0 += y0;
                    x1 += y1;
                }
            }
            x1 += __shfl_sync(0xffffffffu, x0, 31);
            G[lane] = x0;
            G[32 + lane] = x1;
            const double glast = __shfl_sync(0xffffffffu, x1, 31);
            float* gm = p.gam + (sc * p.n_vheads + h) * kGamFloats;
            gm[lane] = static_cast<float>(x0);
            gm[32 + lane] = static_cast<float>(x1);
            gm[kC + lane] = static_cast<float>(exp(x0));
            gm[kC + 32 + lane] = static_cast<float>(exp(x1));
            gm[2 * kC + lane] = static_cast<float>(exp(glast - x0));
            gm[2 * kC + 32 + lane] = static_cast<float>(exp(glast - x1));
        } else if (hw == 1) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int t = 32 * j + lane;
                Bt[t] = static_cast<uint32_t>(t) < nvalid ? p.beta[(tok0 + t) * p.n_vheads + h] : 0.f;
            }
        }
        half_sync();

        // A[t][i] = beta_t e^{Gamma_t - Gamma_i} kk (i < t) -> smem;  P[t][i] = e^{Gamma_t - Gamma_i} qk (i <= t)
        // -> fp16 hi/lo scratch.  32 threads per row, two columns each.
        __half* tp = p.tp + (sc * p.n_vheads + h) * kTpHalves;
#pragma unroll 4
        for (int e = th; e < kC * kC / 2; e += 128) {
            const int t = e / (kC / 2), i = (e % (kC / 2)) * 2;
            const double gt = G[t];
            const double2 gi = *reinterpret_cast<const double2*>(G + i);
            const float2 kk = *reinterpret_cast<const float2*>(KK + t * LA + i);
            const float2 qk = *reinterpret_cast<const float2*>(QK + t * LA + i);
            const float bt = Bt[t];
            const float d0 = (i <= t) ? expf(static_cast<float>(gt - gi.x)) : 0.f;
            const float d1 = (i + 1 <= t) ? expf(static_cast<float>(gt - gi.y)) : 0.f;
            const float a[2] = {(i < t) ? bt * d0 * kk.x : 0.f, (i + 1 < t) ? bt * d1 * kk.y : 0.f};
            const float pv[2] = {(i <= t) ? d0 * qk.x : 0.f, (i + 1 <= t) ? d1 * qk.y : 0.f};
            *reinterpret_cast<float2*>(Am + t * LA + i) = make_float2(a[0], a[1]);
            __half2 ph, pl;
            split2(pv[0], pv[1], ph, pl);
            *reinterpret_cast<__half2*>(tp + 2 * kC * kC + t * kC + i) = ph;
            *reinterpret_cast<__half2*>(tp + 3 * kC * kC + t * kC + i) = pl;
        }
        half_sync();

        // ---- T = (I + A)^-1, blocked by 16 (L = I + A is unit lower triangular) ----
        // T_ii = L_ii^-1: the four diagonal blocks by forward substitution, one column per thread (threads 0-63 of the half);
        // then the blocks below, by distance d = i - j from the diagonal: T_ij = -T_ii sum_{j<=k<i} A_ik T_kj,
        // every thread of the half on the 16x16 products, four columns of a row each (float4 operands).
        // The blocks above the diagonal are zero.
        if (th < kC) {
            const int o = th & ~15, c = th & 15;
            float x[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) x[t] = (t == c) ? 1.f : 0.f;
#pragma unroll
            for (int t = 1; t < 16; ++t) {
                float s0 = 0.f, s1 = 0.f;
#pragma unroll
                for (int i = 0; i < t; ++i) {
                    if (i & 1)
                        s1 = fmaf(Am[(o + t) * LA + o + i], x[i], s1);
                    else
                        s0 = fmaf(Am[(o + t) * LA + o + i], x[i], s0);
                }
                if (t > c) x[t] = -(s0 + s1);
            }
#pragma unroll
            for (int t = 0; t < 16; ++t) Tm[(o + t) * LA + o + c] = x[t];
        } else {
            for (int e = th - kC; e < 6 * 256; e += 128 - kC) {   // the 6 blocks above the diagonal
                const int blk = e >> 8, r = (e >> 4) & 15, c = e & 15;
                const int bi = blk < 3 ? 0 : blk < 5 ? 1 : 2, bj = blk < 3 ? blk + 1 : blk < 5 ? blk - 1 : 3;
                Tm[(16 * bi + r) * LA + 16 * bj + c] = 0.f;
            }
        }
        half_sync();
#pragma unroll 1
        for (int d = 1; d < 4; ++d) {
            const int nb = 4 - d;                     // blocks (j + d, j), j < nb; a thread: 4 columns of a row
            for (int e = th; e < nb * 64; e += 128) {
                const int j = e >> 6, r = (e >> 2) & 15, c = (e & 3) * 4, i = j + d;
                float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int k = j; k < i; ++k) {
                    const float* arow = Am + (16 * i + r) * LA + 16 * k;
#pragma unroll
                    for (int m4 = 0; m4 < 16; m4 += 4) {
                        const float4 a4 = *reinterpret_cast<const float4*>(arow + m4);
                        const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
                        for (int mm = 0; mm < 4; ++mm) {
                            const float4 tv =
                                *reinterpret_cast<const float4*>(Tm + (16 * k + m4 + mm) * LA + 16 * j + c);
                            s.x = fmaf(av[mm], tv.x, s.x);
                            s.y = fmaf(av[mm], tv.y, s.y);
                            s.z = fmaf(av[mm], tv.z, s.z);
                            s.w = fmaf(av[mm], tv.w, s.w);
                        }
                    }
                }
                *reinterpret_cast<float4*>(Xs + (j << 8) + r * 16 + c) = s;
            }
            half_sync();
            for (int e = th; e < nb * 64; e += 128) {
                const int j = e >> 6, r = (e >> 2) & 15, c = (e & 3) * 4, i = j + d;
                const float* trow = Tm + (16 * i + r) * LA + 16 * i;
                float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int m4 = 0; m4 < 16; m4 += 4) {
                    const float4 a4 = *reinterpret_cast<const float4*>(trow + m4);
                    const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
                    for (int mm = 0; mm < 4; ++mm) {
                        const float4 xv = *reinterpret_cast<const float4*>(Xs + (j << 8) + (m4 + mm) * 16 + c);
                        s.x = fmaf(av[mm], xv.x, s.x);
                        s.y = fmaf(av[mm], xv.y, s.y);
                        s.z = fmaf(av[mm], xv.z, s.z);
                        s.w = fmaf(av[mm], xv.w, s.w);
                    }
                }
                *reinterpret_cast<float4*>(Tm + (16 * i + r) * LA + 16 * j + c) = make_float4(-s.x, -s.y, -s.z, -s.w);
            }
            half_sync();
        }

        // ---- T -> fp16 hi/lo scratch ----
        for (int e = th; e < kC * kC / 2; e += 128) {
            const int t = e / (kC / 2), c = (e % (kC / 2)) * 2;
            __half2 thi, tl;
            split2(Tm[t * LA + c], Tm[t * LA + c + 1], thi, tl);
            *reinterpret_cast<__half2*>(tp + 0 * kC * kC + t * kC + c) = thi;
            *reinterpret_cast<__half2*>(tp + 1 * kC * kC + t * kC + c) = tl;
        }
        half_sync();   // G, Bt, Am, Tm are rewritten for the half's next v-head
    }
}

// ------------------------------------------------------------------ state
// smem of the state kernel, in halves unless noted:
//   K hi/lo   x2 buffers [64][LDH]   P hi/lo x2 buffers [64][LDC]   (chunk c uses buffer c & 1)
//   Q hi/lo      [64][LDH]           T hi/lo            [64][LDC]
//   S hi/lo      [32][LDH]           Rm^T, U^T, Ud^T hi/lo [32][LDC]
//   V [64][32] fp32, (Gamma, e^Gamma, e^(Gamma_63 - Gamma)) and beta x2 [64] fp32
constexpr int kStateSmem =
    (4 * kC * LDH + 4 * kC * LDC + 2 * kC * LDH + 2 * kC * LDC + 2 * kR * LDH + 6 * kR * LDC) * 2 + kC * kR * 4 +
    2 * (3 + 1) * kC * 4;
static_assert(kStateSmem <= 232448, "state kernel shared memory");

__global__ void __launch_bounds__(256, 1) k_gdn_chunk_state(const ChunkParams p) {
    extern __shared__ __align__(16) uint8_t sms[];
    __half* Kb = reinterpret_cast<__half*>(sms);   // [2 buf][hi, lo][64][LDH]
    __half* Pb = Kb + 4 * kC * LDH;                // [2 buf][hi, lo][64][LDC]
    __half* Qh = Pb + 4 * kC * LDC;                // [64][LDH]
    __half* Ql = Qh + kC * LDH;
    __half* Th = Ql + kC * LDH;                    // [64][LDC]
    __half* Tl = Th + kC * LDC;
    __half* Sh = Tl + kC * LDC;                    // [32][LDH]  S slice (rows r, cols c)
    __half* Sl = Sh + kR * LDH;
    __half* Rh = Sl + kR * LDH;                    // [32][LDC]  Rm^T  (r, token)
    __half* Rl = Rh + kR * LDC;
    __half* Uh = Rl + kR * LDC;                    // [32][LDC]  U^T
    __half* Ul = Uh + kR * LDC;
    __half* Dh = Ul + kR * LDC;                    // [32][LDC]  (decayed U)^T
    __half* Dl = Dh + kR * LDC;
    float* Vs = reinterpret_cast<float*>(Dl + kR * LDC);   // [64][32]
    float* Gb = Vs + kC * kR;                      // [2][3][64] Gamma, e^Gamma, e^(Gamma_63 - Gamma)
    float* Bb = Gb + 2 * kGamFloats;               // [2][64] beta

    const uint32_t rb = blockIdx.x, h = blockIdx.y, sq = blockIdx.z;
    const uint32_t kh = h % p.num_k_heads;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, tq = lane & 3;
    const size_t v_row = static_cast<size_t>(p.n_vheads) * kD;
    float* Sg = p.S + (static_cast<size_t>(sq) * p.n_vheads + h) * kD * kD + static_cast<size_t>(rb) * kR * kD;
    const float inv_sqrt_d = 1.0f / sqrtf(static_cast<float>(kD));

    auto sc_of = [&](uint32_t ch) { return static_cast<size_t>(sq) * p.n_chunks + ch; };
    auto tok_of = [&](uint32_t ch) { return static_cast<size_t>(sq) * p.T + static_cast<size_t>(ch) * kC; };
    auto nvalid_of = [&](uint32_t ch) { return min(static_cast<uint32_t>(kC), p.T - ch * kC); };
    // cp.async staging of chunk ch, one piece at a time (each piece's buffer must be free)
    auto stage_kp = [&](uint32_t ch) {   // K hi/lo, P hi/lo, Gamma, beta into buffer ch & 1
        const int b = ch & 1;
        const size_t sc = sc_of(ch);
        const __half* kq = p.kq + (sc * p.num_k_heads + kh) * kKqHalves;
        for (int i = tid; i < 2 * kC * (kD / 8); i += 256) {
            const int a = i / (kC * (kD / 8)), r = (i / (kD / 8)) % kC, c = (i % (kD / 8)) * 8;
            cp16(Kb + (2 * b + a) * kC * LDH + r * LDH + c, kq + (static_cast<size_t>(a) * kC + r) * kD + c, true);
        }
        const __half* tp = p.tp + (sc * p.n_vheads + h) * kTpHalves + 2 * kC * kC;   // P hi, P lo
        for (int i = tid; i < 2 * kC * (kC / 8); i += 256) {
            const int a = i / (kC * (kC / 8)), r = (i / (kC / 8)) % kC, c = (i % (kC / 8)) * 8;
            cp16(Pb + (2 * b + a) * kC * LDC + r * LDC + c, tp + (static_cast<size_t>(a) * kC + r) * kC + c, true);
        }
        if (tid < static_cast<int>(kGamFloats / 4))
            cp16(Gb + b * kGamFloats + 4 * tid, p.gam + (sc * p.n_vheads + h) * kGamFloats + 4 * tid, true);
        if (tid >= 64 && tid < 64 + kC) {
            const int t = tid - 64;
            Bb[b * kC + t] = static_cast<uint32_t>(t) < nvalid_of(ch) ? p.beta[(tok_of(ch) + t) * p.n_vheads + h] : 0.f;
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    auto stage_qv = [&](uint32_t ch) {   // Q hi/lo and this slice's V
        const size_t sc = sc_of(ch);
        const __half* kq = p.kq + (sc * p.num_k_heads + kh) * kKqHalves + 2 * kC * kD;   // Q hi, Q lo
        for (int i = tid; i < 2 * kC * (kD / 8); i += 256) {
            const int a = i / (kC * (kD / 8)), r = (i / (kD / 8)) % kC, c = (i % (kD / 8)) * 8;
            cp16(Qh + a * kC * LDH + r * LDH + c, kq + (static_cast<size_t>(a) * kC + r) * kD + c, true);
        }
        const uint32_t nv = nvalid_of(ch);
        const size_t tok0 = tok_of(ch);
        for (int i = tid; i < kC * (kR / 4); i += 256) {
            const int t = i / (kR / 4), c = (i % (kR / 4)) * 4;
            const bool ok = static_cast<uint32_t>(t) < nv;
            cp16(Vs + t * kR + c, p.v + (ok ? (tok0 + t) * v_row + h * kD + rb * kR + c : 0), ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    auto stage_t = [&](uint32_t ch) {   // T hi/lo
        const __half* tp = p.tp + (sc_of(ch) * p.n_vheads + h) * kTpHalves;
        for (int i = tid; i < 2 * kC * (kC / 8); i += 256) {
            const int a = i / (kC * (kC / 8)), r = (i / (kC / 8)) % kC, c = (i % (kC / 8)) * 8;
            cp16(Th + a * kC * LDC + r * LDC + c, tp + (static_cast<size_t>(a) * kC + r) * kC + c, true);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    // S slice accumulators: warp -> row tile ms = warp & 1 (16 rows), columns 32 * (warp >> 1) .. +31
    const int ms = warp & 1, cq = warp >> 1;
    float sacc[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int r = 16 * ms + g + ((e >> 1) << 3), c = 32 * cq + 8 * n + 2 * tq + (e & 1);
            sacc[n][e] = Sg[static_cast<size_t>(r) * kD + c];
        }
    }
    auto publish_s = [&]() {
#pragma unroll
        for (int n = 0; n < 4; ++n) {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int r = 16 * ms + g + 8 * half, c = 32 * cq + 8 * n + 2 * tq;
                __half2 hi, lo;
                split2(sacc[n][2 * half], sacc[n][2 * half + 1], hi, lo);
                *reinterpret_cast<__half2*>(Sh + r * LDH + c) = hi;
                *reinterpret_cast<__half2*>(Sl + r * LDH + c) = lo;
            }
        }
    };
    publish_s();
    stage_kp(0);
    stage_qv(0);
    stage_t(0);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();

    const uint32_t Qh_u = smem_u32(Qh), Ql_u = smem_u32(Ql);
    const uint32_t Th_u = smem_u32(Th), Tl_u = smem_u32(Tl);
    const uint32_t Sh_u = smem_u32(Sh), Sl_u = smem_u32(Sl), Rh_u = smem_u32(Rh), Rl_u = smem_u32(Rl);
    const uint32_t Uh_u = smem_u32(Uh), Ul_u = smem_u32(Ul), Dh_u = smem_u32(Dh), Dl_u = smem_u32(Dl);

    for (uint32_t ch = 0; ch < p.n_chunks; ++ch) {
        const int b = ch & 1;
        const bool more = ch + 1 < p.n_chunks;
        const uint32_t nvalid = nvalid_of(ch);
        const size_t tok0 = tok_of(ch);
        const uint32_t Kh_u = smem_u32(Kb + (2 * b) * kC * LDH), Kl_u = smem_u32(Kb + (2 * b + 1) * kC * LDH);
        const uint32_t Ph_u = smem_u32(Pb + (2 * b) * kC * LDC), Pl_u = smem_u32(Pb + (2 * b + 1) * kC * LDC);
        const float* Ge = Gb + b * kGamFloats + kC;       // e^Gamma_t
        const float* Gd = Gb + b * kGamFloats + 2 * kC;   // e^(Gamma_63 - Gamma_t)
        const float* Bs = Bb + b * kC;
        if (more) stage_kp(ch + 1);   // the other buffer: chunk ch - 1 is done with it

        // ---- phase A: R1 = K S^T (warps 0-3) and O1 = Q S^T (warps 4-7); m-tile = warp & 3 ----
        const int mt = warp & 3, which = warp >> 2;
        float acc[4][4];
#pragma unroll
        for (int n = 0; n < 4; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
        {
            const uint32_t ah_b = which ? Qh_u : Kh_u, al_b = which ? Ql_u : Kl_u;
#pragma unroll
            for (int ks = 0; ks < kD / 16; ++ks) {
                uint32_t ah[4], al[4];
                ldsm4(a_addr(ah_b, 16 * mt, 16 * ks, LDH, lane), ah);
                ldsm4(a_addr(al_b, 16 * mt, 16 * ks, LDH, lane), al);
#pragma unroll
                for (int np = 0; np < 2; ++np) {
                    uint32_t bh[4], bl[4];
                    ldsm4(bnk_addr(Sh_u, 16 * np, 16 * ks, LDH, lane), bh);
                    ldsm4(bnk_addr(Sl_u, 16 * np, 16 * ks, LDH, lane), bl);
                    mma3(acc[2 * np], ah, al, bh[0], bh[1], bl[0], bl[1]);
                    mma3(acc[2 * np + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
                }
            }
        }
        // epilogue A: Rm = beta (V - gamma R1) -> Rm^T hi/lo;  O1 <- gamma O1 (kept in registers)
        {
            const int ta = 16 * mt + g, tb = ta + 8;
            const float ga = Ge[ta], gb = Ge[tb];
            if (which == 0) {
                const float ba = Bs[ta], bb = Bs[tb];
#pragma unroll
                for (int n = 0; n < 4; ++n) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int t = (e < 2) ? ta : tb, r = 8 * n + 2 * tq + (e & 1);
                        const float rm = ((e < 2) ? ba : bb) * (Vs[t * kR + r] - ((e < 2) ? ga : gb) * acc[n][e]);
                        __half hi, lo;
                        split1(rm, hi, lo);
                        Rh[r * LDC + t] = hi;
                        Rl[r * LDC + t] = lo;
                    }
                }
            } else {
#pragma unroll
                for (int n = 0; n < 4; ++n) {
                    acc[n][0] *= ga;
                    acc[n][1] *= ga;
                    acc[n][2] *= gb;
                    acc[n][3] *= gb;
                }
            }
        }
        __syncthreads();
        if (more) stage_qv(ch + 1);   // Q and V of this chunk are consumed

        // ---- phase B: U = T Rm, all warps: m-tile = warp & 3, S-row tiles 16 * (warp >> 2) .. +15 ----
        {
            const int np = warp >> 2;
            float u[2][4];
#pragma unroll
            for (int n = 0; n < 2; ++n) u[n][0] = u[n][1] = u[n][2] = u[n][3] = 0.f;
            for (int ks = 0; ks <= mt; ++ks) {   // T is lower triangular
                uint32_t th[4], tl[4], bh[4], bl[4];
                ldsm4(a_addr(Th_u, 16 * mt, 16 * ks, LDC, lane), th);
                ldsm4(a_addr(Tl_u, 16 * mt, 16 * ks, LDC, lane), tl);
                ldsm4(bnk_addr(Rh_u, 16 * np, 16 * ks, LDC, lane), bh);
                ldsm4(bnk_addr(Rl_u, 16 * np, 16 * ks, LDC, lane), bl);
                mma3(u[0], th, tl, bh[0], bh[1], bl[0], bl[1]);
                mma3(u[1], th, tl, bh[2], bh[3], bl[2], bl[3]);
            }
#pragma unroll
            for (int n = 0; n < 2; ++n) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int t = 16 * mt + g + ((e >> 1) << 3), r = 16 * np + 8 * n + 2 * tq + (e & 1);
                    __half hi, lo;
                    split1(u[n][e], hi, lo);
                    Uh[r * LDC + t] = hi;
                    Ul[r * LDC + t] = lo;
                    split1(u[n][e] * Gd[t], hi, lo);
                    Dh[r * LDC + t] = hi;
                    Dl[r * LDC + t] = lo;
                }
            }
        }
        __syncthreads();
        if (more) stage_t(ch + 1);   // T of this chunk is consumed

        // ---- phase C1 (warps 4-7): O = gamma O1 + P U, written out / sqrt(hv) ----
        if (which == 1) {
            for (int ks = 0; ks <= mt; ++ks) {   // P is lower triangular
                uint32_t ph[4], pl[4];
                ldsm4(a_addr(Ph_u, 16 * mt, 16 * ks, LDC, lane), ph);
                ldsm4(a_addr(Pl_u, 16 * mt, 16 * ks, LDC, lane), pl);
#pragma unroll
                for (int np = 0; np < 2; ++np) {
                    uint32_t bh[4], bl[4];
                    ldsm4(bnk_addr(Uh_u, 16 * np, 16 * ks, LDC, lane), bh);
                    ldsm4(bnk_addr(Ul_u, 16 * np, 16 * ks, LDC, lane), bl);
                    mma3(acc[2 * np], ph, pl, bh[0], bh[1], bl[0], bl[1]);
                    mma3(acc[2 * np + 1], ph, pl, bh[2], bh[3], bl[2], bl[3]);
                }
            }
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int t = 16 * mt + g + 8 * half;
                if (static_cast<uint32_t>(t) < nvalid) {
                    float* o = p.out + (tok0 + t) * v_row + h * kD + rb * kR;
#pragma unroll
                    for (int n = 0; n < 4; ++n)
                        *reinterpret_cast<float2*>(o + 8 * n + 2 * tq) =
                            make_float2(acc[n][2 * half] * inv_sqrt_d, acc[n][2 * half + 1] * inv_sqrt_d);
                }
            }
        }
        // ---- phase C2 (all warps): S <- gamma_last S + (decayed U)^T K ----
        {
            const float gl = Ge[kC - 1];
#pragma unroll
            for (int n = 0; n < 4; ++n) {
                sacc[n][0] *= gl;
                sacc[n][1] *= gl;
                sacc[n][2] *= gl;
                sacc[n][3] *= gl;
            }
#pragma unroll
            for (int ks = 0; ks < kC / 16; ++ks) {
                uint32_t dh[4], dl[4];
                ldsm4(a_addr(Dh_u, 16 * ms, 16 * ks, LDC, lane), dh);
                ldsm4(a_addr(Dl_u, 16 * ms, 16 * ks, LDC, lane), dl);
#pragma unroll
                for (int np = 0; np < 2; ++np) {
                    uint32_t bh[4], bl[4];
                    ldsm4t(bkn_addr(Kh_u, 16 * ks, 32 * cq + 16 * np, LDH, lane), bh);
                    ldsm4t(bkn_addr(Kl_u, 16 * ks, 32 * cq + 16 * np, LDH, lane), bl);
                    mma3(sacc[2 * np], dh, dl, bh[0], bh[1], bl[0], bl[1]);
                    mma3(sacc[2 * np + 1], dh, dl, bh[2], bh[3], bl[2], bl[3]);
                }
            }
        }
        publish_s();
        asm volatile("cp.async.wait_group 0;" ::: "memory");   // chunk ch + 1 staged
        __syncthreads();
    }
#pragma unroll
    for (int n = 0; n < 4; ++n) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int r = 16 * ms + g + 8 * half, c = 32 * cq + 8 * n + 2 * tq;
            *reinterpret_cast<float2*>(Sg + static_cast<size_t>(r) * kD + c) =
                make_float2(sacc[n][2 * half], sacc[n][2 * half + 1]);
        }
    }
}

}  // namespace

size_t gdn_chunk_scratch_bytes(uint32_t n_seqs, uint32_t T, uint32_t num_k_heads, uint32_t n_vheads) {
    const size_t n_chunks = (T + kC - 1) / kC;
    const size_t sc = static_cast<size_t>(n_seqs) * n_chunks;
    const size_t kq = sc * num_k_heads * kKqHalves * 2;
    const size_t tp = sc * n_vheads * kTpHalves * 2;
    const size_t gam = sc * n_vheads * kGamFloats * 4;
    return kq + tp + gam;
}

// Geometry was checked by the caller (hk == hv == 128, aligned pointers).
int gdn_prefill_chunked(float* S, float* out, const float* q, const float* k, const float* v, const float* gate,
                        const float* beta, uint32_t n_seqs, uint32_t T, uint32_t num_k_heads, uint32_t n_vheads,
                        void* scratch, cudaStream_t st, char* err, size_t errlen) {
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        if (cudaFuncSetAttribute(k_gdn_chunk_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, kPrepSmem) !=
                cudaSuccess ||
            cudaFuncSetAttribute(k_gdn_chunk_state, cudaFuncAttributeMaxDynamicSharedMemorySize, kStateSmem) !=
                cudaSuccess) {
            set_err(err, errlen, "gdn_prefill: shared-memory attribute failed");
            return -1;
        }
        attr_done[dev] = true;
    }
    const uint32_t n_chunks = (T + kC - 1) / kC;
    const size_t sc = static_cast<size_t>(n_seqs) * n_chunks;
    ChunkParams p{};
    p.q = q;
    p.k = k;
    p.v = v;
    p.gate = gate;
    p.beta = beta;
    p.S = S;
    p.out = out;
    p.kq = static_cast<__half*>(scratch);
    p.tp = p.kq + sc * num_k_heads * kKqHalves;
    p.gam = reinterpret_cast<float*>(p.tp + sc * n_vheads * kTpHalves);
    p.T = T;
    p.n_chunks = n_chunks;
    p.num_k_heads = num_k_heads;
    p.n_vheads = n_vheads;
    k_gdn_chunk_prep<<<dim3(n_chunks, num_k_heads, n_seqs), 256, kPrepSmem, st>>>(p);
    YATTN_CHECK_LAUNCH(err, errlen, "gdn_prefill chunk prep");
    k_gdn_chunk_state<<<dim3(kD / kR, n_vheads, n_seqs), 256, kStateSmem, st>>>(p);
    YATTN_CHECK_LAUNCH(err, errlen, "gdn_prefill chunk state");
    return 0;
}

}  // namespace yattn
