// gemv.cu -- the per-layer linear layers around attention: y = W x for Q4_K
// and fp16 weights, one token (GEMV) or a few (GEMM with weights read once).
//
// Reference: cuda_k_gemv_q4k / cuda_k_gemm_q4k (cuda_kernels.cu:161-249: one
// CTA per output row and token, fp32 x, each weight dequantised as
// d*sc*nib - dmin*mn) and cuda_k_gemv_f16 / cuda_k_gemm_f16
// (cuda_kernels.cu:36-128: cuBLAS with x rounded to fp16 when a handle is
// given, else one thread per row in fp32).  The CPU engine's matmul
// (matvec.c:514, 789) computes the same products; its AVX2 Q4_K path
// quantises x to int8 first.
//
// Here both read each weight byte once per launch, which is the bound (HBM):
//   Q4_K: a 256-weight block is 144 B (d, dmin fp16; 12 B of 6-bit scales and
//         mins; 128 B of nibbles).  Lane l of a warp takes nibble bytes
//         4l..4l+3 of every block of a row: low nibbles of group 2(l/8), high
//         nibbles of group 2(l/8)+1.  Per group it forms sum(nib*x) and sum(x)
//         and adds d*sc*sum(nib*x) - dmin*mn*sum(x), the reference's
//         per-weight expression summed in another order.
//   fp16: lane l takes 8 consecutive weights (16 B) per 256-weight stripe.
// A CTA works on R rows at once so each x value a lane loads serves R weights
// (x would otherwise cost 8x the weight bytes in L1 traffic), and on NT tokens
// at once so each weight serves NT tokens.  Its warps split the rows' length,
// so a matrix of few rows still spreads over the whole GPU, and reduce through
// shared memory at the end.  Accumulation is fp32; x stays fp32 (the
// reference's cuBLAS path rounds it to fp16).
#include "common.cuh"

#include <algorithm>

namespace yattn {
namespace {

constexpr int kWarps = 8;          // warps per CTA
constexpr int kQ4kBlock = 144;     // bytes per 256 weights

__device__ __forceinline__ uint32_t byte_of(const uint4& h, int k) {   // byte k (4..15) of a 16-byte header
    const uint32_t w = k < 8 ? h.y : k < 12 ? h.z : h.w;
    return (w >> (8 * (k & 3))) & 0xFFu;
}

// 6-bit scale and min of group j (0..7) from the 12 scale bytes at header bytes 4..15 (matvec.c:26-35).
__device__ __forceinline__ void scale_min(const uint4& h, int j, float& sc, float& mn) {
    auto q = [&](int k) { return byte_of(h, 4 + k); };
    uint32_t s, m;
    if (j < 4) {
        s = q(j) & 63u;
        m = q(j + 4) & 63u;
    } else {
        s = (q(j + 4) & 0xFu) | ((q(j - 4) >> 6) << 4);
        m = (q(j + 4) >> 4) | ((q(j) >> 6) << 4);
    }
    sc = static_cast<float>(s);
    mn = static_cast<float>(m);
}

__device__ __forceinline__ float half_lo(uint32_t v) { return __half2float(__ushort_as_half(static_cast<unsigned short>(v & 0xFFFFu))); }
__device__ __forceinline__ float half_hi(uint32_t v) { return __half2float(__ushort_as_half(static_cast<unsigned short>(v >> 16))); }

__device__ __forceinline__ uint4 ldg_nc16(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ldg_nc4(const void* p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sums acc[r][t] over the CTA's warps and writes y.  red: kWarps * R * NT floats of shared memory.
template <int R, int NT>
__device__ __forceinline__ void reduce_store(float (&acc)[R][NT], float* red, float* y, uint32_t row0, uint32_t out,
                                             uint32_t nt) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const float v = warp_sum(acc[r][t]);
            if (lane == 0) red[(warp * R + r) * NT + t] = v;
        }
    __syncthreads();
    if (threadIdx.x < R * NT) {
        const int r = threadIdx.x / NT, t = threadIdx.x % NT;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += red[(w * R + r) * NT + t];
        if (row0 + r < out && t < static_cast<int>(nt)) y[static_cast<size_t>(t) * out + row0 + r] = v;
    }
}

// One CTA per R consecutive rows; warp w takes blocks w, w + kWarps, ... of every row (the row's length split
// across the warps, so even a short matrix fills the GPU), U blocks per step with all their loads in flight.
// y[t][row] for tokens [0, nt); x [nt][in], y [nt][out].
template <int R, int NT, int U>
__global__ void __launch_bounds__(kWarps * 32) k_gemv_q4k(float* __restrict__ y, const uint8_t* __restrict__ w,
                                                         const float* __restrict__ x, uint32_t out, uint32_t in,
                                                         uint32_t nt) {
    __shared__ float red[kWarps * R * NT];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t row0 = blockIdx.x * R;
    const uint32_t nb = in / 256;
    const size_t row_bytes = static_cast<size_t>(nb) * kQ4kBlock;
    const int pp = lane >> 3, e0 = 4 * (lane & 7);
    const int g0 = 2 * pp, g1 = g0 + 1;
    float acc[R][NT];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    const uint8_t* rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = w + static_cast<size_t>(min(row0 + r, out - 1)) * row_bytes;

    for (uint32_t b0 = warp; b0 < nb; b0 += U * kWarps) {
        uint4 hdr[U][R];
        uint32_t qv[U][R];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint32_t b = min(b0 + u * kWarps, nb - 1);   // past the row: a repeat, weighted 0 below
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const uint8_t* blk = rows[r] + static_cast<size_t>(b) * kQ4kBlock;
                hdr[u][r] = ldg_nc16(blk);
                qv[u][r] = ldg_nc4(blk + 16 + 4 * lane);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint32_t b = b0 + u * kWarps;
            if (b >= nb) break;
            float xs0[NT][4], xs1[NT][4], sx0[NT], sx1[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if (t < static_cast<int>(nt)) {
                    const float* xb = x + static_cast<size_t>(t) * in + b * 256;
                    const float4 a = *reinterpret_cast<const float4*>(xb + g0 * 32 + e0);
                    const float4 c = *reinterpret_cast<const float4*>(xb + g1 * 32 + e0);
                    xs0[t][0] = a.x; xs0[t][1] = a.y; xs0[t][2] = a.z; xs0[t][3] = a.w;
                    xs1[t][0] = c.x; xs1[t][1] = c.y; xs1[t][2] = c.z; xs1[t][3] = c.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) xs0[t][i] = xs1[t][i] = 0.f;
                }
                sx0[t] = (xs0[t][0] + xs0[t][1]) + (xs0[t][2] + xs0[t][3]);
                sx1[t] = (xs1[t][0] + xs1[t][1]) + (xs1[t][2] + xs1[t][3]);
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const float d = half_lo(hdr[u][r].x), dmin = half_hi(hdr[u][r].x);
                float sc0, mn0, sc1, mn1;
                scale_min(hdr[u][r], g0, sc0, mn0);
                scale_min(hdr[u][r], g1, sc1, mn1);
                const float d0 = d * sc0, m0 = dmin * mn0, d1 = d * sc1, m1 = dmin * mn1;
                float nl[4], nh[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    nl[i] = static_cast<float>((qv[u][r] >> (8 * i)) & 0xFu);
                    nh[i] = static_cast<float>((qv[u][r] >> (8 * i + 4)) & 0xFu);
                }
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    float s0 = nl[0] * xs0[t][0], s1 = nh[0] * xs1[t][0];
#pragma unroll
                    for (int i = 1; i < 4; ++i) {
                        s0 = fmaf(nl[i], xs0[t][i], s0);
                        s1 = fmaf(nh[i], xs1[t][i], s1);
                    }
                    acc[r][t] += (d0 * s0 - m0 * sx0[t]) + (d1 * s1 - m1 * sx1[t]);
                }
            }
        }
    }
    reduce_store<R, NT>(acc, red, y, row0, out, nt);
}

// Single-token Q4_K GEMV.  A warp step covers 4 blocks of R rows: lane l takes nibble bytes 16(l%8)..+15 of
// block 4*step + l/8, i.e. elements e0..e0+15 (e0 = 16*(l%2)) of the pair p = (l%8)/2: group 2p from the low
// nibbles, group 2p+1 from the high ones.  Four nibbles become bytes 0x80|n with one LOP3, and each byte
// becomes the float 1 + n/128 with one byte permute (into byte 2 of 1.0f), so
//   sum(n*x) = 128 * (sum((1 + n/128) * x) - sum(x)),
// one FFMA per weight; sum(x) per group is shared by the R rows.  Each group's scale and min are decoded once
// per block by one lane and passed to the two lanes that use them.
// The CTA's 8 warps are KS k-slices (steps ks, ks + KS, ...) of 8/KS row groups of R rows, KS chosen so every
// warp has a step even when a row has few blocks; the slices meet in shared memory.
template <int R, int KS>
__global__ void __launch_bounds__(kWarps * 32) k_gemv_q4k_t1(float* __restrict__ y, const uint8_t* __restrict__ w,
                                                            const float* __restrict__ x, uint32_t out, uint32_t in) {
    constexpr int RG = kWarps / KS;                   // row groups per CTA
    __shared__ float red[kWarps * R];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rg = warp / KS, ks = warp % KS;
    const uint32_t row0 = (blockIdx.x * RG + rg) * R;
    const uint32_t nb = in / 256;
    const size_t row_bytes = static_cast<size_t>(nb) * kQ4kBlock;
    const int k = lane & 7, sub = lane >> 3;          // chunk of the block, block of the step
    const int p = k >> 1, e0 = 16 * (k & 1);
    const int glo = 2 * p, ghi = glo + 1;
    const int src_lo = (lane & ~7) | glo, src_hi = (lane & ~7) | ghi;   // lanes holding my groups' scales
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    const uint8_t* rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = w + static_cast<size_t>(min(row0 + r, out - 1)) * row_bytes;
    const uint32_t nsteps = (nb + 3) / 4;
    uint4 hA[R], qA[R];
    auto load = [&](uint32_t st, uint4 (&H)[R], uint4 (&Q)[R]) {
        const uint32_t bb = min(st * 4 + sub, nb - 1);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const uint8_t* blk = rows[r] + static_cast<size_t>(bb) * kQ4kBlock;
            H[r] = ldg_nc16(blk);
            Q[r] = ldg_nc16(blk + 16 + 16 * k);
        }
    };
    auto compute = [&](uint32_t st, const uint4 (&H)[R], const uint4 (&Q)[R]) {
        const uint32_t b = st * 4 + sub;
        const bool valid = b < nb;
        const uint32_t bb = valid ? b : nb - 1;
        float xl[16], xh[16];
        const float* xb = x + static_cast<size_t>(bb) * 256;
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
            const float4 a = *reinterpret_cast<const float4*>(xb + glo * 32 + e0 + i);
            const float4 c = *reinterpret_cast<const float4*>(xb + ghi * 32 + e0 + i);
            xl[i] = a.x; xl[i + 1] = a.y; xl[i + 2] = a.z; xl[i + 3] = a.w;
            xh[i] = c.x; xh[i + 1] = c.y; xh[i + 2] = c.z; xh[i + 3] = c.w;
        }
        float sxl = 0.f, sxh = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            sxl += xl[i];
            sxh += xh[i];
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            // my lane decodes group k of this block; the lanes of groups glo / ghi pass theirs over
            float sc, mn;
            scale_min(H[r], k, sc, mn);
            const float d = half_lo(H[r].x), dmin = half_hi(H[r].x);
            const float dk = d * sc, mk = dmin * mn;
            const float d_lo = __shfl_sync(0xffffffffu, dk, src_lo), m_lo = __shfl_sync(0xffffffffu, mk, src_lo);
            const float d_hi = __shfl_sync(0xffffffffu, dk, src_hi), m_hi = __shfl_sync(0xffffffffu, mk, src_hi);
            const uint32_t q[4] = {Q[r].x, Q[r].y, Q[r].z, Q[r].w};
            float sl[4], sh[4];   // four partial sums each: short FMA chains
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                sl[j] = 0.f;
                sh[j] = 0.f;
                // the word's 4 low / 4 high nibbles as bytes 0x80|n: byte 2 of the float 1.0f (0x3F800000) is
                // 0x80, so placing 0x80|n there by one byte permute gives 1 + n/128 exactly
                const uint32_t lob = (q[j] & 0x0F0F0F0Fu) | 0x80808080u;
                const uint32_t hib = ((q[j] >> 4) & 0x0F0F0F0Fu) | 0x80808080u;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t sel = 0x7044u | (static_cast<uint32_t>(i) << 8);   // bytes [0, 0, b_i, 0x3F]
                    const float fl = __uint_as_float(__byte_perm(lob, 0x3F000000u, sel));
                    const float fh = __uint_as_float(__byte_perm(hib, 0x3F000000u, sel));
                    sl[j] = fmaf(fl, xl[4 * j + i], sl[j]);
                    sh[j] = fmaf(fh, xh[4 * j + i], sh[j]);
                }
            }
            const float nl = 128.f * (((sl[0] + sl[1]) + (sl[2] + sl[3])) - sxl);   // sum(n*x), low group
            const float nh = 128.f * (((sh[0] + sh[1]) + (sh[2] + sh[3])) - sxh);
            const float v = (d_lo * nl - m_lo * sxl) + (d_hi * nh - m_hi * sxh);
            acc[r] += valid ? v : 0.f;
        }
    };
    for (uint32_t st = ks; st < nsteps; st += KS) {
        load(st, hA, qA);
        compute(st, hA, qA);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const float v = warp_sum(acc[r]);
        if (lane == 0) red[warp * R + r] = v;
    }
    __syncthreads();
    if (threadIdx.x < RG * R) {
        const int g = threadIdx.x / R, r = threadIdx.x % R;
        float v = 0.f;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) v += red[(g * KS + kk) * R + r];
        const uint32_t row = (blockIdx.x * RG + g) * R + r;
        if (row < out) y[row] = v;
    }
}

// fp16 weights [out][in], in % 8 == 0 and 16-byte aligned rows and x.  One CTA per R rows; warp w takes
// 256-weight stripes w, w + kWarps, ... of every row, U stripes per step.
template <int R, int NT, int U>
__global__ void __launch_bounds__(kWarps * 32) k_gemv_f16(float* __restrict__ y, const uint16_t* __restrict__ w,
                                                         const float* __restrict__ x, uint32_t out, uint32_t in,
                                                         uint32_t nt) {
    __shared__ float red[kWarps * R * NT];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t row0 = blockIdx.x * R;
    const uint32_t ns = (in + 255) / 256;   // stripes per row
    float acc[R][NT];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    const uint16_t* rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = w + static_cast<size_t>(min(row0 + r, out - 1)) * in;
    for (uint32_t s0 = warp; s0 < ns; s0 += U * kWarps) {
        uint4 wv[U][R];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint32_t c = (s0 + u * kWarps) * 256 + 8 * lane;
            const bool ok = c < in;
#pragma unroll
            for (int r = 0; r < R; ++r) wv[u][r] = ok ? ldg_nc16(rows[r] + c) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint32_t c = (s0 + u * kWarps) * 256 + 8 * lane;
            if (c >= in) continue;
            float xv[NT][8];
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if (t < static_cast<int>(nt)) {
                    const float4 a = *reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * in + c);
                    const float4 b = *reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * in + c + 4);
                    xv[t][0] = a.x; xv[t][1] = a.y; xv[t][2] = a.z; xv[t][3] = a.w;
                    xv[t][4] = b.x; xv[t][5] = b.y; xv[t][6] = b.z; xv[t][7] = b.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) xv[t][i] = 0.f;
                }
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const uint32_t q[4] = {wv[u][r].x, wv[u][r].y, wv[u][r].z, wv[u][r].w};
                float wf[8];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    wf[2 * i] = half_lo(q[i]);
                    wf[2 * i + 1] = half_hi(q[i]);
                }
#pragma unroll
                for (int t = 0; t < NT; ++t)
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[r][t] = fmaf(wf[i], xv[t][i], acc[r][t]);
            }
        }
    }
    reduce_store<R, NT>(acc, red, y, row0, out, nt);
}

// fp16 weights, any in or alignment: one warp per row, scalar loads.
__global__ void __launch_bounds__(kWarps * 32) k_gemv_f16_any(float* __restrict__ y, const uint16_t* __restrict__ w,
                                                             const float* __restrict__ x, uint32_t out, uint32_t in,
                                                             uint32_t nt) {
    const int lane = threadIdx.x & 31;
    const uint32_t row = blockIdx.x * kWarps + (threadIdx.x >> 5);
    if (row >= out) return;
    const uint16_t* wr = w + static_cast<size_t>(row) * in;
    for (uint32_t t = 0; t < nt; ++t) {
        float acc = 0.f;
        for (uint32_t c = lane; c < in; c += 32)
            acc = fmaf(__half2float(__ushort_as_half(wr[c])), x[static_cast<size_t>(t) * in + c], acc);
        acc = warp_sum(acc);
        if (lane == 0) y[static_cast<size_t>(t) * out + row] = acc;
    }
}

constexpr int kR = 4;   // rows per CTA
constexpr int kNT = 4;  // tokens per pass over the weights

constexpr int kR1 = 4;  // rows per warp of the single-token Q4_K kernel

template <int KS>
void launch_q4k_t1(float* y, const uint8_t* w, const float* x, uint32_t out, uint32_t in, cudaStream_t st) {
    constexpr uint32_t rows_per_cta = (kWarps / KS) * kR1;
    k_gemv_q4k_t1<kR1, KS><<<(out + rows_per_cta - 1) / rows_per_cta, kWarps * 32, 0, st>>>(y, w, x, out, in);
}

template <int NT>
void launch_q4k(float* y, const uint8_t* w, const float* x, uint32_t out, uint32_t in, uint32_t nt, cudaStream_t st) {
    if (NT == 1) {
        // as many k-slices as a row has steps (up to the CTA's 8 warps): the fewest rows per CTA, so even a
        // matrix of 1024 rows spreads over every SM
        const uint32_t nsteps = (in / 256 + 3) / 4;   // 4-block steps per row
        if (nsteps >= 8)
            launch_q4k_t1<8>(y, w, x, out, in, st);
        else if (nsteps >= 4)
            launch_q4k_t1<4>(y, w, x, out, in, st);
        else if (nsteps >= 2)
            launch_q4k_t1<2>(y, w, x, out, in, st);
        else
            launch_q4k_t1<1>(y, w, x, out, in, st);
    } else {
        k_gemv_q4k<kR, NT, 1><<<(out + kR - 1) / kR, kWarps * 32, 0, st>>>(y, w, x, out, in, nt);
    }
}
template <int NT>
void launch_f16(float* y, const uint16_t* w, const float* x, uint32_t out, uint32_t in, uint32_t nt, cudaStream_t st) {
    k_gemv_f16<kR, NT, NT == 1 ? 2 : 1><<<(out + kR - 1) / kR, kWarps * 32, 0, st>>>(y, w, x, out, in, nt);
}

int gemv_q4k(float* y, const uint8_t* w, const float* x, uint32_t out, uint32_t in, uint32_t B, cudaStream_t st,
             char* err, size_t errlen, const char* who) {
    if (!y || !w || !x || out == 0 || in == 0 || B == 0 || (in % 256) != 0) {
        set_err(err, errlen, "%s: bad args (out=%u in=%u B=%u; in must be a multiple of 256)", who, out, in, B);
        return -1;
    }
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15)) {
        set_err(err, errlen, "%s: x and w must be 16-byte aligned", who);
        return -1;
    }
    // tokens in passes of kNT (one token alone takes the single-token kernel)
    for (uint32_t t0 = 0; t0 < B; t0 += kNT) {
        const uint32_t nt = std::min<uint32_t>(kNT, B - t0);
        float* yt = y + static_cast<size_t>(t0) * out;
        const float* xt = x + static_cast<size_t>(t0) * in;
        if (nt == 1)
            launch_q4k<1>(yt, w, xt, out, in, 1, st);
        else
            launch_q4k<kNT>(yt, w, xt, out, in, nt, st);
    }
    YATTN_CHECK_LAUNCH(err, errlen, who);
    return 0;
}

int gemv_f16(float* y, const uint16_t* w, const float* x, uint32_t out, uint32_t in, uint32_t B, cudaStream_t st,
             char* err, size_t errlen, const char* who) {
    if (!y || !w || !x || out == 0 || in == 0 || B == 0) {
        set_err(err, errlen, "%s: bad args (out=%u in=%u B=%u)", who, out, in, B);
        return -1;
    }
    const bool vec = (in % 8) == 0 && !(reinterpret_cast<uintptr_t>(w) & 15) && !(reinterpret_cast<uintptr_t>(x) & 15);
    for (uint32_t t0 = 0; t0 < B; t0 += kNT) {
        const uint32_t nt = std::min<uint32_t>(kNT, B - t0);
        float* yt = y + static_cast<size_t>(t0) * out;
        const float* xt = x + static_cast<size_t>(t0) * in;
        if (!vec)
            k_gemv_f16_any<<<(out + kWarps - 1) / kWarps, kWarps * 32, 0, st>>>(yt, w, xt, out, in, nt);
        else if (nt == 1)
            launch_f16<1>(yt, w, xt, out, in, 1, st);
        else
            launch_f16<kNT>(yt, w, xt, out, in, nt, st);
    }
    YATTN_CHECK_LAUNCH(err, errlen, who);
    return 0;
}

}  // namespace
}  // namespace yattn

using namespace yattn;

extern "C" int yattn_gemv_q4k(float* y, const uint8_t* w, const float* x, uint32_t out, uint32_t in, uint32_t B,
                              void* stream, char* err, size_t errlen) {
    return gemv_q4k(y, w, x, out, in, B, static_cast<cudaStream_t>(stream), err, errlen, "gemv_q4k");
}

extern "C" int yattn_gemv_f16(float* y, const uint16_t* w, const float* x, uint32_t out, uint32_t in, uint32_t B,
                              void* stream, char* err, size_t errlen) {
    return gemv_f16(y, w, x, out, in, B, static_cast<cudaStream_t>(stream), err, errlen, "gemv_f16");
}

// ---- drop-ins with the reference's names and signatures (legacy default stream) ----

extern "C" int cuda_k_gemv_q4k(float* y, const uint8_t* w, const float* x, uint32_t out, uint32_t in, char* err,
                               size_t errlen) {
    return gemv_q4k(y, w, x, out, in, 1, nullptr, err, errlen, "gemv_q4k");
}

extern "C" int cuda_k_gemm_q4k(float* y, const uint8_t* w, const float* x, uint32_t out, uint32_t in, uint32_t B,
                               char* err, size_t errlen) {
    return gemv_q4k(y, w, x, out, in, B, nullptr, err, errlen, "gemm_q4k");
}

// cublas / xf16 are accepted for the signature and not used: x stays fp32.
extern "C" int cuda_k_gemv_f16(void* cublas, float* y, const uint16_t* w, const float* x, uint16_t* xf16,
                               uint32_t out, uint32_t in, char* err, size_t errlen) {
    (void)cublas;
    (void)xf16;
    return gemv_f16(y, w, x, out, in, 1, nullptr, err, errlen, "gemv_f16");
}

extern "C" int cuda_k_gemm_f16(void* cublas, float* y, const uint16_t* w, const float* x, uint16_t* xf16,
                               uint32_t out, uint32_t in, uint32_t B, char* err, size_t errlen) {
    (void)cublas;
    (void)xf16;
    return gemv_f16(y, w, x, out, in, B, nullptr, err, errlen, "gemm_f16");
}
