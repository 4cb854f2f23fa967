// gdn_inputs.cu -- the qwen35 GDN layer's input preparation, between the
// projections and the state update, for T tokens of many sequences.
//
// Reference, per token (engine.c:785-821): the gates, beta = sigmoid(beta_in)
// and gate = softplus(alpha + dt) * A (engine.c:787-793); the causal
// depthwise conv1d over a kwidth-row delay line (conv1d_update,
// matvec.c:956-967) followed by silu (engine.c:812); the split into q, k, v and
// l2norm_inplace (matvec.c:941-948) of every q and k head (engine.c:815-821).
// The engine does this one token at a time; here every token of a chunk is
// independent once the delay line is read, so one launch covers all tokens.
//
// Arithmetic follows the reference's fp32 operation order without FMA
// contraction (the reference is built as C99): the conv sums its taps oldest
// first, l2norm sums squares in index order (one thread per row, from shared
// memory), and the gates' and l2norm's divisions and square roots are
// IEEE-rounded.  The silu of every channel uses the device's fast exponential
// and division (its per-element cost bounds the launch), a few ulps from the
// host's; the gates use expf and log1pf.
#include "common.cuh"

#include <algorithm>

namespace yattn {
namespace {

constexpr int kThreads = 256;      // most channels of one head segment (head dims up to 256)
constexpr int kMaxKw = 8;          // conv taps held in registers
// Tokens per block: 32 for chunks, 8 for short ones (a decode step).  At least kMaxKw - 1, so only the first
// tile reads the delay line that the first tile also rewrites.
constexpr int kTTLong = 32, kTTShort = 8;
static_assert(kTTShort >= kMaxKw - 1, "a tile must cover the delay line");

struct InParams {
    const float* qkv;              // [n_seqs][T][conv_chan]
    float* conv_state;             // [n_seqs][kw][conv_chan], updated
    const float* conv_w;           // [conv_chan][kw]
    const float* alpha;            // [n_seqs][T][nv]
    const float* beta_in;          // [n_seqs][T][nv]
    const float* dt;               // [nv]
    const float* a;                // [nv]
    float* q;                      // [n_seqs][T][nk*hk]
    float* k;                      // [n_seqs][T][nk*hk]
    float* v;                      // [n_seqs][T][nv*hv]
    float* gate;                   // [n_seqs][T][nv]
    float* beta;                   // [n_seqs][T][nv]
    uint32_t T, conv_chan, kw, nk, hk, nv, hv;
    float eps;
};

// Segment s of a block: q head s (s < nk), k head s - nk (s < 2nk), v head s - 2nk (s < 2nk + nv), else the
// gates of the block's tokens.  KW = conv taps (the delay line's rows), kTT = tokens per block.  One thread
// per channel of a segment (blockDim = the wider head dim rounded to a warp).
template <int KW, int kTT>
__global__ void __launch_bounds__(kThreads) k_gdn_inputs(const InParams p) {
    __shared__ float rows[kTT][kThreads + 1];   // silu outputs of a q/k segment, +1 column against bank conflicts
    __shared__ float scale[kTT];
    const uint32_t seg = blockIdx.x, sq = blockIdx.z;
    const uint32_t t0 = blockIdx.y * kTT;
    const uint32_t nt = min(static_cast<uint32_t>(kTT), p.T - t0);
    const uint32_t key_dim = p.nk * p.hk, value_dim = p.nv * p.hv;
    const size_t tok0 = static_cast<size_t>(sq) * p.T + t0;    // row of token t0 in the [n_seqs][T] arrays
    const uint32_t tid = threadIdx.x;

    if (seg == 2 * p.nk + p.nv) {   // gates (engine.c:787-793)
        for (uint32_t u = tid; u < nt * p.nv; u += blockDim.x) {
            const uint32_t t = u / p.nv, h = u % p.nv;
            const size_t i = (tok0 + t) * p.nv + h;
            p.beta[i] = 1.0f / __fadd_rn(1.0f, expf(-p.beta_in[i]));
            const float ab = __fadd_rn(p.alpha[i], p.dt[h]);
            p.gate[i] = __fmul_rn(log1pf(expf(ab)), p.a[h]);
        }
        return;
    }
    const bool is_q = seg < p.nk, is_k = !is_q && seg < 2 * p.nk;
    const uint32_t seg_len = (is_q || is_k) ? p.hk : p.hv;
    const uint32_t ch0 = is_q ? seg * p.hk : is_k ? key_dim + (seg - p.nk) * p.hk
                                                 : 2 * key_dim + (seg - 2 * p.nk) * p.hv;
    constexpr uint32_t kw = KW;
    if (tid < seg_len) {
        const uint32_t ch = ch0 + tid;
        const float* xs = p.qkv + static_cast<size_t>(sq) * p.T * p.conv_chan + ch;   // token t at xs[t*conv_chan]
        float* st = p.conv_state + static_cast<size_t>(sq) * kw * p.conv_chan + ch;   // row i at st[i*conv_chan]
        float w[KW], win[KW];
#pragma unroll
        for (int i = 0; i < KW; ++i) w[i] = p.conv_w[static_cast<size_t>(ch) * kw + i];
        // delay line before token t0: win[i] = input of token t0 - (kw - 1) + i, i < kw - 1; tokens before the
        // chunk come from the state (row kw - 1 is the newest)
#pragma unroll
        for (int i = 0; i < KW - 1; ++i) {
            const int64_t j = static_cast<int64_t>(t0) - (KW - 1) + i;
            win[i] = j >= 0 ? xs[static_cast<size_t>(j) * p.conv_chan]
                            : st[static_cast<size_t>(static_cast<int64_t>(KW) + j) * p.conv_chan];
        }
        // every input of the tile in flight at once (the stores below could alias them for the compiler)
        float xv[kTT];
#pragma unroll
        for (int t = 0; t < kTT; ++t) xv[t] = t < static_cast<int>(nt) ? xs[static_cast<size_t>(t0 + t) * p.conv_chan] : 0.f;
        float* vout = p.v + tok0 * value_dim + (ch0 - 2 * key_dim) + tid;
        float fin[KW];   // the window at the tile's last token: the delay line after it
#pragma unroll
        for (int t = 0; t < kTT; ++t) {
            if (t < static_cast<int>(nt)) {
                win[KW - 1] = xv[t];
                if (t == static_cast<int>(nt) - 1) {
#pragma unroll
                    for (int i = 0; i < KW; ++i) fin[i] = win[i];
                }
                float acc = 0.0f;   // conv1d_update: taps oldest first
#pragma unroll
                for (int i = 0; i < KW; ++i) acc = __fadd_rn(acc, __fmul_rn(win[i], w[i]));
                // silu with the fast exponential and division (the per-element cost of this launch): a few ulps
                // from the reference's expf and IEEE division, far inside the tolerance of the layer
                const float y = __fdividef(acc, __fadd_rn(1.0f, __expf(-acc)));
                if (is_q || is_k)
                    rows[t][tid] = y;
                else
                    vout[static_cast<size_t>(t) * value_dim] = y;
#pragma unroll
                for (int i = 0; i < KW - 1; ++i) win[i] = win[i + 1];
            }
        }
        if (blockIdx.y == 0) {
            // the delay line after the last token: row i = input of token T - kw + i.  Only this thread touches
            // column ch of the state, and only blocks of the first tile read it, so read everything first.  With
            // one tile the window already holds it.
            if (gridDim.y > 1) {
#pragma unroll
                for (int i = 0; i < KW; ++i) fin[i] = xs[static_cast<size_t>(p.T - KW + i) * p.conv_chan];
            }
#pragma unroll
            for (int i = 0; i < KW; ++i) st[static_cast<size_t>(i) * p.conv_chan] = fin[i];
        }
    }
    if (!(is_q || is_k)) return;
    __syncthreads();
    if (tid < nt) {   // l2norm_inplace: squares summed in index order
        float s = 0.0f;
#pragma unroll 8
        for (uint32_t c = 0; c < seg_len; ++c) s = __fadd_rn(s, __fmul_rn(rows[tid][c], rows[tid][c]));
        scale[tid] = 1.0f / fmaxf(sqrtf(s), p.eps);
    }
    __syncthreads();
    float* out = (is_q ? p.q : p.k) + tok0 * key_dim + (is_q ? ch0 : ch0 - key_dim);
    if (tid < seg_len) {   // one channel per thread, token by token (coalesced rows, no index division)
        for (uint32_t t = 0; t < nt; ++t)
            out[static_cast<size_t>(t) * key_dim + tid] = __fmul_rn(rows[t][tid], scale[t]);
    }
}

}  // namespace
}  // namespace yattn

using namespace yattn;

extern "C" int yattn_gdn_inputs(const float* qkv, float* conv_state, const float* conv_w, const float* alpha,
                                const float* beta_in, const float* ssm_dt, const float* ssm_a, float* q, float* k,
                                float* v, float* gate, float* beta, uint32_t n_seqs, uint32_t T, uint32_t conv_chan,
                                uint32_t kwidth, uint32_t num_k_heads, uint32_t hk, uint32_t n_vheads, uint32_t hv,
                                float eps, void* stream, char* err, size_t errlen) {
    if (n_seqs == 0 || T == 0) return 0;
    if (!qkv || !conv_state || !conv_w || !alpha || !beta_in || !ssm_dt || !ssm_a || !q || !k || !v || !gate ||
        !beta) {
        set_err(err, errlen, "gdn_inputs: null pointer");
        return -1;
    }
    if (num_k_heads == 0 || n_vheads == 0 || hk == 0 || hv == 0 || hk > kThreads || hv > kThreads ||
        static_cast<uint64_t>(2) * num_k_heads * hk + static_cast<uint64_t>(n_vheads) * hv != conv_chan) {
        set_err(err, errlen, "gdn_inputs: conv_chan %u != 2*%u*%u + %u*%u (head dims up to %d)", conv_chan,
                num_k_heads, hk, n_vheads, hv, kThreads);
        return -1;
    }
    if (kwidth == 0 || kwidth > static_cast<uint32_t>(kMaxKw)) {
        set_err(err, errlen, "gdn_inputs: kwidth %u (1..%d)", kwidth, kMaxKw);
        return -1;
    }
    const bool long_tiles = T >= 64;
    const uint32_t tt = long_tiles ? kTTLong : kTTShort;
    const uint32_t tiles = (T + tt - 1) / tt;
    const uint32_t segs = 2 * num_k_heads + n_vheads + 1;
    if (tiles > 65535 || n_seqs > 65535 || segs > 0x7FFFFFFFu) {
        set_err(err, errlen, "gdn_inputs: grid too large (T=%u, n_seqs=%u)", T, n_seqs);
        return -1;
    }
    InParams p{qkv, conv_state, conv_w, alpha, beta_in, ssm_dt, ssm_a, q, k, v, gate, beta,
               T, conv_chan, kwidth, num_k_heads, hk, n_vheads, hv, eps};
    const dim3 grid(segs, tiles, n_seqs);
    const uint32_t threads = (std::max(hk, hv) + 31) / 32 * 32;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
#define YATTN_GDN_IN(KW)                                                                    \
    (long_tiles ? k_gdn_inputs<KW, kTTLong><<<grid, threads, 0, st>>>(p)                    \
                : k_gdn_inputs<KW, kTTShort><<<grid, threads, 0, st>>>(p))
    switch (kwidth) {
        case 1: YATTN_GDN_IN(1); break;
        case 2: YATTN_GDN_IN(2); break;
        case 3: YATTN_GDN_IN(3); break;
        case 4: YATTN_GDN_IN(4); break;
        case 5: YATTN_GDN_IN(5); break;
        case 6: YATTN_GDN_IN(6); break;
        case 7: YATTN_GDN_IN(7); break;
        default: YATTN_GDN_IN(8); break;
    }
#undef YATTN_GDN_IN
    YATTN_CHECK_LAUNCH(err, errlen, "gdn_inputs");
    return 0;
}
