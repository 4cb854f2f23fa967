// decode.cu -- GQA decode attention over the fp16 KV cache (sm_100a).
//
// Reference semantics: engine.c:1074-1096 (CPU loop) and the reference GPU
// kernel k_attn_flash_decode (inference/cuda/cuda_kernels.cu:543-600): for
// query head hh, kv head hh*n_kv/n_heads, scores q.k_t / sqrt(d) over t=0..pos,
// softmax, out = sum p_t v_t.
//
// Design (B200): one CTA = one (item, kv_head, key split).
//   * warp 4 (producer) streams the split's K and V rows into a 4-stage shared
//     memory ring with cp.async.bulk (TMA, non-tensor) completing on mbarriers;
//   * warps 0-3 (consumers) each take 8 of the 32 tokens of a stage.  The kv
//     head's query group (<= 8 heads) sits in registers, each lane owning
//     head_dim/32 dims.  Per-lane partial dot products for (token, head) pairs
//     are summed across the warp with a transpose-reduce (31 shuffles per 32
//     sums, lane l ends with sum l), the online softmax runs in the log2
//     domain, and p.V accumulates in registers with packed fp32 FMAs;
//   * the 4 warps' (m, l, o) are merged in shared memory; a split writes its
//     partial to the workspace and the last split of a (item, kv_head) to
//     arrive (atomic counter) merges all splits with log-sum-exp weights.
// All math is fp32 (fp16 K/V converted exactly), like the reference.
#include "common.cuh"

#include <algorithm>
#include <mutex>
#include <vector>

namespace yattn {
namespace {

constexpr int kTok = 32;            // tokens per stage
constexpr int kConsumers = 4;       // consumer warps
constexpr int kThreads = 32 * (kConsumers + 1);

template <int HD> struct DecodeCfg {
    static constexpr int DPL = HD / 32;                    // dims per lane
    static constexpr int ROWB = HD * 2;                    // bytes of one K (or V) row slice
    static constexpr int NST = (HD >= 256) ? 3 : 4;        // pipeline stages
    static constexpr int STAGEB = 2 * kTok * ROWB;         // K tile + V tile
};

struct DecodeParams {
    const YattnDecodeItem* items;
    const YattnDecodeWork* work;      // nullptr: single item, uniform splits (see below)
    YattnDecodeItem item0;            // used when work == nullptr
    uint32_t split_len;               // uniform split length when work == nullptr
    uint32_t n_splits0;               // splits per kv head when work == nullptr
    uint32_t t_base;                  // key offset when work == nullptr
    uint32_t t_end0;                  // end key (exclusive) when work == nullptr
    uint32_t n_heads, n_kv, kv_dim;
    float scale_log2;                 // log2(e) / sqrt(head_dim)
    float* part_ml;                   // [n_parts][G][2]
    float* part_o;                    // [n_parts][G][HD]
    uint32_t* counters;               // [n_groups]
    int* status;
    int partial_only;                 // write (m,l,o) for the whole work unit, never merge
    float* out_ml;                    // partial_only: [n_heads][2]
    float* out_o;                     // partial_only: [n_heads][HD]
};

__device__ __forceinline__ void group_of(uint32_t kvh, uint32_t n_heads, uint32_t n_kv, uint32_t& first,
                                         uint32_t& cnt) {
    // heads hh with hh*n_kv/n_heads == kvh: ceil(kvh*n_heads/n_kv) .. ceil((kvh+1)*n_heads/n_kv)-1
    uint32_t a = (kvh * n_heads + n_kv - 1) / n_kv;
    uint32_t b = ((kvh + 1) * n_heads + n_kv - 1) / n_kv;
    first = a;
    cnt = b - a;
}

template <int V>
__device__ __forceinline__ void transpose_reduce(float (&a)[V], int lane) {
    // Sum a[i] over the warp; afterwards a[0] holds sum #(lane >> (5 - log2 V))
    // for V <= 32 (replicated over the low lanes).
    static_assert(V == 8 || V == 16 || V == 32, "V");
    constexpr int LOGV = (V == 8) ? 3 : (V == 16) ? 4 : 5;
    int c = V;
#pragma unroll
    for (int step = 0; step < LOGV; ++step) {
        const int off = 16 >> step;
        const bool up = (lane & off) != 0;
        c >>= 1;
#pragma unroll
        for (int j = 0; j < V / 2; ++j) {
            if (j < c) {
                float send = up ? a[j] : a[j + c];
                float keep = up ? a[j + c] : a[j];
                a[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
        }
    }
#pragma unroll
    for (int off = 16 >> LOGV; off >= 1; off >>= 1) a[0] += __shfl_xor_sync(0xffffffffu, a[0], off);
}

template <int HD, int G>
__global__ void __launch_bounds__(kThreads, 2) k_decode(const DecodeParams p) {
    using C = DecodeCfg<HD>;
    constexpr int DPL = C::DPL;
    constexpr int GP = (G <= 1) ? 1 : (G <= 2) ? 2 : (G <= 4) ? 4 : 8;   // padded group
    constexpr int TR = (GP == 8) ? 4 : 8;                                 // tokens per reduce round
    constexpr int NR = 8 / TR;                                            // rounds per warp share
    constexpr int V = TR * GP;                                            // values per lane per round
    constexpr int REP = (V < 32) ? ((V == 16) ? 1 : 2) : 0;               // replicated low lane bits
    constexpr int TB = ((GP == 1) ? 0 : (GP == 2) ? 1 : (GP == 4) ? 2 : 3) + REP;   // first token bit

    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* stages = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::NST * C::STAGEB);
    uint64_t* empty = full + C::NST;
    float* sp = reinterpret_cast<float*>(empty + C::NST);       // [4][32] probabilities
    float* salpha = sp + kConsumers * 32;                        // [4][8]
    float* mrg_ml = salpha + kConsumers * 8;                     // [4][G][2]
    volatile int* abort_flag = reinterpret_cast<volatile int*>(mrg_ml + kConsumers * G * 2);
    int* last_flag = const_cast<int*>(abort_flag) + 1;
    float* mrg_o = reinterpret_cast<float*>(stages);             // [4][G][HD], aliases the ring after use

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // ---- work unit ----
    YattnDecodeItem it;
    uint32_t kvh, t0, t1, n_splits, split, part_base, group;
    if (p.work) {
        const YattnDecodeWork w = p.work[blockIdx.x];
        it = p.items[w.item];
        kvh = w.kv_head;
        t0 = w.t_begin;
        t1 = w.t_end;
        n_splits = w.n_splits;
        split = w.split;
        part_base = w.part_base;
        group = w.group;
    } else {
        it = p.item0;
        kvh = blockIdx.x / p.n_splits0;
        split = blockIdx.x % p.n_splits0;
        n_splits = p.n_splits0;
        t0 = p.t_base + split * p.split_len;
        t1 = min(t0 + p.split_len, p.t_end0);
        part_base = kvh * p.n_splits0;
        group = kvh;
    }
    uint32_t gfirst, gcnt;
    group_of(kvh, p.n_heads, p.n_kv, gfirst, gcnt);
    const uint32_t ntok = t1 - t0;
    const uint32_t ntiles = (ntok + kTok - 1) / kTok;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::NST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumers);
        }
        abort_flag[0] = 0;
        last_flag[0] = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumers) {
        // ================= producer =================
        const uint16_t* kb = it.k + static_cast<size_t>(kvh) * HD;
        const uint16_t* vb = it.v + static_cast<size_t>(kvh) * HD;
        uint32_t issued = 0;
        for (uint32_t i = 0; i < ntiles; ++i) {
            const int s = i % C::NST;
            if (i >= static_cast<uint32_t>(C::NST)) {
                if (!warp_wait_bounded(&empty[s], ((i / C::NST) & 1u) ^ 1u, p.status, ST_DECODE_EMPTY_TIMEOUT,
                                       abort_flag))
                    break;
            }
            const uint32_t tile0 = t0 + i * kTok;
            const uint32_t nrows = min(static_cast<uint32_t>(kTok), t1 - tile0);
            uint8_t* kdst = stages + s * C::STAGEB;
            uint8_t* vdst = kdst + kTok * C::ROWB;
            if (lane == 0) mbar_arrive_expect_tx(&full[s], 2u * nrows * C::ROWB);
            __syncwarp();
            for (uint32_t r = lane; r < nrows; r += 32) {
                const size_t off = static_cast<size_t>(tile0 + r) * p.kv_dim;
                bulk_g2s(kdst + r * C::ROWB, kb + off, C::ROWB, &full[s]);
                bulk_g2s(vdst + r * C::ROWB, vb + off, C::ROWB, &full[s]);
            }
            issued = i + 1;
        }
        // Never leave with copies in flight: wait (bounded) for the last stages issued.
        for (uint32_t i = (issued > static_cast<uint32_t>(C::NST) ? issued - C::NST : 0); i < issued; ++i) {
            volatile int dummy = 0;
            mbar_wait_bounded(&full[i % C::NST], (i / C::NST) & 1u, p.status, ST_DECODE_FULL_TIMEOUT, &dummy);
        }
        return;
    }

    // ================= consumers =================
    // query group in registers: lane owns dims [lane*DPL, lane*DPL + DPL)
    float qr[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int d = 0; d < DPL; ++d) qr[g][d] = 0.f;
        if (static_cast<uint32_t>(g) < gcnt) {
            const float* qh = it.q + static_cast<size_t>(gfirst + g) * HD + lane * DPL;
            if constexpr (DPL == 4) {
                float4 t = *reinterpret_cast<const float4*>(qh);
                qr[g][0] = t.x; qr[g][1] = t.y; qr[g][2] = t.z; qr[g][3] = t.w;
            } else if constexpr (DPL == 8) {
                float4 t0v = *reinterpret_cast<const float4*>(qh);
                float4 t1v = *reinterpret_cast<const float4*>(qh + 4);
                qr[g][0] = t0v.x; qr[g][1] = t0v.y; qr[g][2] = t0v.z; qr[g][3] = t0v.w;
                qr[g][4] = t1v.x; qr[g][5] = t1v.y; qr[g][6] = t1v.z; qr[g][7] = t1v.w;
            } else {
                float2 t = *reinterpret_cast<const float2*>(qh);
                qr[g][0] = t.x; qr[g][1] = t.y;
            }
        }
    }
    float oacc[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int d = 0; d < DPL; ++d) oacc[g][d] = 0.f;

    // this lane's (token, head) slot after the transpose-reduce
    const int idx = lane >> REP;
    const int my_t = idx / GP;
    const int my_g = idx % GP;
    float m_mine = -INFINITY, l_mine = 0.f;
    float* spw = sp + warp * 32;
    float* saw = salpha + warp * 8;

    for (uint32_t i = 0; i < ntiles; ++i) {
        const int s = i % C::NST;
        if (!warp_wait_bounded(&full[s], (i / C::NST) & 1u, p.status, ST_DECODE_FULL_TIMEOUT, abort_flag)) break;
        const uint32_t nrows = min(static_cast<uint32_t>(kTok), t1 - (t0 + i * kTok));
        const int nvalid = max(0, min(8, static_cast<int>(nrows) - warp * 8));
        const uint8_t* kt = stages + s * C::STAGEB + warp * 8 * C::ROWB;
        const uint8_t* vt = kt + kTok * C::ROWB;
#pragma unroll
        for (int rr = 0; rr < NR; ++rr) {
            const int nv = min(TR, nvalid - rr * TR);
            if (nv <= 0) break;
            // ---- partial scores for TR tokens x GP heads ----
            float part[V];
#pragma unroll
            for (int t = 0; t < TR; ++t) {
                const uint8_t* row = kt + (rr * TR + t) * C::ROWB + lane * DPL * 2;
                float kf[DPL];
                if constexpr (DPL == 4) {
                    uint2 raw = *reinterpret_cast<const uint2*>(row);
                    float2 a = h2f2(raw.x), b = h2f2(raw.y);
                    kf[0] = a.x; kf[1] = a.y; kf[2] = b.x; kf[3] = b.y;
                } else if constexpr (DPL == 8) {
                    uint4 raw = *reinterpret_cast<const uint4*>(row);
                    float2 a = h2f2(raw.x), b = h2f2(raw.y), c = h2f2(raw.z), d = h2f2(raw.w);
                    kf[0] = a.x; kf[1] = a.y; kf[2] = b.x; kf[3] = b.y;
                    kf[4] = c.x; kf[5] = c.y; kf[6] = d.x; kf[7] = d.y;
                } else {
                    uint32_t raw = *reinterpret_cast<const uint32_t*>(row);
                    float2 a = h2f2(raw);
                    kf[0] = a.x; kf[1] = a.y;
                }
#pragma unroll
                for (int g = 0; g < GP; ++g) {
                    float acc = 0.f;
                    if (g < G) {
                        float2 a2 = make_float2(0.f, 0.f);
#pragma unroll
                        for (int d = 0; d < DPL; d += 2)
                            a2 = __ffma2_rn(make_float2(qr[g][d], qr[g][d + 1]), make_float2(kf[d], kf[d + 1]), a2);
                        acc = a2.x + a2.y;
                    }
                    part[t * GP + g] = acc;
                }
            }
            transpose_reduce<V>(part, lane);
            // ---- online softmax for this lane's (token, head) ----
            const bool valid = my_t < nv;
            const float sc = valid ? part[0] * p.scale_log2 : -INFINITY;
            float tmax = sc;
#pragma unroll
            for (int b = TB; b < 5; ++b) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1 << b));
            const float m_new = fmaxf(m_mine, tmax);
            const float pv = ex2_approx(sc - m_new);
            const float alpha = ex2_approx(m_mine - m_new);
            float psum = pv;
#pragma unroll
            for (int b = TB; b < 5; ++b) psum += __shfl_xor_sync(0xffffffffu, psum, 1 << b);
            l_mine = l_mine * alpha + psum;
            m_mine = m_new;
            spw[idx] = pv;
            if (my_t == 0) saw[my_g] = alpha;
            __syncwarp();
            // ---- rescale and accumulate p.V ----
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float a = saw[g];
#pragma unroll
                for (int d = 0; d < DPL; ++d) oacc[g][d] *= a;
            }
            for (int t = 0; t < nv; ++t) {
                const uint8_t* row = vt + (rr * TR + t) * C::ROWB + lane * DPL * 2;
                float vf[DPL];
                if constexpr (DPL == 4) {
                    uint2 raw = *reinterpret_cast<const uint2*>(row);
                    float2 a = h2f2(raw.x), b = h2f2(raw.y);
                    vf[0] = a.x; vf[1] = a.y; vf[2] = b.x; vf[3] = b.y;
                } else if constexpr (DPL == 8) {
                    uint4 raw = *reinterpret_cast<const uint4*>(row);
                    float2 a = h2f2(raw.x), b = h2f2(raw.y), c = h2f2(raw.z), d = h2f2(raw.w);
                    vf[0] = a.x; vf[1] = a.y; vf[2] = b.x; vf[3] = b.y;
                    vf[4] = c.x; vf[5] = c.y; vf[6] = d.x; vf[7] = d.y;
                } else {
                    uint32_t raw = *reinterpret_cast<const uint32_t*>(row);
                    float2 a = h2f2(raw);
                    vf[0] = a.x; vf[1] = a.y;
                }
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float pg = spw[t * GP + g];
                    const float2 p2 = make_float2(pg, pg);
#pragma unroll
                    for (int d = 0; d < DPL; d += 2) {
                        float2 r = __ffma2_rn(p2, make_float2(vf[d], vf[d + 1]), make_float2(oacc[g][d], oacc[g][d + 1]));
                        oacc[g][d] = r.x;
                        oacc[g][d + 1] = r.y;
                    }
                }
            }
            __syncwarp();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---- merge the 4 consumer warps (ring is free: every stage was consumed) ----
    named_bar_sync(1, 32 * kConsumers);
    if (abort_flag[0]) return;
    if (my_t == 0 && (lane & ((1 << REP) - 1)) == 0 && my_g < G) {
        mrg_ml[(warp * G + my_g) * 2 + 0] = m_mine;
        mrg_ml[(warp * G + my_g) * 2 + 1] = l_mine;
    }
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int d = 0; d < DPL; ++d) mrg_o[(warp * G + g) * HD + lane * DPL + d] = oacc[g][d];
    named_bar_sync(1, 32 * kConsumers);

    const int tid = threadIdx.x;   // 0..127
    const bool single = (n_splits == 1) && !p.partial_only;
    for (int e = tid; e < static_cast<int>(gcnt) * HD; e += 32 * kConsumers) {
        const int g = e / HD, d = e % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kConsumers; ++w) M = fmaxf(M, mrg_ml[(w * G + g) * 2]);
        float o = 0.f, l = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumers; ++w) {
            const float mw = mrg_ml[(w * G + g) * 2];
            const float sc = (mw == -INFINITY) ? 0.f : ex2_approx(mw - M);
            o += sc * mrg_o[(w * G + g) * HD + d];
            l += sc * mrg_ml[(w * G + g) * 2 + 1];
        }
        const uint32_t hh = gfirst + g;
        if (single) {
            float r = o / l;
            if (it.gate) r *= 1.0f / (1.0f + __expf(-it.gate[static_cast<size_t>(hh) * HD + d]));
            it.out[static_cast<size_t>(hh) * HD + d] = r;
        } else if (p.partial_only) {
            p.out_o[static_cast<size_t>(hh) * HD + d] = o;
            if (d == 0) {
                p.out_ml[hh * 2 + 0] = M;
                p.out_ml[hh * 2 + 1] = l;
            }
        } else {
            const size_t slot = static_cast<size_t>(part_base + split) * G + g;
            p.part_o[slot * HD + d] = o;
            if (d == 0) {
                p.part_ml[slot * 2 + 0] = M;
                p.part_ml[slot * 2 + 1] = l;
            }
        }
    }
    if (single || p.partial_only) return;

    // ---- last split of this (item, kv_head) merges all splits ----
    __threadfence();
    named_bar_sync(1, 32 * kConsumers);
    if (tid == 0) {
        const uint32_t prev = atomicAdd(&p.counters[group], 1u);
        last_flag[0] = (prev == n_splits - 1) ? 1 : 0;
    }
    named_bar_sync(1, 32 * kConsumers);
    if (!last_flag[0]) return;
    __threadfence();
    for (int e = tid; e < static_cast<int>(gcnt) * HD; e += 32 * kConsumers) {
        const int g = e / HD, d = e % HD;
        float M = -INFINITY;
        for (uint32_t sidx = 0; sidx < n_splits; ++sidx)
            M = fmaxf(M, __ldcg(&p.part_ml[(static_cast<size_t>(part_base + sidx) * G + g) * 2]));
        float o = 0.f, l = 0.f;
        for (uint32_t sidx = 0; sidx < n_splits; ++sidx) {
            const size_t slot = static_cast<size_t>(part_base + sidx) * G + g;
            const float sc = ex2_approx(__ldcg(&p.part_ml[slot * 2]) - M);
            o += sc * __ldcg(&p.part_o[slot * HD + d]);
            l += sc * __ldcg(&p.part_ml[slot * 2 + 1]);
        }
        const uint32_t hh = gfirst + g;
        float r = o / l;
        if (it.gate) r *= 1.0f / (1.0f + __expf(-it.gate[static_cast<size_t>(hh) * HD + d]));
        it.out[static_cast<size_t>(hh) * HD + d] = r;
    }
    if (tid == 0) p.counters[group] = 0u;   // ready for the next launch
}

// ---------------------------------------------------------------- merge kernel
__global__ void k_merge_partials(float* out, const float* ml, const float* o, uint32_t n_parts, uint32_t n_heads,
                                 uint32_t hd, const float* gate) {
    const uint32_t hh = blockIdx.x;
    for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x) {
        float M = -INFINITY;
        for (uint32_t s = 0; s < n_parts; ++s) {
            const float l = ml[(static_cast<size_t>(s) * n_heads + hh) * 2 + 1];
            if (l > 0.f) M = fmaxf(M, ml[(static_cast<size_t>(s) * n_heads + hh) * 2]);
        }
        float acc = 0.f, l = 0.f;
        for (uint32_t s = 0; s < n_parts; ++s) {
            const size_t slot = static_cast<size_t>(s) * n_heads + hh;
            const float ls = ml[slot * 2 + 1];
            if (!(ls > 0.f)) continue;
            const float sc = ex2_approx(ml[slot * 2] - M);
            acc += sc * o[slot * hd + d];
            l += sc * ls;
        }
        float r = acc / l;
        if (gate) r *= 1.0f / (1.0f + __expf(-gate[static_cast<size_t>(hh) * hd + d]));
        out[static_cast<size_t>(hh) * hd + d] = r;
    }
}

// ------------------------------------------------------------------ dispatch
template <int HD, int G>
int launch_t(const DecodeParams& p, uint32_t grid, cudaStream_t st, char* err, size_t errlen) {
    using C = DecodeCfg<HD>;
    const size_t smem = C::NST * C::STAGEB + 2 * C::NST * 8 + (kConsumers * 32 + kConsumers * 8) * 4 +
                        kConsumers * G * 2 * 4 + 16;
    static_assert(C::NST * C::STAGEB >= kConsumers * G * HD * 4, "merge area must fit in the ring");
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(k_decode<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) {
            set_err(err, errlen, "decode: smem attribute: %s", cudaGetErrorString(e));
            return -1;
        }
        attr_done[dev] = true;
    }
    k_decode<HD, G><<<grid, kThreads, smem, st>>>(p);
    YATTN_CHECK_LAUNCH(err, errlen, "decode");
    return 0;
}

template <int HD>
int launch_hd(const DecodeParams& p, uint32_t gmax, uint32_t grid, cudaStream_t st, char* err, size_t errlen) {
    switch (gmax) {
        case 1: return launch_t<HD, 1>(p, grid, st, err, errlen);
        case 2: return launch_t<HD, 2>(p, grid, st, err, errlen);
        case 3: return launch_t<HD, 3>(p, grid, st, err, errlen);
        case 4: return launch_t<HD, 4>(p, grid, st, err, errlen);
        case 5: return launch_t<HD, 5>(p, grid, st, err, errlen);
        case 6: return launch_t<HD, 6>(p, grid, st, err, errlen);
        case 7: return launch_t<HD, 7>(p, grid, st, err, errlen);
        case 8: return launch_t<HD, 8>(p, grid, st, err, errlen);
        default: set_err(err, errlen, "decode: %u query heads per kv head (max 8)", gmax); return -1;
    }
}

int launch_decode(const DecodeParams& p, uint32_t head_dim, uint32_t grid, cudaStream_t st, char* err,
                  size_t errlen) {
    const uint32_t gmax = (p.n_heads + p.n_kv - 1) / p.n_kv;
    switch (head_dim) {
        case 64: return launch_hd<64>(p, gmax, grid, st, err, errlen);
        case 128: return launch_hd<128>(p, gmax, grid, st, err, errlen);
        case 256: return launch_hd<256>(p, gmax, grid, st, err, errlen);
        default: set_err(err, errlen, "decode: head_dim %u not supported (64/128/256)", head_dim); return -1;
    }
}

int check_geom(uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t kv_dim, char* err, size_t errlen) {
    if (n_heads == 0 || n_kv == 0 || n_kv > n_heads) {
        set_err(err, errlen, "decode: bad head counts n_heads=%u n_kv_heads=%u", n_heads, n_kv);
        return -1;
    }
    if (hd != 64 && hd != 128 && hd != 256) {
        set_err(err, errlen, "decode: head_dim %u not supported (64/128/256)", hd);
        return -1;
    }
    if ((n_heads + n_kv - 1) / n_kv > 8) {
        set_err(err, errlen, "decode: %u query heads per kv head (max 8)", (n_heads + n_kv - 1) / n_kv);
        return -1;
    }
    if (kv_dim < n_kv * hd || (kv_dim % 8) != 0) {
        set_err(err, errlen, "decode: kv_dim %u must be >= n_kv_heads*head_dim and a multiple of 8", kv_dim);
        return -1;
    }
    return 0;
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

uint32_t gmax_of(uint32_t n_heads, uint32_t n_kv) { return (n_heads + n_kv - 1) / n_kv; }

// Uniform split length for `tokens` keys of n_kv heads aiming at `target` CTAs.
uint32_t auto_split(uint64_t token_heads, uint32_t target) {
    uint64_t len = (token_heads + target - 1) / target;
    len = std::max<uint64_t>(len, 128);
    len = (len + kTok - 1) / kTok * kTok;
    return static_cast<uint32_t>(std::min<uint64_t>(len, 1u << 30));
}

size_t ws_bytes_for(uint32_t n_parts, uint32_t n_groups, uint32_t gmax, uint32_t hd) {
    size_t c = (static_cast<size_t>(n_groups) * 4 + 255) / 256 * 256;
    size_t ml = (static_cast<size_t>(n_parts) * gmax * 2 * 4 + 255) / 256 * 256;
    size_t o = static_cast<size_t>(n_parts) * gmax * hd * 4;
    return c + ml + o;
}

void carve_ws(void* ws, uint32_t n_parts, uint32_t n_groups, uint32_t gmax, DecodeParams& p) {
    uint8_t* b = static_cast<uint8_t*>(ws);
    size_t c = (static_cast<size_t>(n_groups) * 4 + 255) / 256 * 256;
    size_t ml = (static_cast<size_t>(n_parts) * gmax * 2 * 4 + 255) / 256 * 256;
    p.counters = reinterpret_cast<uint32_t*>(b);
    p.part_ml = reinterpret_cast<float*>(b + c);
    p.part_o = reinterpret_cast<float*>(b + c + ml);
}

}  // namespace

// Single query, uniform splits, internal or given workspace.  Shared by the
// drop-in decode, yattn_attn_decode and yattn_decode_partial.
int decode_single(float* out, const float* q, const uint16_t* k, const uint16_t* v, const float* gate,
                  uint32_t t_begin, uint32_t t_end, uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t kv_dim,
                  float* partial_ml, float* partial_o, void* ws, size_t ws_bytes, cudaStream_t st, char* err,
                  size_t errlen) {
    if (check_geom(n_heads, n_kv, hd, kv_dim, err, errlen)) return -1;
    if (t_end <= t_begin) {
        set_err(err, errlen, "decode: empty key range [%u, %u)", t_begin, t_end);
        return -1;
    }
    if (!q || !k || !v || (!out && !partial_ml)) {
        set_err(err, errlen, "decode: null pointer argument");
        return -1;
    }
    if (!aligned16(k) || !aligned16(v) || !aligned16(q)) {
        set_err(err, errlen, "decode: q, kcache and vcache must be 16-byte aligned");
        return -1;
    }
    DevCtx* ctx = dev_ctx(err, errlen);
    if (!ctx) return -1;
    const uint32_t gmax = gmax_of(n_heads, n_kv);
    const uint32_t ntok = t_end - t_begin;
    const bool partial_only = partial_ml != nullptr;
    uint32_t split = auto_split(static_cast<uint64_t>(ntok) * n_kv, static_cast<uint32_t>(ctx->num_sms) * 4);
    if (partial_only) split = ntok;   // one work unit per kv head: the partial covers the whole range
    const uint32_t ns = (ntok + split - 1) / split;
    DecodeParams p{};
    p.items = nullptr;
    p.work = nullptr;
    p.item0.q = q;
    p.item0.out = out;
    p.item0.k = k;
    p.item0.v = v;
    p.item0.gate = gate;
    p.item0.pos = t_end - 1;
    p.split_len = split;
    p.n_splits0 = ns;
    p.t_base = t_begin;
    p.t_end0 = t_end;
    p.n_heads = n_heads;
    p.n_kv = n_kv;
    p.kv_dim = kv_dim;
    p.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(hd));
    p.status = ctx->status;
    p.partial_only = partial_only ? 1 : 0;
    p.out_ml = partial_ml;
    p.out_o = partial_o;
    if (ns > 1 && !partial_only) {
        const size_t need = ws_bytes_for(ns * n_kv, n_kv, gmax, hd);
        if (ws) {
            if (ws_bytes < need) {
                set_err(err, errlen, "decode: workspace %zu bytes < %zu needed", ws_bytes, need);
                return -1;
            }
        } else {
            if (ctx->ws_bytes < need) {
                if (ctx->ws) cudaFree(ctx->ws);
                ctx->ws = nullptr;
                ctx->ws_bytes = 0;
                if (cudaMalloc(&ctx->ws, need) != cudaSuccess) {
                    set_err(err, errlen, "decode: cudaMalloc(%zu) of the workspace failed", need);
                    return -1;
                }
                ctx->ws_bytes = need;
                if (cudaMemset(ctx->ws, 0, need) != cudaSuccess) {
                    set_err(err, errlen, "decode: workspace memset failed");
                    return -1;
                }
            }
            ws = ctx->ws;
        }
        carve_ws(ws, ns * n_kv, n_kv, gmax, p);
    }
    return launch_decode(p, hd, ns * n_kv, st, err, errlen);
}

int decode_reserve(size_t bytes, char* err, size_t errlen) {
    DevCtx* ctx = dev_ctx(err, errlen);
    if (!ctx) return -1;
    if (ctx->ws_bytes >= bytes) return 0;
    if (ctx->ws) cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
    if (cudaMalloc(&ctx->ws, bytes) != cudaSuccess || cudaMemset(ctx->ws, 0, bytes) != cudaSuccess) {
        set_err(err, errlen, "reserve: cudaMalloc/cudaMemset(%zu) failed", bytes);
        return -1;
    }
    ctx->ws_bytes = bytes;
    return 0;
}

}  // namespace yattn

using namespace yattn;

extern "C" int yattn_decode_plan(const uint32_t* pos_host, uint32_t n_items, uint32_t n_kv_heads,
                                 uint32_t split_tokens, uint32_t target_ctas, YattnDecodeWork* work_host,
                                 uint32_t work_cap, uint32_t* n_work, uint32_t* n_parts, uint32_t* n_groups,
                                 char* err, size_t errlen) {
    if (!pos_host || !work_host || !n_work || !n_parts || !n_groups || n_kv_heads == 0 || n_kv_heads > 65535) {
        set_err(err, errlen, "decode_plan: bad arguments");
        return -1;
    }
    uint64_t total = 0;
    for (uint32_t i = 0; i < n_items; ++i) total += static_cast<uint64_t>(pos_host[i]) + 1;
    total *= n_kv_heads;
    if (target_ctas == 0) target_ctas = static_cast<uint32_t>(dev_num_sms()) * 4;
    const uint32_t split = split_tokens ? (split_tokens + kTok - 1) / kTok * kTok : auto_split(total, target_ctas);
    std::vector<YattnDecodeWork> w;
    uint32_t parts = 0, groups = 0;
    for (uint32_t i = 0; i < n_items; ++i) {
        const uint32_t ntok = pos_host[i] + 1;
        const uint32_t ns = (ntok + split - 1) / split;
        if (ns > 65535) {
            set_err(err, errlen, "decode_plan: %u splits for item %u (max 65535)", ns, i);
            return -1;
        }
        for (uint32_t h = 0; h < n_kv_heads; ++h) {
            for (uint32_t s = 0; s < ns; ++s) {
                YattnDecodeWork x{};
                x.item = i;
                x.kv_head = static_cast<uint16_t>(h);
                x.n_splits = static_cast<uint16_t>(ns);
                x.split = s;
                x.t_begin = s * split;
                x.t_end = std::min(ntok, (s + 1) * split);
                x.part_base = ns > 1 ? parts : 0u;
                x.group = ns > 1 ? groups : 0u;
                w.push_back(x);
            }
            if (ns > 1) {
                parts += ns;
                groups += 1;
            }
        }
    }
    // longest units first: the tail of the grid is made of the short ones
    std::stable_sort(w.begin(), w.end(), [](const YattnDecodeWork& a, const YattnDecodeWork& b) {
        return (a.t_end - a.t_begin) > (b.t_end - b.t_begin);
    });
    if (w.size() > work_cap) {
        set_err(err, errlen, "decode_plan: %zu work units exceed work_cap %u", w.size(), work_cap);
        *n_work = static_cast<uint32_t>(w.size());
        return -1;
    }
    memcpy(work_host, w.data(), w.size() * sizeof(YattnDecodeWork));
    *n_work = static_cast<uint32_t>(w.size());
    *n_parts = parts;
    *n_groups = groups;
    return 0;
}

extern "C" size_t yattn_decode_workspace_bytes(uint32_t n_parts, uint32_t n_groups, uint32_t n_heads,
                                               uint32_t n_kv_heads, uint32_t head_dim) {
    if (n_kv_heads == 0) return 0;
    return ws_bytes_for(n_parts, n_groups, gmax_of(n_heads, n_kv_heads), head_dim);
}

extern "C" int yattn_decode_workspace_init(void* workspace, size_t ws_bytes, void* stream, char* err,
                                           size_t errlen) {
    if (!workspace) return 0;
    cudaError_t e = cudaMemsetAsync(workspace, 0, ws_bytes, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        set_err(err, errlen, "decode_workspace_init: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

extern "C" int yattn_decode_run(const YattnDecodeItem* items_dev, const YattnDecodeWork* work_dev, uint32_t n_work,
                                uint32_t n_parts, uint32_t n_groups, uint32_t n_heads, uint32_t n_kv_heads,
                                uint32_t head_dim, uint32_t kv_dim, void* workspace, size_t ws_bytes, void* stream,
                                char* err, size_t errlen) {
    if (check_geom(n_heads, n_kv_heads, head_dim, kv_dim, err, errlen)) return -1;
    if (n_work == 0) return 0;
    if (!items_dev || !work_dev) {
        set_err(err, errlen, "decode_run: null items/work");
        return -1;
    }
    const uint32_t gmax = gmax_of(n_heads, n_kv_heads);
    const size_t need = ws_bytes_for(n_parts, n_groups, gmax, head_dim);
    if (n_parts > 0 && (!workspace || ws_bytes < need)) {
        set_err(err, errlen, "decode_run: workspace %zu bytes < %zu needed", ws_bytes, need);
        return -1;
    }
    DevCtx* ctx = dev_ctx(err, errlen);
    if (!ctx) return -1;
    DecodeParams p{};
    p.items = items_dev;
    p.work = work_dev;
    p.n_heads = n_heads;
    p.n_kv = n_kv_heads;
    p.kv_dim = kv_dim;
    p.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(head_dim));
    p.status = ctx->status;
    if (n_parts > 0) carve_ws(workspace, n_parts, n_groups, gmax, p);
    return launch_decode(p, head_dim, n_work, static_cast<cudaStream_t>(stream), err, errlen);
}

extern "C" size_t yattn_decode_partial_workspace_bytes(uint32_t n_tokens, uint32_t n_heads, uint32_t n_kv_heads,
                                                       uint32_t head_dim) {
    (void)n_tokens; (void)n_heads; (void)n_kv_heads; (void)head_dim;
    return 0;   // one work unit per kv head writes straight to ml/o
}

extern "C" int yattn_decode_partial(float* ml, float* o, const float* q, const uint16_t* kcache,
                                    const uint16_t* vcache, uint32_t t_begin, uint32_t t_end, uint32_t n_heads,
                                    uint32_t n_kv_heads, uint32_t head_dim, uint32_t kv_dim, void* workspace,
                                    size_t ws_bytes, void* stream, char* err, size_t errlen) {
    if (!ml || !o) {
        set_err(err, errlen, "decode_partial: null ml/o");
        return -1;
    }
    return decode_single(nullptr, q, kcache, vcache, nullptr, t_begin, t_end, n_heads, n_kv_heads, head_dim,
                         kv_dim, ml, o, workspace, ws_bytes, static_cast<cudaStream_t>(stream), err, errlen);
}

extern "C" int yattn_merge_partials(float* out, const float* ml, const float* o, uint32_t n_parts, uint32_t n_heads,
                                    uint32_t head_dim, const float* gate, void* stream, char* err, size_t errlen) {
    if (!out || !ml || !o || n_parts == 0 || n_heads == 0 || head_dim == 0) {
        set_err(err, errlen, "merge_partials: bad arguments");
        return -1;
    }
    k_merge_partials<<<n_heads, 128, 0, static_cast<cudaStream_t>(stream)>>>(out, ml, o, n_parts, n_heads,
                                                                             head_dim, gate);
    YATTN_CHECK_LAUNCH(err, errlen, "merge_partials");
    return 0;
}

extern "C" int yattn_attn_decode(float* att_out, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                                 const float* gate, uint32_t pos, uint32_t n_heads, uint32_t n_kv_heads,
                                 uint32_t head_dim, uint32_t kv_dim, void* stream, char* err, size_t errlen) {
    return decode_single(att_out, q, kcache, vcache, gate, 0, pos + 1, n_heads, n_kv_heads, head_dim, kv_dim,
                         nullptr, nullptr, nullptr, 0, static_cast<cudaStream_t>(stream), err, errlen);
}

extern "C" int yattn_reserve(size_t bytes, char* err, size_t errlen) { return decode_reserve(bytes, err, errlen); }

extern "C" void cuda_k_attn_decode(float* att_out, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                                   uint32_t pos, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                                   uint32_t kv_dim) {
    char err[256];
    err[0] = 0;
    if (decode_single(att_out, q, kcache, vcache, nullptr, 0, pos + 1, n_heads, n_kv_heads, head_dim, kv_dim,
                      nullptr, nullptr, nullptr, 0, nullptr, err, sizeof(err)) != 0)
        set_last_error(err);
}

// ------------------------------------------------------- allocation-free decode
//
// Some callers cannot call cudaMalloc at the point where they decode: a
// serving loop that runs under a fixed device-memory budget carved out up
// front, a host whose allocator must not be re-entered from the decode thread,
// or a C caller that owns every buffer and has no way to hand the library a
// workspace.  For them, yattn_attn_decode_noalloc keeps the split-KV scratch
// (per-split (m, l, o) partials, the merge counters and a status word) in the
// fixed array below, which every GPU that loads the library holds until exit.
// The array is shared by every call on a device: calls that overlap on the GPU
// (different streams, or host threads) race on it and must be serialised by
// the caller.

namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;   // 4 MiB per device
constexpr size_t kNoAllocHeader = 256;              // status word, then 256-aligned counters + partials

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch, looked up once per device.  In host
// code the symbol itself is only a host-side stand-in, never a device address.
void* g_noalloc_addr[64];
std::mutex g_noalloc_mu;

void* noalloc_scratch(int dev, char* err, size_t errlen) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr) {
            set_err(err, errlen, "decode_noalloc: cudaGetSymbolAddress of the static scratch failed: %s",
                    cudaGetErrorString(e));
            return nullptr;
        }
        g_noalloc_addr[dev] = ptr;
    }
    return g_noalloc_addr[dev];
}

}  // namespace

extern "C" int yattn_attn_decode_noalloc(float* att_out, const float* q, const uint16_t* kcache,
                                         const uint16_t* vcache, const float* gate, uint32_t pos, uint32_t n_heads,
                                         uint32_t n_kv_heads, uint32_t head_dim, uint32_t kv_dim, void* stream,
                                         char* err, size_t errlen) {
    if (check_geom(n_heads, n_kv_heads, head_dim, kv_dim, err, errlen)) return -1;
    if (!att_out || !q || !kcache || !vcache) {
        set_err(err, errlen, "decode_noalloc: null pointer argument");
        return -1;
    }
    if (!aligned16(kcache) || !aligned16(vcache) || !aligned16(q)) {
        set_err(err, errlen, "decode_noalloc: q, kcache and vcache must be 16-byte aligned");
        return -1;
    }
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        set_err(err, errlen, "decode_noalloc: no usable CUDA device");
        return -1;
    }
    // The split schedule is the one yattn_attn_decode uses, so both give the same result.
    const uint32_t ntok = pos + 1;
    const uint32_t gmax = gmax_of(n_heads, n_kv_heads);
    const uint32_t split = auto_split(static_cast<uint64_t>(ntok) * n_kv_heads, static_cast<uint32_t>(dev_num_sms()) * 4);
    const uint32_t ns = (ntok + split - 1) / split;
    const size_t need = ns > 1 ? ws_bytes_for(ns * n_kv_heads, n_kv_heads, gmax, head_dim) : 0;
    if (need > kNoAllocScratchBytes - kNoAllocHeader) {
        set_err(err, errlen,
                "decode_noalloc: this query needs %zu bytes of split-KV scratch, more than the %zu-byte static "
                "scratch (%u splits x %u kv heads x %u q heads x head_dim %u); use yattn_attn_decode",
                need, kNoAllocScratchBytes - kNoAllocHeader, ns, n_kv_heads, gmax, head_dim);
        return -1;
    }
    // First call on a device: looks up the scratch address (no allocation).
    uint8_t* base = static_cast<uint8_t*>(noalloc_scratch(dev, err, errlen));
    if (!base) return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    DecodeParams p{};
    p.item0.q = q;
    p.item0.out = att_out;
    p.item0.k = kcache;
    p.item0.v = vcache;
    p.item0.gate = gate;
    p.item0.pos = pos;
    p.split_len = split;
    p.n_splits0 = ns;
    p.t_base = 0;
    p.t_end0 = ntok;
    p.n_heads = n_heads;
    p.n_kv = n_kv_heads;
    p.kv_dim = kv_dim;
    p.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(head_dim));
    p.status = reinterpret_cast<int*>(base);
    // The array keeps the previous call's contents: the status word and the merge
    // counters must start at zero, the partials are fully rewritten before use.
    size_t clear = sizeof(int);
    if (ns > 1) {
        carve_ws(base + kNoAllocHeader, ns * n_kv_heads, n_kv_heads, gmax, p);
        clear = kNoAllocHeader + static_cast<size_t>(n_kv_heads) * sizeof(uint32_t);
    }
    cudaError_t e = cudaMemsetAsync(base, 0, clear, st);
    if (e != cudaSuccess) {
        set_err(err, errlen, "decode_noalloc: clearing the scratch failed: %s", cudaGetErrorString(e));
        return -1;
    }
    return launch_decode(p, head_dim, ns * n_kv_heads, st, err, errlen);
}
