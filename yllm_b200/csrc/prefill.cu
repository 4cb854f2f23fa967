// prefill.cu -- causal batched prefill attention on tcgen05 / TMEM / TMA (sm_100a).
//
// Reference semantics: engine.c:533-563 (CPU batched prefill) and the
// reference GPU kernel k_attn_flash_prefill (inference/cuda/cuda_kernels.cu:602-655):
// B query tokens at positions pos_start..pos_start+B-1; token b (q row
// q + b*q_stride + hh*head_dim) attends keys 0..pos_start+b of kv head
// hh*n_kv/n_heads; out has q's layout.  Optional qwen35 sigmoid output gate
// (engine.c:958-960).
//
// One CTA = one (query head, 128-row query tile), heaviest tiles first.  Warps:
//   0-7  softmax: row i of the tile (TMEM lane i) belongs to warps i/32 and
//        i/32 + 4, which split each key block's columns in halves.  They load
//        the fp32 Q tile once: Q_hi = fp16(q) goes to smem (SWIZZLE_128B
//        K-major).  The default kernel (QLO) also writes Q_lo = fp16(q - Q_hi)
//        to free TMEM columns, and S gets a second product Q_lo K^T (TS form),
//        so q keeps about 22 significant bits, as the engine's fp32 projections
//        need; it runs with two S buffers instead of three to make room.  A
//        caller whose q is fp16 by construction asks for the hi-only kernel,
//        which checks that claim (status 202 if a q value is not an fp16
//        value) and runs three S buffers and no second product.  Per key
//        block each reads its half of S from TMEM, applies the causal mask
//        (diagonal blocks only), and the two halves of a row combine their
//        maxima through shared memory; the online softmax runs in the log2
//        domain (the running max only moves when it grows by more than 2^8, so
//        O in TMEM is rarely rescaled).  Each writes P back over the S columns
//        it has read as two fp16 planes P_hi + P_lo (P_lo = fp16(p - P_hi),
//        ~22 bits instead of fp16's 11), 16 columns of each per 32-key chunk.
//        Each half keeps its own partial row sum; the epilogue adds them.
//   8    TMA for K blocks, 10 TMA for V blocks: separate rings, no multicast.
//   9    MMA: one thread issues S(j) = Q K(j)^T (A, B from smem; + Q_lo K(j)^T
//        with A from TMEM in the QLO kernel) into a ring of NSB (3, or 2 with
//        Q_lo) TMEM S buffers and O += P_hi V + P_lo V with A = P read
//        straight from TMEM (B = V from smem).  S runs up to NSB blocks ahead of
//        the softmax; the tensor core runs its MMAs in issue order, so S(j+NSB)
//        cannot overwrite P(j) before PV(j) has read it.
// Keys past the end of the cache are zero-filled by TMA and masked.
#include "common.cuh"
#include "tcgen05.cuh"

#include <algorithm>

namespace yattn {
namespace {

constexpr int BM = 128;
constexpr int kPThreads = 352;

// One CTA per SM (TMEM: all 512 columns).  128-key blocks (64 at head_dim 256),
// three TMEM S buffers.  The V ring is one stage shallower than the K ring at
// head_dim >= 128: V(j) is needed only by PV(j), two blocks after its slot frees.
template <int HD> struct PCfg {
    static constexpr int BN = HD >= 256 ? 64 : 128;
    static constexpr int KST = HD >= 256 ? 2 : 3;           // K ring depth
    static constexpr int VST = HD >= 128 ? 2 : 3;           // V ring depth
    static constexpr int Q_BYTES = BM * HD * 2;
    static constexpr int KV_BYTES = BN * HD * 2;            // one K (or V) block
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + Q_BYTES;
    static constexpr int OFF_V = OFF_K + KST * KV_BYTES;
    static constexpr int OFF_X = OFF_V + VST * KV_BYTES;    // [2 blocks][2 halves][BM] floats: row maxima / sums
    static constexpr int OFF_BAR = OFF_X + 2 * 2 * BM * 4;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;       // + barriers, + alignment slack
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr int NSB = 3;                           // S buffers in TMEM (P is written over its S)
    static constexpr uint32_t COL_S = 0;                     // S buffer b at [b*BN, (b+1)*BN)
    static constexpr uint32_t COL_O = NSB * BN;
    static_assert(NSB * BN + HD <= static_cast<int>(TMEM_COLS), "TMEM columns");
    // Q_lo (the A operand of the second S product, 16-bit pairs, HD/2 columns):
    // 16-key chunk kk at qlo_col(kk).  head_dim 64: after O, beside three S buffers.
    // 128: the third S buffer.  256: the third S buffer, then after O.
    static constexpr int NSB_QLO = HD == 64 ? 3 : 2;
    __host__ __device__ static constexpr uint32_t qlo_col(int kk) {
        return HD == 64 ? COL_O + HD + 8u * kk
             : HD == 128 ? 2u * BN + 8u * kk
             : (kk < 8 ? 2u * BN + 8u * kk : COL_O + HD + 8u * (kk - 8));
    }
    static_assert(qlo_col(HD / 16 - 1) + 8 <= TMEM_COLS, "Q_lo columns");
    static_assert(SMEM <= 232448, "shared memory");
    static_assert(KST * KV_BYTES >= 8 * 32 * 128, "the epilogue's store boxes fit in the K ring");
};

struct PrefillParams {
    const float* q;
    float* out;
    const float* gate;
    uint32_t q_stride, pos_start, B, n_heads, n_kv;
    uint32_t n_qt;                    // 128-row query tiles
    float scale_log2;
    int* status;
};

template <int KST, int VST> struct Bars {
    uint64_t k_full[KST], k_empty[KST], v_full[VST], v_empty[VST];
    // per S buffer b: S(j) ready, P(j) written, PV(j) accumulated, for the blocks j with j % 3 == b
    uint64_t s_full[3], p_full[3], pv_done[3];
    uint64_t o_done, q_full, mma_drain;
    uint32_t tmem_base;
    int abort_flag;
};

// One TMA producer: block j of a K or V stream into a DEPTH-deep ring.
template <int HD, int DEPTH>
__device__ __forceinline__ void produce(const CUtensorMap* map, uint8_t* ring, uint64_t* full, uint64_t* empty,
                                        uint32_t kvh, uint32_t nkb, int* status, volatile int* abort_flag) {
    using C = PCfg<HD>;
    constexpr int BN = C::BN;
    prefetch_tensormap(map);
    uint32_t issued = 0;
    for (uint32_t j = 0; j < nkb; ++j) {
        const int s = j % DEPTH;
        if (j >= static_cast<uint32_t>(DEPTH) &&
            !mbar_wait_bounded(&empty[s], ((j / DEPTH) & 1u) ^ 1u, status, ST_PREFILL_TIMEOUT, abort_flag))
            break;
        mbar_arrive_expect_tx(&full[s], C::KV_BYTES);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
            tma_load_2d(ring + s * C::KV_BYTES + c * BN * 128, map, static_cast<int32_t>(kvh * HD + c * 64),
                        static_cast<int32_t>(j * BN), &full[s]);
        issued = j + 1;
    }
    // no load may still be landing when the CTA exits
    volatile int dummy = 0;
    for (uint32_t j = (issued > static_cast<uint32_t>(DEPTH) ? issued - DEPTH : 0); j < issued; ++j)
        mbar_wait_bounded(&full[j % DEPTH], (j / DEPTH) & 1u, status, ST_PREFILL_TIMEOUT, &dummy);
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

template <int HD, bool QLO>
__global__ void __launch_bounds__(kPThreads, 1)
    k_prefill(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
              const __grid_constant__ CUtensorMap tmO, const PrefillParams p) {
    using C = PCfg<HD>;
    constexpr int BN = C::BN;
    constexpr int HB = BN / 2;        // columns of a block per half
    constexpr int KST = C::KST;
    constexpr int VST = C::VST;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem + C::OFF_Q;
    uint8_t* sK = smem + C::OFF_K;
    uint8_t* sV = smem + C::OFF_V;
    float* xch = reinterpret_cast<float*>(smem + C::OFF_X);
    Bars<KST, VST>* bars = reinterpret_cast<Bars<KST, VST>*>(smem + C::OFF_BAR);
    volatile int* abort_flag = &bars->abort_flag;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // tile rank k in size order (heaviest first)
    const uint32_t k = blockIdx.x;
    const uint32_t hh = k % p.n_heads;
    const uint32_t qt = p.n_qt - 1 - k / p.n_heads;
    const uint32_t kvh = hh * p.n_kv / p.n_heads;
    const uint32_t row0 = qt * BM;
    const uint32_t rows_valid = min(static_cast<uint32_t>(BM), p.B - row0);
    const uint32_t qpos0 = p.pos_start + row0;
    const uint32_t kmax = qpos0 + rows_valid - 1;
    const uint32_t nkb = kmax / BN + 1;

    // The softmax warps' share of the fp32 Q tile (one batch of loads in flight per thread), issued before the
    // barrier and TMEM setup below so that the loads' latency passes meanwhile.
    constexpr int C4 = HD / 4;
    constexpr int QITER = BM * C4 / 256;
    static_assert(QITER <= 32, "Q loads in one batch");
    float4 qv[QITER];
    if (warp < 8) {
#pragma unroll
        for (int i = 0; i < QITER; ++i) {
            const int idx = threadIdx.x + i * 256;
            const uint32_t b = row0 + idx / C4;
            qv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (b < p.B)
                qv[i] = __ldcs(reinterpret_cast<const float4*>(p.q + static_cast<size_t>(b) * p.q_stride +
                                                               static_cast<size_t>(hh) * HD + (idx % C4) * 4));
        }
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < KST; ++s) {
            mbar_init(&bars->k_full[s], 1);
            mbar_init(&bars->k_empty[s], 1);
        }
        for (int s = 0; s < VST; ++s) {
            mbar_init(&bars->v_full[s], 1);
            mbar_init(&bars->v_empty[s], 1);
        }
        for (int s = 0; s < C::NSB; ++s) {
            mbar_init(&bars->s_full[s], 1);
            mbar_init(&bars->p_full[s], 8);
            mbar_init(&bars->pv_done[s], 1);
        }
        mbar_init(&bars->o_done, 1);
        mbar_init(&bars->q_full, 8);
        mbar_init(&bars->mma_drain, 1);
        bars->abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(&bars->tmem_base, C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 8) {
        if (lane == 0) produce<HD, KST>(&tmK, sK, bars->k_full, bars->k_empty, kvh, nkb, p.status, abort_flag);
    } else if (warp == 10) {
        if (lane == 0) produce<HD, VST>(&tmV, sV, bars->v_full, bars->v_empty, kvh, nkb, p.status, abort_flag);
    } else if (warp == 9) {
        // ================= MMA issuer =================
        if (lane == 0) {
            constexpr uint32_t IDESC_QK = idesc_f16(BM, BN, 0);
            constexpr uint32_t IDESC_PV = idesc_f16(BM, HD, 1);
            // Shared-memory descriptors are built once: a descriptor's address field counts 16-byte
            // units, so one at `base + off` is the base descriptor + off / 16 (every operand lies
            // inside this CTA's shared memory, below 256 KB, so the 14-bit field never carries).
            const uint64_t dq0 = sdesc_sw128(sQ, 16, 1024);
            const uint64_t dk0 = sdesc_sw128(sK, 16, 1024);
            const uint64_t dv0 = sdesc_sw128(sV, BN * 128, 1024);
            bool ok = mbar_wait_bounded(&bars->q_full, 0, p.status, ST_PREFILL_TIMEOUT, abort_flag);
            tc_fence_after();
            {
                constexpr uint32_t nsb = QLO ? C::NSB_QLO : C::NSB;
                // S buffer and phase of the next S(jj) and of the next PV(jj): both advance by one
                // block per call (no division by the runtime buffer count)
                uint32_t s_sb = 0, pv_sb = 0, pv_ph = 0;
                // S(jj) = Q K(jj)^T into S buffer jj % nsb.  That buffer last held P(jj - nsb), whose PV
                // product was issued earlier; the tensor core runs one thread's MMAs in issue order.
                auto do_s = [&](uint32_t jj) -> bool {
                    const int s = jj % KST;
                    if (!mbar_wait_bounded(&bars->k_full[s], (jj / KST) & 1u, p.status, ST_PREFILL_TIMEOUT, abort_flag))
                        return false;
                    const uint32_t sb = s_sb;
                    if (++s_sb == nsb) s_sb = 0;
                    tc_fence_after();
                    const uint64_t dk = dk0 + ((s * C::KV_BYTES) >> 4);
    #pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk) {
                        const uint64_t a = dq0 + (((kk >> 2) * (BM * 128) + (kk & 3) * 32) >> 4);
                        const uint64_t b = dk + (((kk >> 2) * (BN * 128) + (kk & 3) * 32) >> 4);
                        umma_f16(tmem + C::COL_S + sb * BN, a, b, IDESC_QK, kk > 0 ? 1u : 0u);
                    }
                    if constexpr (QLO) {   // + Q_lo K^T, A (16-key chunk kk of Q_lo) from TMEM
    #pragma unroll
                        for (int kk = 0; kk < HD / 16; ++kk) {
                            const uint64_t b = dk + (((kk >> 2) * (BN * 128) + (kk & 3) * 32) >> 4);
                            umma_f16_ts(tmem + C::COL_S + sb * BN, tmem + C::qlo_col(kk), b, IDESC_QK, 1u);
                        }
                    }
                    umma_commit(&bars->s_full[sb]);
                    umma_commit(&bars->k_empty[s]);
                    return true;
                };
                // O += P_hi V + P_lo V with A = P(jj) read from TMEM: keys [16kk, 16kk+16) of a plane
                // are the 8 columns at 32*(kk/2) + 16*plane + 8*(kk%2) of the block's S buffer.
                auto do_pv = [&](uint32_t jj) -> bool {
                    const int s = jj % VST;
                    const uint32_t sb = pv_sb, ph = pv_ph;
                    if (!mbar_wait_bounded(&bars->p_full[sb], ph, p.status, ST_PREFILL_TIMEOUT, abort_flag) ||
                        !mbar_wait_bounded(&bars->v_full[s], (jj / VST) & 1u, p.status, ST_PREFILL_TIMEOUT, abort_flag))
                        return false;
                    if (++pv_sb == nsb) {
                        pv_sb = 0;
                        pv_ph ^= 1u;
                    }
                    tc_fence_after();
                    const uint32_t pcol = tmem + C::COL_S + sb * BN;
                    const uint64_t dv = dv0 + ((s * C::KV_BYTES) >> 4);
    #pragma unroll
                    for (int plane = 0; plane < 2; ++plane) {
    #pragma unroll
                        for (int kk = 0; kk < BN / 16; ++kk) {
                            const uint64_t b = dv + ((kk * 16 * 128) >> 4);
                            umma_f16_ts(tmem + C::COL_O, pcol + 32 * (kk >> 1) + 16 * plane + 8 * (kk & 1), b, IDESC_PV,
                                        (jj > 0 || plane > 0 || kk > 0) ? 1u : 0u);
                        }
                    }
                    umma_commit(&bars->v_empty[s]);
                    umma_commit(&bars->pv_done[sb]);
                    return true;
                };
                // Queue: S(0..nsb-1), then PV(j), S(j+nsb) as each P(j) arrives, so the next S blocks
                // are ready before the softmax asks for them.
                for (uint32_t j = 0; ok && j < nkb && j < nsb; ++j) ok = do_s(j);
                for (uint32_t j = 0; ok && j < nkb; ++j) {
                    ok = do_pv(j);
                    if (ok && j + nsb < nkb) ok = do_s(j + nsb);
                }
            }
            if (ok) umma_commit(&bars->o_done);
            // drain: every MMA issued so far completes before TMEM is freed
            umma_commit(&bars->mma_drain);
            volatile int dummy = 0;
            mbar_wait_bounded(&bars->mma_drain, 0, p.status, ST_PREFILL_TIMEOUT, &dummy);
        }
    } else if (warp < 8) {
        // ================= softmax warps 0-7 =================
        const int qd = warp & 3;                                     // TMEM lane quadrant
        const int h = warp >> 2;                                     // half of each key block's columns
        const int r = qd * 32 + lane;                                // row of the tile
        const uint32_t trow = tmem + (static_cast<uint32_t>(qd * 32) << 16);
        // ---- Q tile: fp32 -> Q_hi = fp16(q) (smem, swizzled K-major) and, if any q of the
        //      tile is not an fp16 value, Q_lo = fp16(q - Q_hi) (TMEM); 256 threads, one batch
        //      of loads in flight each ----
        {
            const float4* v = qv;   // loaded before the setup
            // hi and lo halves of this thread's q, packed (4 registers per float4 loaded)
            uint2 qh[QITER], ql[QITER];
            bool any_lo = false;
#pragma unroll
            for (int i = 0; i < QITER; ++i) {
                const __half2 h0 = __floats2half2_rn(v[i].x, v[i].y), h1 = __floats2half2_rn(v[i].z, v[i].w);
                const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
                qh[i].x = h2_bits(h0);
                qh[i].y = h2_bits(h1);
                if constexpr (QLO) {
                    ql[i].x = h2_bits(__floats2half2_rn(v[i].x - f0.x, v[i].y - f0.y));
                    ql[i].y = h2_bits(__floats2half2_rn(v[i].z - f1.x, v[i].w - f1.y));
                } else {
                    any_lo = any_lo || (f0.x != v[i].x) || (f0.y != v[i].y) || (f1.x != v[i].z) || (f1.y != v[i].w);
                }
            }
            if constexpr (!QLO) {
                // the caller said q is fp16 by construction: a value that is not is reported
                // (status 202) and the tile runs on Q_hi alone
                if (__any_sync(0xffffffffu, any_lo) && lane == 0) atomicCAS(p.status, 0, ST_PREFILL_Q_NOT_F16);
            } else {
                // Q_lo goes through the Q buffer (this thread's elements), so the thread that owns
                // a row's TMEM lane can pick it up; Q_hi then overwrites it.
#pragma unroll
                for (int i = 0; i < QITER; ++i) {
                    const int idx = threadIdx.x + i * 256;
                    *reinterpret_cast<uint2*>(sQ + sw128_offset(idx / C4, (idx % C4) * 4, BM)) = ql[i];
                }
                named_bar_sync(5, 256);
                // row r, this half's dims [h*HD/2, +HD/2): 32 dims (16 TMEM columns) at a time
#pragma unroll
                for (int c = 0; c < HD / 64; ++c) {
                    const int d0 = h * (HD / 2) + c * 32;
                    uint32_t w[16];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const uint4 x = *reinterpret_cast<const uint4*>(sQ + sw128_offset(r, d0 + 8 * u, BM));
                        w[4 * u] = x.x;
                        w[4 * u + 1] = x.y;
                        w[4 * u + 2] = x.z;
                        w[4 * u + 3] = x.w;
                    }
                    tmem_st16(trow + C::qlo_col(d0 / 16), w);
                }
                tmem_wait_st();
                named_bar_sync(5, 256);           // every row's Q_lo is read before Q_hi replaces it
            }
#pragma unroll
            for (int i = 0; i < QITER; ++i) {
                const int idx = threadIdx.x + i * 256;
                *reinterpret_cast<uint2*>(sQ + sw128_offset(idx / C4, (idx % C4) * 4, BM)) = qh[i];
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->q_full);
        }
        const uint32_t qpos = qpos0 + r;
        const float sl2 = p.scale_log2;
        float m_run = -INFINITY, l_run = 0.f;                        // m_run in scaled log2 units; l_run: this half
        bool ok = true;
        // The two halves of a row meet at a named barrier once per block.  Every wait result
        // goes through that barrier (AND-reduced), so both halves always leave together and
        // neither is left at a barrier its partner will not reach.
        {
            constexpr uint32_t nsb = QLO ? C::NSB_QLO : C::NSB;
            uint32_t sb = 0, sph = 0;            // S buffer of block j and its phase
            uint32_t pb = 0, pph = 0;            // the same for block j - 1 (its PV completion)
            for (uint32_t j = 0; j < nkb; ++j) {
                const bool got = warp_wait_bounded(&bars->s_full[sb], sph, p.status, ST_PREFILL_TIMEOUT, abort_flag);
                const uint32_t scol = trow + C::COL_S + sb * BN + h * HB;  // this half's columns of S(j)
                float sv[HB];
                if (got) {
                    tc_fence_after();
    #pragma unroll
                    for (int c = 0; c < HB / 32; ++c) {
                        uint32_t rr[32];
                        tmem_ld32(scol + c * 32, rr);
    #pragma unroll
                        for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(rr[i]);
                    }
                    tmem_wait_ld();
                } else {
    #pragma unroll
                    for (int c = 0; c < HB; ++c) sv[c] = -INFINITY;
                }
                // ---- causal mask (diagonal blocks only), row max of raw scores over both halves ----
                const uint32_t kbase = j * BN + h * HB;
                if (j * BN + BN - 1 > qpos0) {
    #pragma unroll
                    for (int c = 0; c < HB; ++c)
                        if (kbase + c > qpos) sv[c] = -INFINITY;
                }
                float mx4[4] = {sv[0], sv[1], sv[2], sv[3]};
    #pragma unroll
                for (int c = 4; c < HB; c += 4) {
                    mx4[0] = fmaxf(mx4[0], sv[c]);
                    mx4[1] = fmaxf(mx4[1], sv[c + 1]);
                    mx4[2] = fmaxf(mx4[2], sv[c + 2]);
                    mx4[3] = fmaxf(mx4[3], sv[c + 3]);
                }
                float* xb = xch + (j & 1) * (2 * BM);                    // two slots alternate by block parity
                xb[h * BM + r] = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
                if (!named_bar_and(1 + qd, 64, got)) {                   // the row's two halves
                    ok = false;
                    break;
                }
                const float mx = fmaxf(xb[r], xb[BM + r]) * sl2;
                const float m_new = fmaxf(m_run, mx);
                const bool grow = m_new > m_run + 8.0f;                  // keep a stale max up to 2^8 headroom
                const float m_use = grow ? m_new : m_run;
                const float alpha = grow ? ex2_approx(m_run - m_use) : 1.0f;
                // a row whose keys so far are all masked keeps m = -inf and gets p = 0
                const float m_sub = (m_use == -INFINITY) ? 0.f : m_use;
                // ---- p = 2^(s*scale - m): one FFMA + ex2 per element; P hi/lo over this half's S ----
                // pairs of elements in packed fp32x2 arithmetic (FFMA2 / FADD2): half the FMA, add and
                // subtract instructions of the scalar form
                const float2 sl2x2 = make_float2(sl2, sl2), negm = make_float2(-m_sub, -m_sub);
                const float2 neg1 = make_float2(-1.f, -1.f);
                float2 rs2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    #pragma unroll
                for (int c = 0; c < HB / 32; ++c) {   // 32 keys -> 16 columns of P_hi, then 16 of P_lo
                    uint32_t hi[16], lo[16];
    #pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float2 x = __ffma2_rn(make_float2(sv[c * 32 + 2 * i], sv[c * 32 + 2 * i + 1]), sl2x2, negm);
                        const float2 pp = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                        rs2[i & 1] = __fadd2_rn(rs2[i & 1], pp);
                        const __half2 hv = __floats2half2_rn(pp.x, pp.y);
                        const float2 r = __ffma2_rn(__half22float2(hv), neg1, pp);   // p - fp16(p)
                        hi[i] = h2_bits(hv);
                        lo[i] = h2_bits(__floats2half2_rn(r.x, r.y));
                    }
                    tmem_st16(scol + c * 32, hi);
                    tmem_st16(scol + c * 32 + 16, lo);
                }
                l_run = l_run * alpha + ((rs2[0].x + rs2[0].y) + (rs2[1].x + rs2[1].y));
                m_run = m_use;
                // ---- O rescale (rare), this half's columns of O: PV(j-1) must have finished ----
                // (both halves of these rows see the same `grow`, so both come here)
                if (j >= 1 && __any_sync(0xffffffffu, grow)) {
                    const bool done =
                        warp_wait_bounded(&bars->pv_done[pb], pph, p.status, ST_PREFILL_TIMEOUT, abort_flag);
                    if (!named_bar_and(1 + qd, 64, done)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
    #pragma unroll 1
                    for (int c = 0; c < HD / 64; ++c) {
                        const uint32_t oc = trow + C::COL_O + h * (HD / 2) + c * 32;
                        uint32_t rr[32];
                        tmem_ld32(oc, rr);
                        tmem_wait_ld();
    #pragma unroll
                        for (int i = 0; i < 32; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * alpha);
                        tmem_st32(oc, rr);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->p_full[sb]);
                pb = sb;
                pph = sph;
                if (++sb == nsb) {
                    sb = 0;
                    sph ^= 1u;
                }
            }
        }
        // ---- epilogue: O / l (x sigmoid(gate)) -> out; each half takes its HD/2 columns ----
        // the last PV's completion, on a barrier of its own; the row sums of the two halves
        // meet in the exchange slots (slot 0 after a barrier: the last block's maxima are read)
        // The slot block nkb-1 did not use is free: both halves read it (block nkb-2's maxima)
        // before they met at block nkb-1's barrier.
        ok = ok && warp_wait_bounded(&bars->o_done, 0, p.status, ST_PREFILL_TIMEOUT, abort_flag);
        float* xl = xch + (nkb & 1) * (2 * BM);
        xl[h * BM + r] = l_run;
        ok = named_bar_and(1 + qd, 64, ok);
        if (ok) {
            tc_fence_after();
            const float inv_l = 1.0f / (xl[r] + xl[BM + r]);
            if (!p.gate) {
                // Each warp stages 32 rows x 32 columns at a time in a 128-byte-swizzled box in
                // the K ring (every K block has been consumed) and one lane stores the box with a
                // tensor copy, so rows go out as whole 128-byte segments; rows past B are clipped
                // by the map.
                uint8_t* box = sK + warp * (32 * 128);
#pragma unroll 1
                for (int c = 0; c < HD / 64; ++c) {
                    const int col = h * (HD / 2) + c * 32;
                    if (lane == 0) bulk_wait_group_read<0>();         // this warp's previous box has been read
                    __syncwarp();
                    uint32_t rr[32];
                    tmem_ld32(trow + C::COL_O + col, rr);
                    tmem_wait_ld();
#pragma unroll
                    for (int k4 = 0; k4 < 8; ++k4) {
                        float4 o;
                        o.x = __uint_as_float(rr[k4 * 4]) * inv_l;
                        o.y = __uint_as_float(rr[k4 * 4 + 1]) * inv_l;
                        o.z = __uint_as_float(rr[k4 * 4 + 2]) * inv_l;
                        o.w = __uint_as_float(rr[k4 * 4 + 3]) * inv_l;
                        *reinterpret_cast<float4*>(box + lane * 128 + ((k4 ^ (lane & 7)) << 4)) = o;
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmO, box, static_cast<int32_t>(hh * HD + col), static_cast<int32_t>(row0 + qd * 32));
                        bulk_commit_group();
                    }
                }
                // the boxes have been read before the CTA (and its shared memory) goes; the stores' global writes
                // complete with the grid
                if (lane == 0) bulk_wait_group_read<0>();
            } else {
                const uint32_t b = row0 + r;
#pragma unroll 1
                for (int c = 0; c < HD / 64; ++c) {
                    const int col = h * (HD / 2) + c * 32;
                    uint32_t rr[32];
                    tmem_ld32(trow + C::COL_O + col, rr);
                    tmem_wait_ld();
                    if (b < p.B) {
                        float* dst = p.out + static_cast<size_t>(b) * p.q_stride + static_cast<size_t>(hh) * HD + col;
                        const float* g = p.gate + static_cast<size_t>(b) * p.q_stride + static_cast<size_t>(hh) * HD + col;
#pragma unroll
                        for (int i = 0; i < 32; i += 4) {
                            const float4 gv = *reinterpret_cast<const float4*>(g + i);
                            float4 o;
                            o.x = __uint_as_float(rr[i]) * inv_l / (1.0f + __expf(-gv.x));
                            o.y = __uint_as_float(rr[i + 1]) * inv_l / (1.0f + __expf(-gv.y));
                            o.z = __uint_as_float(rr[i + 2]) * inv_l / (1.0f + __expf(-gv.z));
                            o.w = __uint_as_float(rr[i + 3]) * inv_l / (1.0f + __expf(-gv.w));
                            *reinterpret_cast<float4*>(dst + i) = o;
                        }
                    }
                }
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ------------------------------------------------------------------ host side

template <int HD, bool QLO>
int launch_prefill(const CUtensorMap& mk, const CUtensorMap& mv, const PrefillParams& p, uint32_t n_qtiles,
                   cudaStream_t st, char* err, size_t errlen) {
    using C = PCfg<HD>;
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(k_prefill<HD, QLO>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) {
            set_err(err, errlen, "prefill: smem attribute (%d bytes): %s", C::SMEM, cudaGetErrorString(e));
            return -1;
        }
        attr_done[dev] = true;
    }
    PrefillParams q = p;
    const uint32_t n_tiles = p.n_heads * n_qtiles;
    q.n_qt = n_qtiles;
    CUtensorMap mo;   // out as fp32 rows of q_stride, for the epilogue's tensor-copy stores
    if (encode_f32_store_map(&mo, p.out, p.n_heads * HD, p.q_stride, p.B, 32, err, errlen)) return -1;
    k_prefill<HD, QLO><<<n_tiles, kPThreads, C::SMEM, st>>>(mk, mv, mo, q);
    YATTN_CHECK_LAUNCH(err, errlen, "prefill");
    return 0;
}

}  // namespace

int prefill(float* out, const float* q, const uint16_t* kc, const uint16_t* vc, const float* gate,
            uint32_t pos_start, uint32_t B, uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t kv_dim,
            uint32_t q_stride, uint32_t flags, cudaStream_t st, char* err, size_t errlen) {
    if (!out || !q || !kc || !vc) {
        set_err(err, errlen, "prefill: null pointer argument");
        return -1;
    }
    if (B == 0) return 0;
    if (flags & ~static_cast<uint32_t>(YATTN_PREFILL_Q_F16)) {
        set_err(err, errlen, "prefill: unknown flags 0x%x", flags);
        return -1;
    }
    if (n_heads == 0 || n_kv == 0 || n_kv > n_heads) {
        set_err(err, errlen, "prefill: bad head counts n_heads=%u n_kv_heads=%u", n_heads, n_kv);
        return -1;
    }
    if (hd != 64 && hd != 128 && hd != 256) {
        set_err(err, errlen, "prefill: head_dim %u not supported (64/128/256)", hd);
        return -1;
    }
    if (kv_dim < n_kv * hd || (kv_dim % 8) != 0) {
        set_err(err, errlen, "prefill: kv_dim %u must be >= n_kv_heads*head_dim and a multiple of 8", kv_dim);
        return -1;
    }
    if (q_stride < n_heads * hd || (q_stride % 4) != 0) {
        set_err(err, errlen, "prefill: q_stride %u must be >= n_heads*head_dim and a multiple of 4", q_stride);
        return -1;
    }
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(kc) |
         reinterpret_cast<uintptr_t>(vc) | reinterpret_cast<uintptr_t>(gate)) & 15u) {
        set_err(err, errlen, "prefill: q, out, gate, kcache and vcache must be 16-byte aligned");
        return -1;
    }
    if (static_cast<uint64_t>(pos_start) + B > 0x7fffffffull) {
        set_err(err, errlen, "prefill: pos_start + B too large");
        return -1;
    }
    DevCtx* ctx = dev_ctx(err, errlen);
    if (!ctx) return -1;
    const uint32_t n_keys = pos_start + B;
    const uint32_t bn = hd == 64 ? PCfg<64>::BN : hd == 128 ? PCfg<128>::BN : PCfg<256>::BN;   // key block
    CUtensorMap mk, mv;
    if (encode_kv_map(&mk, kc, kv_dim, n_keys, bn, err, errlen) || encode_kv_map(&mv, vc, kv_dim, n_keys, bn, err, errlen))
        return -1;
    PrefillParams p{};
    p.q = q;
    p.out = out;
    p.gate = gate;
    p.q_stride = q_stride;
    p.pos_start = pos_start;
    p.B = B;
    p.n_heads = n_heads;
    p.n_kv = n_kv;
    p.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(hd));
    p.status = ctx->status;
    const uint32_t n_qtiles = (B + BM - 1) / BM;
    const bool f16q = (flags & YATTN_PREFILL_Q_F16) != 0;
    switch (hd) {
        case 64: return f16q ? launch_prefill<64, false>(mk, mv, p, n_qtiles, st, err, errlen)
                             : launch_prefill<64, true>(mk, mv, p, n_qtiles, st, err, errlen);
        case 128: return f16q ? launch_prefill<128, false>(mk, mv, p, n_qtiles, st, err, errlen)
                              : launch_prefill<128, true>(mk, mv, p, n_qtiles, st, err, errlen);
        default: return f16q ? launch_prefill<256, false>(mk, mv, p, n_qtiles, st, err, errlen)
                             : launch_prefill<256, true>(mk, mv, p, n_qtiles, st, err, errlen);
    }
}

}  // namespace yattn

using namespace yattn;

extern "C" int yattn_attn_prefill(float* att_out, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                                  const float* gate, uint32_t pos_start, uint32_t B, uint32_t n_heads,
                                  uint32_t n_kv_heads, uint32_t head_dim, uint32_t kv_dim, uint32_t q_stride,
                                  uint32_t flags, void* stream, char* err, size_t errlen) {
    return prefill(att_out, q, kcache, vcache, gate, pos_start, B, n_heads, n_kv_heads, head_dim, kv_dim, q_stride,
                   flags, static_cast<cudaStream_t>(stream), err, errlen);
}

extern "C" void cuda_k_attn_prefill(float* att_out, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                                    uint32_t pos_start, uint32_t B, uint32_t n_heads, uint32_t n_kv_heads,
                                    uint32_t head_dim, uint32_t kv_dim, uint32_t q_stride) {
    char err[256];
    err[0] = 0;
    // the engine passes its fp32 projections: the q hi + lo kernel
    if (prefill(att_out, q, kcache, vcache, nullptr, pos_start, B, n_heads, n_kv_heads, head_dim, kv_dim, q_stride, 0,
                nullptr, err, sizeof(err)) != 0)
        set_last_error(err);
}
