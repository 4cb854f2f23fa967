// decode.cu -- GQA decode attention over the fp16 KV cache (sm_100a).
//
// Reference semantics: engine.c:1074-1096 (CPU loop) and the reference GPU
// kernel k_attn_flash_decode (inference/cuda/cuda_kernels.cu:543-600): for
// query head hh, kv head hh*n_kv/n_heads, scores q.k_t / sqrt(d) over t=0..pos,
// softmax, out = sum p_t v_t.
//
// Design (B200): one CTA = one (item, group of HC kv heads, key split).
//   * the producer warp streams the split's K and V rows into a shared-memory
//     ring with cp.async.bulk (TMA, non-tensor), one bulk copy per token row
//     covering the HC kv heads' contiguous slices (2 KB for Llama-3-8B), rows
//     padded by 16 B in shared memory for conflict-free ldmatrix;
//   * each consumer warp owns one kv head of the group and 16 tokens of every
//     stage and runs both products on the tensor cores with mma.sync m16n8k16
//     in the transposed form S^T = K Q^T and O^T += V^T P^T (tokens / dims on
//     M, the <= 8 query heads of the kv head on N).  q and p are split into
//     fp16 hi + lo parts, so the products keep ~22 bits against the engine's
//     fp32 loop; K and V are the cache's fp16 values, exact.  The online
//     softmax runs in the log2 domain with warp-shuffle max/sum;
//   * the warps' (m, l, o) are merged in shared memory; a split writes its
//     partials to the workspace and the last split of an (item, head group) to
//     arrive (atomic counter) merges all splits with log-sum-exp weights.
#include "common.cuh"
#include "exchange.cuh"
#include "tcgen05.cuh"

#include <algorithm>
#include <mutex>
#include <vector>

namespace yattn {
namespace {

constexpr int kSplitQuant = 64;     // split lengths are multiples of this
constexpr uint32_t kSplitMin = 128;  // shortest split of a balanced plan (keys)
constexpr uint32_t kMaxSplits = 32;  // most splits of one (item, head group) in a balanced plan
constexpr uint32_t kUnitCost = 320;  // keys charged for each further unit of a CTA

// Per head_dim: NCW consumer warps and a ring of NST stages.  A stage holds K and V
// of 16 tokens per consumer warp: exactly STAGE_TM bytes for the tensor copies,
// STAGE_ROW with the row copies' 16-byte row padding (largest at HC = 1).
template <int HD> struct DecodeCfg {
    static constexpr int NCW = (HD >= 256) ? 4 : 8;
    static constexpr int THREADS = 32 * (NCW + 1);
    static constexpr int STAGE_TM = 2 * 16 * NCW * HD * 2;
    static constexpr int STAGE_ROW = 2 * 16 * NCW * (HD * 2 + 16);
    static constexpr int NST = (HD <= 64) ? 5 : 3;
    static constexpr int PT_BYTES = 2 * 8 * 48;                       // per warp: P^T hi and lo, 8 heads x 16 tokens
    static constexpr int HC_TM_MAX = HD <= 128 ? 2 : 1;               // most kv heads per CTA of the TM kernels
};

// Kv heads per CTA of the tensor-copy (TM) kernels: two at head_dim <= 128 (a stage
// of 64 tokens, so each copy is 64 tokens x 128 B = 8 KB), else one.
__host__ __device__ inline uint32_t tm_heads_per_cta(uint32_t n_kv, uint32_t hd) {
    return (hd <= 128 && n_kv % 2 == 0) ? 2u : 1u;   // within DecodeCfg<hd>::HC_TM_MAX
}

// Kv heads per CTA for a geometry: the largest of 8/4/2/1 (at most NCW) dividing n_kv.
__host__ __device__ inline uint32_t heads_per_cta(uint32_t n_kv, uint32_t hd) {
    const uint32_t cap = hd >= 256 ? 4u : 8u;
    for (uint32_t hc = cap; hc > 1; hc >>= 1)
        if (n_kv % hc == 0) return hc;
    return 1;
}

struct DecodeParams {
    const YattnDecodeItem* items;
    const YattnDecodeWork* work;      // nullptr: single item, uniform splits (see below)
    YattnDecodeItem item0;            // used when work == nullptr
    uint32_t split_len;               // uniform split length when work == nullptr
    uint32_t n_splits0;               // splits per head group when work == nullptr
    uint32_t t_base;                  // key offset when work == nullptr
    uint32_t t_end0;                  // end key (exclusive) when work == nullptr
    uint32_t n_heads, n_kv, kv_dim, hc;
    uint32_t n_work;                  // entries of work (grouped by cta)
    uint64_t kmap_base, vmap_base;    // TM kernels: global base of the K and V tensor maps
    uint32_t row_bytes;               // TM kernels: kv_dim * 2
    float scale_log2;                 // log2(e) / sqrt(head_dim)
    float* part_ml;                   // [n_parts][G][2]
    float* part_o;                    // [n_parts][G][HD]
    uint32_t* counters;               // [n_groups]
    int* status;
    int partial_only;                 // write the merged (m, l, o) instead of out
    int defer_merge;                  // splits only write partials; k_merge_splits merges them
    float* out_ml;                    // partial_only: [n_heads][2]
    float* out_o;                     // partial_only: [n_heads][HD]
};

// The fused RoPE + KV store of yattn_decode_run_pooled_rope: per item the new
// token's k and v (fp32, rows[item]); q is read unrotated.  inv_freq[j] =
// theta^(-2j/d), the reference's powf values (computed on the host).
constexpr int kRopeMaxPairs = 128;
struct DecodeRope {
    const YattnDecodeNewRow* rows;
    uint64_t pool_rows;                   // rows of the pool: the new rows are written inside it only
    uint32_t kind, n_dims;                // rope kind (0 llama, 1 qwen, 2 M-RoPE), rotated dims
    float inv_freq[kRopeMaxPairs];
};

// Threads of k_decode: NCW consumer warps, the producer, and (ROPE) the RoPE warp.
template <int HD, bool ROPE> constexpr int decode_threads() { return DecodeCfg<HD>::THREADS + (ROPE ? 32 : 0); }

__host__ __device__ __forceinline__ void group_of(uint32_t kvh, uint32_t n_heads, uint32_t n_kv, uint32_t& first,
                                                  uint32_t& cnt) {
    // heads hh with hh*n_kv/n_heads == kvh: ceil(kvh*n_heads/n_kv) .. ceil((kvh+1)*n_heads/n_kv)-1
    uint32_t a = (kvh * n_heads + n_kv - 1) / n_kv;
    uint32_t b = ((kvh + 1) * n_heads + n_kv - 1) / n_kv;
    first = a;
    cnt = b - a;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col)
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
// x = hi + lo with hi = fp16(x), lo = fp16(x - hi): about 22 significant bits in two fp16s.
__device__ __forceinline__ void split_h2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 f = __half22float2(h);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = pack_h2(a - f.x, b - f.y);
}

// First index i of work[0..n) with work[i].cta >= c (units are grouped by cta in
// increasing order).  Called by a whole warp: each round the 32 lanes probe 32
// evenly spaced units, narrowing the range 32-fold per dependent load.
__device__ __forceinline__ uint32_t first_unit_from(const YattnDecodeWork* work, uint32_t n, uint32_t c, int lane) {
    uint32_t lo = 0, hi = n;   // answer in [lo, hi]
    while (hi > lo) {
        const uint32_t step = (hi - lo + 31) / 32;
        const uint32_t idx = lo + static_cast<uint32_t>(lane) * step;
        const bool before = idx < hi && work[idx].cta < c;
        const uint32_t k = __popc(__ballot_sync(0xffffffffu, before));   // probes before the answer
        if (k == 0) return lo;
        const uint32_t nlo = lo + (k - 1) * step + 1;
        hi = min(hi, lo + k * step);
        lo = nlo;
        if (step == 1) return lo;
    }
    return lo;
}

// One unit of a CTA: entry u of the plan, or split u of the single-query form.
struct DecodeUnit {
    YattnDecodeItem it;
    uint32_t kg, t0, t1, n_splits, split, part_base, group, item;
};
__device__ __forceinline__ DecodeUnit unit_of(const DecodeParams& p, uint32_t u, uint32_t HC) {
    DecodeUnit x;
    if (p.work) {
        const YattnDecodeWork w = p.work[u];
        x.it = p.items[w.item];
        x.item = w.item;
        x.kg = w.kv_head / HC;
        x.t0 = w.t_begin;
        x.t1 = w.t_end;
        x.n_splits = w.n_splits;
        x.split = w.split;
        x.part_base = w.part_base;
        x.group = w.group;
    } else {
        x.it = p.item0;
        x.item = 0;
        x.kg = u / p.n_splits0;
        x.split = u % p.n_splits0;
        x.n_splits = p.n_splits0;
        x.t0 = p.t_base + x.split * p.split_len;
        x.t1 = min(x.t0 + p.split_len, p.t_end0);
        x.part_base = x.kg * HC * p.n_splits0;
        x.group = x.kg;
    }
    return x;
}

// DPL consecutive floats from global memory through L2 (written by other CTAs).
template <int DPL> __device__ __forceinline__ void ldcg_vec(const float* src, float (&v)[DPL]) {
    if constexpr (DPL % 4 == 0) {
#pragma unroll
        for (int i = 0; i < DPL; i += 4) {
            const float4 x = __ldcg(reinterpret_cast<const float4*>(src + i));
            v[i] = x.x;
            v[i + 1] = x.y;
            v[i + 2] = x.z;
            v[i + 3] = x.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < DPL; i += 2) {
            const float2 x = __ldcg(reinterpret_cast<const float2*>(src + i));
            v[i] = x.x;
            v[i + 1] = x.y;
        }
    }
}

// The fused RoPE store's two pieces, kept out of line: they run once per unit,
// and inlined they would raise the register pressure of the tile loop.
//
// One warp: query heads [0, nq) of a q slot (nq * HD floats in shared memory, the
// unit's q as read) rotated by RoPE at pos in place.  Each lane takes pairs
// j = lane + 32k, one sincos per pair for all heads, with rope_rotate's
// operations, so the values equal those of the RoPE store.
template <int HD>
__device__ __noinline__ void rope_q_slot(float* slot, uint32_t nq, const float* s_freq, uint32_t kind,
                                         uint32_t n_dims, uint32_t pos, uint32_t lane) {
    const uint32_t half = (kind == 2 ? n_dims : static_cast<uint32_t>(HD)) / 2;
    for (uint32_t j = lane; j < half; j += 32) {
        float sn, cs;
        rope_sincos(s_freq[j], pos, sn, cs);
        uint32_t e0, e1;
        rope_pair(kind, HD, n_dims, j, e0, e1);
        for (uint32_t h = 0; h < nq; ++h) {
            float a = slot[h * HD + e0], b = slot[h * HD + e1];
            rope_apply(a, b, sn, cs);
            slot[h * HD + e0] = a;
            slot[h * HD + e1] = b;
        }
    }
}

// One warp: the new token's row of kv heads [kv0, kv0 + nh) -- k rotated, k and v
// rounded with the engine's f32_to_f16 -- into cache row pos, then a proxy fence,
// so that tensor copies ordered after it read the new values.
// kn_g / vn_g: the new row's fp32 k and v of those heads (16-byte aligned), first
// copied into stage (2 * nh * HD floats of shared memory) with all of a lane's
// loads in flight, so the warp waits out one memory latency, not one per pair.
template <int HD>
__device__ __noinline__ void rope_new_rows(const YattnDecodeItem& it, const float* kn_g, const float* vn_g,
                                           float* stage, uint32_t kv0, uint32_t nh, uint32_t kv_dim,
                                           const float* s_freq, uint32_t kind, uint32_t n_dims, uint32_t lane) {
    {
        constexpr uint32_t kMax = DecodeCfg<HD>::HC_TM_MAX * HD / 4;   // float4 of k (and of v) at most
        constexpr uint32_t kPer = (kMax + 31) / 32;
        const uint32_t n4 = nh * HD / 4;
        float4 xk[kPer], xv[kPer];
#pragma unroll
        for (uint32_t m = 0; m < kPer; ++m) {
            const uint32_t c = lane + 32 * m;
            if (c < n4) {
                xk[m] = __ldg(reinterpret_cast<const float4*>(kn_g) + c);
                xv[m] = __ldg(reinterpret_cast<const float4*>(vn_g) + c);
            }
        }
#pragma unroll
        for (uint32_t m = 0; m < kPer; ++m) {
            const uint32_t c = lane + 32 * m;
            if (c < n4) {
                reinterpret_cast<float4*>(stage)[c] = xk[m];
                reinterpret_cast<float4*>(stage)[n4 + c] = xv[m];
            }
        }
        __syncwarp();
    }
    const float* kn = stage;
    const float* vn = stage + nh * HD;
    const uint32_t nd = kind == 2 ? n_dims : static_cast<uint32_t>(HD);
    const size_t row = static_cast<size_t>(it.pos) * kv_dim + static_cast<size_t>(kv0) * HD;
    uint16_t* kg = const_cast<uint16_t*>(it.k) + row;
    uint16_t* vg = const_cast<uint16_t*>(it.v) + row;
    for (uint32_t w = lane; w < nh * (nd / 2); w += 32) {
        const uint32_t h = w / (nd / 2), j = w % (nd / 2);
        uint32_t e0, e1;
        rope_pair(kind, HD, n_dims, j, e0, e1);
        float a = kn[h * HD + e0], b = kn[h * HD + e1];
        rope_rotate(a, b, s_freq[j], it.pos);
        kg[h * HD + e0] = engine_f32_to_f16(a);
        kg[h * HD + e1] = engine_f32_to_f16(b);
    }
    for (uint32_t w = lane; w < nh * HD; w += 32) {
        if (w % HD >= nd) kg[w] = engine_f32_to_f16(kn[w]);   // past M-RoPE's dims
        vg[w] = engine_f32_to_f16(vn[w]);
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// What the copies of a unit rely on, checked on the device (items live there).
template <bool TM>
__device__ __forceinline__ bool item_bad(const DecodeParams& p, const YattnDecodeItem& it) {
    const uint64_t ka = reinterpret_cast<uint64_t>(it.k), va = reinterpret_cast<uint64_t>(it.v);
    bool bad = ((reinterpret_cast<uintptr_t>(it.q) | reinterpret_cast<uintptr_t>(it.gate)) & 15u) != 0;
    if (TM)
        bad = bad || ka < p.kmap_base || va < p.vmap_base || (ka - p.kmap_base) % p.row_bytes != 0 ||
              (va - p.vmap_base) % p.row_bytes != 0;
    return bad;
}

// The unit that ends at its item's position holds the item's new row (the last split).
__device__ __forceinline__ bool unit_has_new_row(const DecodeUnit& un) {
    return un.t0 < un.t1 && un.t1 == un.it.pos + 1;
}

__device__ __forceinline__ void st_release_cta(uint32_t* p, uint32_t v) {
    asm volatile("st.release.cta.shared.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_cta(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.cta.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}

// Warp-uniform bounded wait until the shared counter *cnt reaches target (acquire).
// On timeout: records code in *status, sets the abort flag and returns false.
__device__ __forceinline__ bool warp_wait_count(const uint32_t* cnt, uint32_t target, int* status, int code,
                                                volatile int* abort_flag) {
    bool ok = true;
    if (static_cast<int>(ld_acquire_cta(cnt) - target) < 0) {
        const unsigned long long t0 = globaltimer_ns();
        for (uint32_t it = 0;; ++it) {
            if (static_cast<int>(ld_acquire_cta(cnt) - target) >= 0) break;
            if ((it & 63u) == 63u) {
                if (*abort_flag) {
                    ok = false;
                    break;
                }
                if (globaltimer_ns() - t0 > kWaitLimitNs) {
                    if (status) atomicCAS(status, 0, code);
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
            }
        }
    }
    return __all_sync(0xffffffffu, ok);
}

// Shared-memory layout of k_decode<HD, G, TM>: the ring of NST stages, (TM) one
// q slot per stage, the ring's barriers, one unit descriptor per stage, the
// consumer warps' P^T staging, their (m, l) for the merge, and flags.
template <int HD, int G, bool TM, bool ROPE = false> struct DecodeSmem {
    using C = DecodeCfg<HD>;
    static constexpr int STAGE = TM ? C::STAGE_TM : C::STAGE_ROW;
    static constexpr int QSLOT = TM ? C::HC_TM_MAX * G * HD * 4 : 0;   // q of a unit's query heads, fp32
    static constexpr int OFF_Q = C::NST * STAGE;
    static constexpr int OFF_BAR = OFF_Q + C::NST * QSLOT;
    static constexpr int OFF_DESC = (OFF_BAR + 2 * C::NST * 8 + 15) / 16 * 16;
    static constexpr int DESC = (static_cast<int>(sizeof(DecodeUnit)) + 15) / 16 * 16;
    static constexpr int OFF_PT = OFF_DESC + C::NST * DESC;
    static constexpr int OFF_ML = OFF_PT + C::NCW * C::PT_BYTES;
    static constexpr int OFF_FLAGS = OFF_ML + C::NCW * G * 2 * 4;
    static constexpr int OFF_FREQ = OFF_FLAGS + 16;                  // ROPE: inverse frequencies
    // ROPE: u32 counters [0] new rows written (RoPE warp), [1] first-tile stages claimed (producer)
    static constexpr int OFF_ROWS = OFF_FREQ + (ROPE ? kRopeMaxPairs * 4 : 0);
    static constexpr int OFF_RSTAGE = OFF_ROWS + (ROPE ? 16 : 0);     // ROPE: the new row's k and v, fp32
    static constexpr int BYTES = OFF_RSTAGE + (ROPE ? 2 * C::HC_TM_MAX * HD * 4 : 0) + (TM ? 1024 : 0);   // + ring alignment slack
    static_assert(2 * 16 * C::NCW * HD * 2 >= C::NCW * G * HD * 4, "the warps' merge fits in one ring stage");
    static_assert(BYTES <= 232448, "shared memory of one CTA");
    static_assert(OFF_RSTAGE % 16 == 0, "16-byte stores into the row staging area");
};

// Warp NCW is the producer; consumer warp w owns kv head kg*HC + (w % HC) of
// the group and tokens [16*(w / HC), +16) of every stage (TOK = 16*NCW/HC tokens).
// Per 16-token step, on the legacy tensor cores (mma.sync m16n8k16, fp32 accumulate):
//   S^T (16 tok x 8 heads) = K (16 x HD) . Q^T (HD x 8),  q = q_hi + q_lo in fp16
//   O^T (HD x 8 heads)    += V^T (HD x 16) . P^T (16 x 8), p = p_hi + p_lo in fp16
//
// TM = true: HC = p.hc kv heads per CTA, 16*NCW/HC tokens per stage, K and V
// staged by 2-D tensor copies of 64 dims x one stage of tokens (8 KB at the
// chosen HC, 128-byte swizzle, no row padding) from the maps kmap / vmap; the
// consumers address the swizzled tiles.  Many-kilobyte copies stream at ~7.2 TB/s where one copy per
// 1-2 KB row tops out at 4.6-6.4 TB/s.  TM = false: one cp.async.bulk per row of
// the head group into padded rows (any base pointers, no tensor map).
//
// Units hand over without a CTA-wide stop.  The producer streams every unit's
// tiles back to back; with a unit's first tile it stores the unit's descriptor
// in that stage's slot, (TM) copies the unit's q into the stage's q slot on the
// same barrier, and prefetches the unit's gate into L2.  The consumers learn
// the unit from the slot, so none of the unit's setup waits on global memory,
// and they merge in the stage of the unit's last tile, which they release only
// after the merge: the producer keeps the other stages streaming meanwhile.
//
// ROPE = true (tensor-copy kernels only): one more warp, the RoPE warp.  For the
// unit that ends at the item's position -- the last split of each (item, head
// group) -- it rotates the new token's k, rounds k and v with the engine's
// f32_to_f16 and writes them into cache row pos; the producer copies the tile
// that holds that row only after it.  For every unit it reads the unit's q heads
// unrotated and writes them rotated into the q slot of the unit's first stage,
// whose full barrier then takes its arrive as a second one.  That is
// engine.c:1052-1072 fused into the attention; the producer only waits on a
// counter before a unit's last tile, and the consumers run the same code as
// without it.
template <int HD, int G, bool TM, bool ROPE = false>
__global__ void __launch_bounds__(decode_threads<HD, ROPE>(), 1)
    k_decode(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
             const DecodeParams p, const __grid_constant__ DecodeRope rope) {
    using C = DecodeCfg<HD>;
    using L = DecodeSmem<HD, G, TM, ROPE>;
    static_assert(!ROPE || TM, "the fused RoPE store runs in the tensor-copy kernels");
    constexpr int NCW = C::NCW;
    constexpr int KS = HD / 16;                                       // k-steps (QK) and m-tiles (PV)
    constexpr int DPL = HD / 32;                                      // dims per lane in the merges
    static_assert(G <= 8, "query group fits the MMA's 8 columns");

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the 128-byte swizzle of the tensor copies repeats every 1024 B: align the ring
    uint8_t* smem = TM ? reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023))
                       : smem_raw;
    uint8_t* stages = smem;
    uint8_t* qslots = smem + L::OFF_Q;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    uint64_t* empty = full + C::NST;
    DecodeUnit* descs = reinterpret_cast<DecodeUnit*>(smem + L::OFF_DESC);   // [NST], stride L::DESC
    uint8_t* pt_all = smem + L::OFF_PT;                                // [NCW][PT_BYTES]
    float* mrg_ml = reinterpret_cast<float*>(smem + L::OFF_ML);         // [NCW][G][2]
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_FLAGS);
    int* last_flag = const_cast<int*>(abort_flag) + 1;
    uint32_t* s_range = reinterpret_cast<uint32_t*>(last_flag + 1);    // [2]
    auto desc_at = [&](int s) -> DecodeUnit* {
        return reinterpret_cast<DecodeUnit*>(reinterpret_cast<uint8_t*>(descs) + s * L::DESC);
    };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t HC = p.hc;
    const uint32_t TOK = 16u * NCW / HC;
    const uint32_t ROWB = HC * HD * 2;                                // bytes of one row copy (HC heads)
    const uint32_t RS = TM ? ROWB : ROWB + 16;                        // smem row stride
    const uint32_t TILEB = TOK * RS;
    const uint32_t STAGEB = 2 * TILEB;

    // ---- this CTA's units: a run of the plan (grouped by cta) or one uniform split ----
    if (warp == 0) {
        uint32_t ub = blockIdx.x, ue = blockIdx.x + 1;
        if (p.work) {   // warp-wide 32-way searches: about two dependent loads each
            ub = first_unit_from(p.work, p.n_work, blockIdx.x, lane);
            ue = first_unit_from(p.work, p.n_work, blockIdx.x + 1, lane);
        }
        if (lane == 0) {
            s_range[0] = ub;
            s_range[1] = ue;
        }
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::NST; ++s) {
            mbar_init(&full[s], ROPE ? 2 : 1);   // ROPE: + the RoPE warp (first tiles) or the producer again
            mbar_init(&empty[s], NCW);
        }
        if (ROPE) {
            reinterpret_cast<volatile uint32_t*>(smem + L::OFF_ROWS)[0] = 0u;
            reinterpret_cast<volatile uint32_t*>(smem + L::OFF_ROWS)[1] = 0u;
        }
        abort_flag[0] = 0;
        fence_mbar_init();
    }
    float* s_freq = reinterpret_cast<float*>(smem + L::OFF_FREQ);
    if constexpr (ROPE) {
        for (uint32_t j = threadIdx.x; j < static_cast<uint32_t>(kRopeMaxPairs); j += blockDim.x)
            s_freq[j] = rope.inv_freq[j];
    }
    __syncthreads();
    const uint32_t u_begin = s_range[0], u_end = s_range[1];

    // The ring runs across units: tile gi (counted over all of this CTA's units)
    // uses stage gi % NST with phase (gi / NST) & 1.  Every unit has at least one
    // tile (an empty key range streams one fully masked tile).
    if (warp == NCW) {
        // ================= producer =================
        if (TM && lane == 0) {
            prefetch_tensormap(&kmap);
            prefetch_tensormap(&vmap);
        }
        uint32_t gi = 0;   // tiles issued so far
        bool ok = true;
        uint32_t nrow = 0;   // ROPE: new rows this CTA's units hold, up to the current unit
        for (uint32_t u = u_begin; u < u_end && ok; ++u) {
            const DecodeUnit un = unit_of(p, u, HC);
            const uint32_t ntiles = max(1u, (un.t1 - un.t0 + TOK - 1) / TOK);
            const bool has_row = ROPE && unit_has_new_row(un);
            {   // items live on the device: check what the copies below rely on
                if (item_bad<TM>(p, un.it)) {
                    if (lane == 0) {
                        atomicCAS(p.status, 0, ST_DECODE_BAD_ITEM);
                        *abort_flag = 1;
                    }
                    break;
                }
            }
            // the query heads of the unit's kv heads are one contiguous run [qa, qe)
            uint32_t qa, qn, qb, qm;
            group_of(un.kg * HC, p.n_heads, p.n_kv, qa, qn);
            group_of(un.kg * HC + HC - 1, p.n_heads, p.n_kv, qb, qm);
            const uint32_t qbytes = (qb + qm - qa) * HD * 4;
            const uint16_t* kb = un.it.k + static_cast<size_t>(un.kg) * HC * HD;
            const uint16_t* vb = un.it.v + static_cast<size_t>(un.kg) * HC * HD;
            const int32_t krow0 =
                TM ? static_cast<int32_t>((reinterpret_cast<uint64_t>(un.it.k) - p.kmap_base) / p.row_bytes) : 0;
            const int32_t vrow0 =
                TM ? static_cast<int32_t>((reinterpret_cast<uint64_t>(un.it.v) - p.vmap_base) / p.row_bytes) : 0;
            for (uint32_t i = 0; i < ntiles; ++i, ++gi) {
                const int s = gi % C::NST;
                if (gi >= static_cast<uint32_t>(C::NST)) {
                    if (!warp_wait_bounded(&empty[s], ((gi / C::NST) & 1u) ^ 1u, p.status, ST_DECODE_EMPTY_TIMEOUT,
                                           abort_flag)) {
                        ok = false;
                        break;
                    }
                }
                const uint32_t tile0 = un.t0 + i * TOK;
                const uint32_t nrows = tile0 < un.t1 ? min(TOK, un.t1 - tile0) : 0u;
                uint8_t* kdst = stages + s * STAGEB;
                uint8_t* vdst = kdst + TILEB;
                if constexpr (ROPE) {
                    // a first tile's stage is free: the RoPE warp may fill its q slot and arrive
                    if (i == 0 && lane == 0) st_release_cta(reinterpret_cast<uint32_t*>(smem + L::OFF_ROWS) + 1, gi + 1);
                    // the new row lies in the unit's last tile: the RoPE warp has written it before that
                    // tile is copied
                    if (has_row && i + 1 == ntiles) {
                        if (!warp_wait_count(reinterpret_cast<const uint32_t*>(smem + L::OFF_ROWS), nrow + 1,
                                             p.status, ST_DECODE_FULL_TIMEOUT, abort_flag)) {
                            ok = false;
                            break;
                        }
                        ++nrow;
                    }
                }
                if (i == 0 && lane == 0) {
                    *desc_at(s) = un;   // published by the arrive on full[s] below
                    if (un.it.gate) bulk_prefetch_l2(un.it.gate + static_cast<size_t>(qa) * HD, qbytes);
                }
                if constexpr (TM) {
                    // whole boxes of TOK rows (rows past the unit are masked; past the map, zero-filled)
                    if (lane == 0) {
                        mbar_arrive_expect_tx(&full[s], STAGEB + (i == 0 && !ROPE ? qbytes : 0u));
                        if (i == 0 && !ROPE)
                            bulk_g2s(qslots + s * L::QSLOT, un.it.q + static_cast<size_t>(qa) * HD, qbytes, &full[s]);
                        if (ROPE && i > 0) mbar_arrive(&full[s]);   // a first tile's second arrive: the RoPE warp
                        for (uint32_t c = 0; c < HC * (HD / 64); ++c) {   // HC heads, 64 dims per box
                            const int32_t x = static_cast<int32_t>(un.kg * HC * HD + c * 64);
                            tma_load_2d(kdst + c * TOK * 128, &kmap, x, krow0 + static_cast<int32_t>(tile0), &full[s]);
                            tma_load_2d(vdst + c * TOK * 128, &vmap, x, vrow0 + static_cast<int32_t>(tile0), &full[s]);
                        }
                    }
                    __syncwarp();
                } else {
                    if (lane == 0) mbar_arrive_expect_tx(&full[s], 2u * nrows * ROWB);
                    __syncwarp();
                    for (uint32_t r = lane; r < nrows; r += 32) {
                        const size_t off = static_cast<size_t>(tile0 + r) * p.kv_dim;
                        bulk_g2s(kdst + r * RS, kb + off, ROWB, &full[s]);
                        bulk_g2s(vdst + r * RS, vb + off, ROWB, &full[s]);
                    }
                }
            }
        }
        // No copy may still be in flight when the CTA exits (consumers stop early on an abort).
        for (uint32_t g = (gi > static_cast<uint32_t>(C::NST) ? gi - C::NST : 0); g < gi; ++g) {
            volatile int dummy = 0;
            mbar_wait_bounded(&full[g % C::NST], (g / C::NST) & 1u, p.status, ST_DECODE_FULL_TIMEOUT, &dummy);
        }
        return;
    }

    if constexpr (ROPE) {
        if (warp == NCW + 1) {
            // ================= RoPE warp =================
            // Per unit, in the producer's order: once the producer has claimed the stage of the
            // unit's first tile, the unit's q heads rotated into that stage's q slot and the first
            // tile's second arrive; then the new row (if the unit holds it) written into the cache
            // and counted in rows_done, which the producer waits for before it copies the unit's
            // last tile.  Its global loads wait here, not in the producer.
            uint32_t* rows_done = reinterpret_cast<uint32_t*>(smem + L::OFF_ROWS);
            const uint32_t* claimed = rows_done + 1;
            uint32_t gi = 0, nrow = 0;
            for (uint32_t u = u_begin; u < u_end; ++u) {
                const DecodeUnit un = unit_of(p, u, HC);
                const uint32_t ntiles = max(1u, (un.t1 - un.t0 + TOK - 1) / TOK);
                if (item_bad<TM>(p, un.it)) break;   // the producer reports it and stops
                // the unit's q heads [qa, qa + nq), read before the wait below (all of a lane's
                // loads in flight), so that their latency passes while the ring still streams
                uint32_t qa, qn, qb, qm;
                group_of(un.kg * HC, p.n_heads, p.n_kv, qa, qn);
                group_of(un.kg * HC + HC - 1, p.n_heads, p.n_kv, qb, qm);
                const uint32_t nq = qb + qm - qa, nq4 = nq * HD / 4;
                constexpr uint32_t kQPer = (C::HC_TM_MAX * G * HD / 4 + 31) / 32;
                const float4* q4 = reinterpret_cast<const float4*>(un.it.q + static_cast<size_t>(qa) * HD);
                float4 xq[kQPer];
    #pragma unroll
                for (uint32_t m = 0; m < kQPer; ++m)
                    if (lane + 32 * m < nq4) xq[m] = __ldg(q4 + lane + 32 * m);
                // Wait until the producer has claimed the stage of the unit's first tile: it waited for
                // that stage's release, so full[s] is in this tile's phase and stays there until the
                // arrive below.  (A parity wait on empty[s] could not tell this tile's phase from one
                // two uses earlier: this warp runs up to whole units ahead of the ring.)
                const int s = gi % C::NST;
                if (!warp_wait_count(claimed, gi + 1, p.status, ST_DECODE_EMPTY_TIMEOUT, abort_flag)) break;
                float* slot = reinterpret_cast<float*>(qslots + s * L::QSLOT);
    #pragma unroll
                for (uint32_t m = 0; m < kQPer; ++m)
                    if (lane + 32 * m < nq4) reinterpret_cast<float4*>(slot)[lane + 32 * m] = xq[m];
                __syncwarp();
                rope_q_slot<HD>(slot, nq, s_freq, rope.kind, rope.n_dims, un.it.pos, lane);
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
                if (unit_has_new_row(un)) {
                    // the rows written lie inside the pool
                    const uint64_t kr = (reinterpret_cast<uint64_t>(un.it.k) - p.kmap_base) / p.row_bytes;
                    const uint64_t vr = (reinterpret_cast<uint64_t>(un.it.v) - p.vmap_base) / p.row_bytes;
                    if (kr + un.it.pos >= rope.pool_rows || vr + un.it.pos >= rope.pool_rows) {
                        if (lane == 0) {
                            atomicCAS(p.status, 0, ST_DECODE_BAD_ITEM);
                            *abort_flag = 1;
                        }
                        break;
                    }
                    const YattnDecodeNewRow nr = rope.rows[un.item];
                    if (((reinterpret_cast<uintptr_t>(nr.k) | reinterpret_cast<uintptr_t>(nr.v)) & 15u) != 0) {
                        if (lane == 0) {
                            atomicCAS(p.status, 0, ST_DECODE_BAD_ITEM);
                            *abort_flag = 1;
                        }
                        break;
                    }
                    const size_t h0 = static_cast<size_t>(un.kg) * HC * HD;
                    rope_new_rows<HD>(un.it, nr.k + h0, nr.v + h0, reinterpret_cast<float*>(smem + L::OFF_RSTAGE),
                                      un.kg * HC, HC, p.kv_dim, s_freq, rope.kind, rope.n_dims, lane);
                    __syncwarp();
                    if (lane == 0) st_release_cta(rows_done, ++nrow);
                }
                gi += ntiles;
            }
            return;
        }
    }

    // ================= consumers =================
    const uint32_t hl = warp % HC;                 // head within the group
    const uint32_t sl = warp / HC;                 // 16-token slice of each stage
    const int g8 = lane >> 2;                      // fragment row group: token (S^T), dim (O^T), head (B)
    const int t4 = lane & 3;                       // fragment column pair: heads 2*t4, 2*t4+1
    const int tid = threadIdx.x;                   // 0..32*NCW-1
    const uint32_t nsl = NCW / HC;                 // slice warps per head
    uint8_t* pt = pt_all + warp * C::PT_BYTES;
    const uint32_t pt_u = smem_u32(pt);
    const uint32_t p_off = (lane & 7) * 48 + ((lane >> 3) & 1) * 16;   // P^T
    // ldmatrix lane addresses relative to the warp's 16-row slice of a tile
    const uint32_t slice = (16 * sl) * RS + hl * HD * 2;
    const uint32_t a_off = slice + ((lane & 7) + ((lane >> 3) & 1) * 8) * RS + ((lane >> 4) & 1) * 16;   // K
    const uint32_t v_off = slice + ((lane & 7) + ((lane >> 4) & 1) * 8) * RS + ((lane >> 3) & 1) * 16;   // V^T
    // TM: tiles are HC*HD/64 panels of [TOK rows][128 B] (head hl's panels from hl*HD/64),
    // 16-byte chunk c of row r at c ^ (r & 7)
    const uint32_t rk = 16 * sl + (lane & 15), rv = 16 * sl + (lane & 7) + ((lane >> 4) & 1) * 8;
    const uint32_t hpan = hl * (HD / 64);
    auto k_addr = [&](uint32_t kt, int kk) -> uint32_t {   // K A-fragment, k-step kk
        if constexpr (TM)
            return kt + (hpan + (kk >> 2)) * TOK * 128 + rk * 128 +
                   ((static_cast<uint32_t>(((kk & 3) << 1) + (lane >> 4)) ^ (lane & 7)) << 4);
        else
            return kt + a_off + kk * 32;
    };
    auto v_addr = [&](uint32_t vt, int mt) -> uint32_t {   // V^T A-fragment, m-tile mt
        if constexpr (TM)
            return vt + (hpan + (mt >> 2)) * TOK * 128 + rv * 128 +
                   ((static_cast<uint32_t>(((mt & 3) << 1) + ((lane >> 3) & 1)) ^ (lane & 7)) << 4);
        else
            return vt + v_off + mt * 32;
    };

    uint32_t tb = 0;   // tiles of this CTA's earlier units
    for (uint32_t u = u_begin; u < u_end; ++u) {
        // The unit's first tile brings its descriptor (and q).  All consumer warps
        // take the same way out if the wait gave up, so the named barriers below
        // always see every consumer warp.
        const int s0 = static_cast<int>(tb % C::NST);
        const bool got = warp_wait_bounded(&full[s0], (tb / C::NST) & 1u, p.status, ST_DECODE_FULL_TIMEOUT, abort_flag);
        if (!named_bar_and(1, 32 * NCW, got)) return;
        const DecodeUnit un = *desc_at(s0);
        const YattnDecodeItem& it = un.it;
        const uint32_t kg = un.kg, t0 = un.t0, t1 = un.t1, n_splits = un.n_splits, split = un.split;
        const uint32_t ntiles = max(1u, (t1 - t0 + TOK - 1) / TOK);
        uint32_t gfirst, gcnt, qa, qn;
        group_of(kg * HC + hl, p.n_heads, p.n_kv, gfirst, gcnt);
        group_of(kg * HC, p.n_heads, p.n_kv, qa, qn);

        // Q^T as the MMA B operand: b0 = q[head g8][16kk + 2t4 .. +1], b1 = q[head g8][16kk + 2t4 + 8 .. +9]
        uint32_t qhi[KS][2], qlo[KS][2];
        {
            const bool hv = static_cast<uint32_t>(g8) < gcnt;
            const float* qh = TM ? reinterpret_cast<const float*>(qslots + s0 * L::QSLOT) +
                                       static_cast<size_t>(gfirst - qa + (hv ? g8 : 0)) * HD
                                 : it.q + static_cast<size_t>(gfirst + (hv ? g8 : 0)) * HD;
    #pragma unroll
            for (int kk = 0; kk < KS; ++kk) {
                float2 x0 = make_float2(0.f, 0.f), x1 = make_float2(0.f, 0.f);
                if (hv) {
                    x0 = *reinterpret_cast<const float2*>(qh + kk * 16 + 2 * t4);
                    x1 = *reinterpret_cast<const float2*>(qh + kk * 16 + 2 * t4 + 8);
                }
                split_h2(x0.x, x0.y, qhi[kk][0], qlo[kk][0]);
                split_h2(x1.x, x1.y, qhi[kk][1], qlo[kk][1]);
            }
        }
        float oc[KS][4];
    #pragma unroll
        for (int mt = 0; mt < KS; ++mt) oc[mt][0] = oc[mt][1] = oc[mt][2] = oc[mt][3] = 0.f;
        float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;    // heads 2*t4 and 2*t4+1

        for (uint32_t i = 0; i < ntiles; ++i) {
            const uint32_t gi = tb + i;
            const int s = gi % C::NST;
            if (i > 0 && !warp_wait_bounded(&full[s], (gi / C::NST) & 1u, p.status, ST_DECODE_FULL_TIMEOUT, abort_flag))
                break;
            const uint32_t tile0 = t0 + i * TOK;
            const uint32_t nrows = tile0 < t1 ? min(TOK, t1 - tile0) : 0u;
            const int nvalid = max(0, min(16, static_cast<int>(nrows) - static_cast<int>(16 * sl)));
            if (nvalid > 0) {
                const uint32_t kt = smem_u32(stages + s * STAGEB);
                const uint32_t vt = kt + TILEB;
                // ---- S^T = K Q^T ----
                // four independent accumulation chains (q hi / lo x even / odd k-step),
                // so the MMA latency is paid KS/2 times instead of 2*KS
                float sc[4], sc1[4] = {0.f, 0.f, 0.f, 0.f}, sc2[4] = {0.f, 0.f, 0.f, 0.f},
                             sc3[4] = {0.f, 0.f, 0.f, 0.f};
                sc[0] = sc[1] = sc[2] = sc[3] = 0.f;
    #pragma unroll
                for (int kk = 0; kk < KS; kk += 2) {
                    uint32_t a[4], b[4];
                    ldsm_x4(k_addr(kt, kk), a);
                    ldsm_x4(k_addr(kt, kk + 1), b);
                    mma16816(sc, a, qhi[kk][0], qhi[kk][1]);
                    mma16816(sc1, b, qhi[kk + 1][0], qhi[kk + 1][1]);
                    mma16816(sc2, a, qlo[kk][0], qlo[kk][1]);
                    mma16816(sc3, b, qlo[kk + 1][0], qlo[kk + 1][1]);
                }
    #pragma unroll
                for (int r = 0; r < 4; ++r) sc[r] = (sc[r] + sc1[r]) + (sc2[r] + sc3[r]);
                // sc: [0] = (token g8, head 2t4), [1] = (g8, 2t4+1), [2] = (g8+8, 2t4), [3] = (g8+8, 2t4+1)
                const bool v0 = g8 < nvalid, v1 = g8 + 8 < nvalid;
                const float s0 = v0 ? sc[0] * p.scale_log2 : -INFINITY;
                const float s1 = v0 ? sc[1] * p.scale_log2 : -INFINITY;
                const float s2 = v1 ? sc[2] * p.scale_log2 : -INFINITY;
                const float s3 = v1 ? sc[3] * p.scale_log2 : -INFINITY;
                float mx_a = fmaxf(s0, s2), mx_b = fmaxf(s1, s3);
    #pragma unroll
                for (int o = 4; o <= 16; o <<= 1) {
                    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, o));
                    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, o));
                }
                const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
                const float al_a = ex2_approx(m_a - mn_a), al_b = ex2_approx(m_b - mn_b);
                const float p0 = ex2_approx(s0 - mn_a), p1 = ex2_approx(s1 - mn_b);
                const float p2 = ex2_approx(s2 - mn_a), p3 = ex2_approx(s3 - mn_b);
                float sum_a = p0 + p2, sum_b = p1 + p3;
    #pragma unroll
                for (int o = 4; o <= 16; o <<= 1) {
                    sum_a += __shfl_xor_sync(0xffffffffu, sum_a, o);
                    sum_b += __shfl_xor_sync(0xffffffffu, sum_b, o);
                }
                l_a = l_a * al_a + sum_a;
                l_b = l_b * al_b + sum_b;
                m_a = mn_a;
                m_b = mn_b;
                // ---- P^T (rows = heads, 16 tokens, 48 B row stride) as fp16 hi and lo planes ----
                {
                    uint32_t h01, l01, h23, l23;
                    split_h2(p0, p1, h01, l01);      // (token g8: heads 2t4, 2t4+1)
                    split_h2(p2, p3, h23, l23);      // (token g8+8: heads 2t4, 2t4+1)
                    uint16_t* hp = reinterpret_cast<uint16_t*>(pt);
                    uint16_t* lp = reinterpret_cast<uint16_t*>(pt + 384);
                    const int ra = (2 * t4) * 24, rb = (2 * t4 + 1) * 24;   // row offsets in halves
                    hp[ra + g8] = static_cast<uint16_t>(h01);
                    hp[rb + g8] = static_cast<uint16_t>(h01 >> 16);
                    hp[ra + g8 + 8] = static_cast<uint16_t>(h23);
                    hp[rb + g8 + 8] = static_cast<uint16_t>(h23 >> 16);
                    lp[ra + g8] = static_cast<uint16_t>(l01);
                    lp[rb + g8] = static_cast<uint16_t>(l01 >> 16);
                    lp[ra + g8 + 8] = static_cast<uint16_t>(l23);
                    lp[rb + g8 + 8] = static_cast<uint16_t>(l23 >> 16);
                }
                __syncwarp();
                uint32_t ph0, ph1, pl0, pl1;
                ldsm_x2(pt_u + p_off, ph0, ph1);
                ldsm_x2(pt_u + 384 + p_off, pl0, pl1);
                // ---- O^T = O^T * alpha + V^T P^T ----
                // V rows past nvalid hold stale (or never written) shared memory: their
                // p is 0, but 0 * NaN would still poison the MMA, so zero those lanes.
                // The A fragment holds tokens 2t4, 2t4+1 (a0, a1) and 2t4+8, 2t4+9 (a2, a3).
                uint32_t vm01 = 0xffffffffu, vm23 = 0xffffffffu;
                if (nvalid < 16) {
                    vm01 = (2 * t4 < nvalid ? 0x0000ffffu : 0u) | (2 * t4 + 1 < nvalid ? 0xffff0000u : 0u);
                    vm23 = (2 * t4 + 8 < nvalid ? 0x0000ffffu : 0u) | (2 * t4 + 9 < nvalid ? 0xffff0000u : 0u);
                }
    #pragma unroll
                for (int mt = 0; mt < KS; ++mt) {
                    oc[mt][0] *= al_a;
                    oc[mt][1] *= al_b;
                    oc[mt][2] *= al_a;
                    oc[mt][3] *= al_b;
                    uint32_t a[4];
                    ldsm_x4_t(v_addr(vt, mt), a);
                    a[0] &= vm01;
                    a[1] &= vm01;
                    a[2] &= vm23;
                    a[3] &= vm23;
                    mma16816(oc[mt], a, ph0, ph1);
                    mma16816(oc[mt], a, pl0, pl1);
                }
                __syncwarp();   // P^T is rewritten by the next step
            }
            __syncwarp();
            // the last tile's stage is released after the merge below has used it
            if (lane == 0 && i + 1 < ntiles) mbar_arrive(&empty[s]);
        }

        // ---- merge the consumer warps in the last tile's stage ----
        // No early exit on the abort flag here: every consumer warp must reach the
        // same named barriers (a timed-out unit just writes meaningless partials).
        const int s_last = static_cast<int>((tb + ntiles - 1) % C::NST);
        float* mrg_o = reinterpret_cast<float*>(stages + s_last * STAGEB);   // [NCW][G][HD]
        named_bar_sync(1, 32 * NCW);
        {
            const int ha = 2 * t4, hb = 2 * t4 + 1;
            if (g8 == 0) {
                if (ha < G) {
                    mrg_ml[(warp * G + ha) * 2 + 0] = m_a;
                    mrg_ml[(warp * G + ha) * 2 + 1] = l_a;
                }
                if (hb < G) {
                    mrg_ml[(warp * G + hb) * 2 + 0] = m_b;
                    mrg_ml[(warp * G + hb) * 2 + 1] = l_b;
                }
            }
    #pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
                const int d0 = mt * 16 + g8, d1 = d0 + 8;
                if (ha < G) {
                    mrg_o[(warp * G + ha) * HD + d0] = oc[mt][0];
                    mrg_o[(warp * G + ha) * HD + d1] = oc[mt][2];
                }
                if (hb < G) {
                    mrg_o[(warp * G + hb) * HD + d0] = oc[mt][1];
                    mrg_o[(warp * G + hb) * HD + d1] = oc[mt][3];
                }
            }
        }
        named_bar_sync(1, 32 * NCW);

        // One warp per output row (kv head h of the group, query head g); lane owns
        // dims lane + 32 i.  The row's nsl slice partials are combined with
        // log-sum-exp weights.
        // this CTA holds the whole key range of its (item, head group), and writes the result itself
        const bool single = n_splits == 1 && !p.defer_merge;
        for (uint32_t row = warp; row < HC * G; row += NCW) {
            const uint32_t h = row / G, g = row % G;
            uint32_t hfirst, hcnt;
            group_of(kg * HC + h, p.n_heads, p.n_kv, hfirst, hcnt);
            if (g >= hcnt) continue;
            float M = -INFINITY;
            for (uint32_t j = 0; j < nsl; ++j) M = fmaxf(M, mrg_ml[((h + j * HC) * G + g) * 2]);
            float acc[DPL], l = 0.f;
    #pragma unroll
            for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
            for (uint32_t j = 0; j < nsl; ++j) {
                const uint32_t w = h + j * HC;
                const float mw = mrg_ml[(w * G + g) * 2];
                const float sc = (mw == -INFINITY) ? 0.f : ex2_approx(mw - M);
                l += sc * mrg_ml[(w * G + g) * 2 + 1];
    #pragma unroll
                for (int i = 0; i < DPL; ++i) acc[i] += sc * mrg_o[(w * G + g) * HD + lane + 32 * i];
            }
            const uint32_t hh = hfirst + g;
            if (single && p.partial_only) {
    #pragma unroll
                for (int i = 0; i < DPL; ++i) p.out_o[static_cast<size_t>(hh) * HD + lane + 32 * i] = acc[i];
                if (lane == 0) {
                    p.out_ml[hh * 2 + 0] = M;
                    p.out_ml[hh * 2 + 1] = l;
                }
            } else if (single) {
                const float inv_l = 1.0f / l;
    #pragma unroll
                for (int i = 0; i < DPL; ++i) {
                    const size_t idx = static_cast<size_t>(hh) * HD + lane + 32 * i;
                    float r = acc[i] * inv_l;
                    if (it.gate) r *= 1.0f / (1.0f + __expf(-it.gate[idx]));
                    it.out[idx] = r;
                }
            } else {
                const size_t slot = static_cast<size_t>(un.part_base + h * n_splits + split) * G + g;
    #pragma unroll
                for (int i = 0; i < DPL; ++i) p.part_o[slot * HD + lane + 32 * i] = acc[i];
                if (lane == 0) *reinterpret_cast<float2*>(&p.part_ml[slot * 2]) = make_float2(M, l);
            }
        }
        named_bar_sync(1, 32 * NCW);   // every warp is done with the merge area
        if (lane == 0) mbar_arrive(&empty[s_last]);
        tb += ntiles;
        if (single || p.defer_merge) continue;

        // ---- last split of this (item, head group) merges all splits ----
        __threadfence();
        named_bar_sync(1, 32 * NCW);
        if (tid == 0) {
            const uint32_t prev = atomicAdd(&p.counters[un.group], 1u);
            last_flag[0] = (prev == n_splits - 1) ? 1 : 0;
        }
        named_bar_sync(1, 32 * NCW);
        if (!last_flag[0]) continue;
        __threadfence();
        // One warp per row; lane owns dims [lane*DPL, +DPL).  Up to SMAX splits,
        // every load (each split's (m, l) and o, and the gate, which the unit's
        // first tile prefetched into L2) is issued before any is used, so a row
        // costs one memory round trip.  More splits go 32 per round: lanes over
        // splits for (m, l), weights to the lanes by shuffles, o loads in flight.
        constexpr int SMAX = 16 / DPL > 4 ? 16 / DPL : 4;
        for (uint32_t row = warp; row < HC * G; row += NCW) {
            const uint32_t h = row / G, g = row % G;
            uint32_t hfirst, hcnt;
            group_of(kg * HC + h, p.n_heads, p.n_kv, hfirst, hcnt);
            if (g >= hcnt) continue;
            const size_t base = static_cast<size_t>(un.part_base + h * n_splits);
            const uint32_t hh = hfirst + g;
            const size_t ob = static_cast<size_t>(hh) * HD + lane * DPL;
            float gt[DPL];
            if (!p.partial_only && it.gate) ldcg_vec<DPL>(it.gate + ob, gt);
            float M = -INFINITY, lsum = 0.f, acc[DPL];
    #pragma unroll
            for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
            if (n_splits <= static_cast<uint32_t>(SMAX)) {
                float2 ml[SMAX];
                float o[SMAX][DPL];
    #pragma unroll
                for (int sx = 0; sx < SMAX; ++sx) {
                    if (static_cast<uint32_t>(sx) < n_splits) {
                        const size_t slot = (base + sx) * G + g;
                        ml[sx] = __ldcg(reinterpret_cast<const float2*>(&p.part_ml[slot * 2]));
                        ldcg_vec<DPL>(&p.part_o[slot * HD + lane * DPL], o[sx]);
                    }
                }
    #pragma unroll
                for (int sx = 0; sx < SMAX; ++sx)
                    if (static_cast<uint32_t>(sx) < n_splits) M = fmaxf(M, ml[sx].x);
    #pragma unroll
                for (int sx = 0; sx < SMAX; ++sx) {
                    if (static_cast<uint32_t>(sx) < n_splits) {
                        const float w = (ml[sx].x == -INFINITY) ? 0.f : ex2_approx(ml[sx].x - M);
                        lsum += w * ml[sx].y;
    #pragma unroll
                        for (int i = 0; i < DPL; ++i) acc[i] += w * o[sx][i];
                    }
                }
            } else {
                float mj = -INFINITY;
                for (uint32_t sidx = lane; sidx < n_splits; sidx += 32)
                    mj = fmaxf(mj, __ldcg(&p.part_ml[((base + sidx) * G + g) * 2]));
    #pragma unroll
                for (int o = 16; o > 0; o >>= 1) mj = fmaxf(mj, __shfl_xor_sync(0xffffffffu, mj, o));
                M = mj;
                for (uint32_t c0 = 0; c0 < n_splits; c0 += 32) {
                    const float2 mlc = c0 + lane < n_splits ? __ldcg(reinterpret_cast<const float2*>(
                                                                   &p.part_ml[((base + c0 + lane) * G + g) * 2]))
                                                             : make_float2(-INFINITY, 0.f);
                    const float wl = (mlc.x == -INFINITY) ? 0.f : ex2_approx(mlc.x - M);
                    lsum += wl * mlc.y;
                    const uint32_t nc = min(32u, n_splits - c0);
    #pragma unroll 4
                    for (uint32_t j = 0; j < nc; ++j) {
                        const float w = __shfl_sync(0xffffffffu, wl, static_cast<int>(j));
                        float o[DPL];
                        ldcg_vec<DPL>(&p.part_o[((base + c0 + j) * G + g) * HD + lane * DPL], o);
    #pragma unroll
                        for (int i = 0; i < DPL; ++i) acc[i] += w * o[i];
                    }
                }
    #pragma unroll
                for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
            }
            if (p.partial_only) {   // merged (m, l, o) of the whole range, for a cross-GPU merge
    #pragma unroll
                for (int i = 0; i < DPL; ++i) p.out_o[ob + i] = acc[i];
                if (lane == 0) {
                    p.out_ml[hh * 2 + 0] = M;
                    p.out_ml[hh * 2 + 1] = lsum;
                }
                continue;
            }
            const float inv_l = 1.0f / lsum;
    #pragma unroll
            for (int i = 0; i < DPL; ++i) {
                float r = acc[i] * inv_l;
                if (it.gate) r *= 1.0f / (1.0f + __expf(-gt[i]));
                it.out[ob + i] = r;
            }
        }
        if (tid == 0) p.counters[un.group] = 0u;   // ready for the next launch
    }
}

// ------------------------------------------------- parallel merge of many splits
// One CTA per query head merges the head's ns split partials with log-sum-exp
// weights.  Every split's (m, l) is loaded in one round (threads over splits);
// the global max and the weights w_s = 2^(m_s - M) go to shared memory; then
// warp w sums w_s o_s over the splits s = w (mod 8) with lanes over dims and the
// loads of 8 splits in flight at a time, and the 8 warps' sums are added.  Used
// when one query has more splits than the last-arriving CTA merges quickly, and
// always for the cross-GPU exchange (EX), which then sends the merged head to
// every rank and merges the ranks' heads (exchange.cuh).
constexpr uint32_t kInKernelMergeMax = 8;
constexpr uint32_t kMergeMaxSplits = 1024;

template <bool EX>
__global__ void __launch_bounds__(256) k_merge_splits(const float* __restrict__ part_ml,
                                                      const float* __restrict__ part_o, uint32_t ns,
                                                      uint32_t n_heads, uint32_t n_kv, uint32_t G, uint32_t hd,
                                                      float* out, const float* gate, float* out_ml, float* out_o,
                                                      const ExchangeArgs ex, int* status) {
    __shared__ float s_w[kMergeMaxSplits];   // m_s, then the weight of split s
    __shared__ float s_l[kMergeMaxSplits];
    __shared__ float s_red[2][8];
    __shared__ float s_o[8][256];
    __shared__ uint32_t s_epoch;
    const uint32_t hh = blockIdx.x;
    const uint32_t kvh = hh * n_kv / n_heads;
    uint32_t gfirst, gcnt;
    group_of(kvh, n_heads, n_kv, gfirst, gcnt);
    const uint32_t gl = hh - gfirst;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int dl = static_cast<int>(hd / 32);     // 2, 4 or 8 dims per lane
    auto slot = [&](uint32_t s) { return (static_cast<size_t>(kvh) * ns + s) * G + gl; };
    if constexpr (EX) exchange_epoch(ex, &s_epoch);
    // ---- every split's (m, l); the maximum m ----
    float mloc = -INFINITY;
    for (uint32_t s = threadIdx.x; s < ns; s += blockDim.x) {
        const float2 ml = __ldcg(reinterpret_cast<const float2*>(part_ml + slot(s) * 2));
        s_w[s] = ml.x;
        s_l[s] = ml.y;
        mloc = fmaxf(mloc, ml.x);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
    if (lane == 0) s_red[0][warp] = mloc;
    __syncthreads();
    float M = s_red[0][0];
#pragma unroll
    for (int w = 1; w < 8; ++w) M = fmaxf(M, s_red[0][w]);
    // ---- weights, the weighted sum of l ----
    float lloc = 0.f;
    for (uint32_t s = threadIdx.x; s < ns; s += blockDim.x) {
        const float m = s_w[s];
        const float w = (m == -INFINITY) ? 0.f : ex2_approx(m - M);
        s_w[s] = w;
        lloc += w * s_l[s];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lloc += __shfl_xor_sync(0xffffffffu, lloc, o);
    if (lane == 0) s_red[1][warp] = lloc;
    __syncthreads();
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) L += s_red[1][w];
    // ---- sum of w_s o_s: warp w takes splits w, w + 8, ...; 8 splits' loads in flight ----
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (uint32_t s0 = warp; s0 < ns; s0 += 64) {
        float ov[8][8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t s = s0 + 8 * j;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                ov[j][i] = (s < ns && i < dl) ? __ldcg(part_o + slot(s) * hd + lane + 32 * i) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t s = s0 + 8 * j;
            const float w = s < ns ? s_w[s] : 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] += w * ov[j][i];
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if (i < dl) s_o[warp][lane + 32 * i] = acc[i];
    __syncthreads();
    for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x) {
        float o = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) o += s_o[w][d];
        if constexpr (EX) {
            s_o[0][d] = o;   // the merged head, for the exchange (each d read and written by one thread)
            continue;
        }
        if (out_ml) {   // merged partial of the whole range
            out_o[static_cast<size_t>(hh) * hd + d] = o;
            if (d == 0) {
                out_ml[hh * 2 + 0] = M;
                out_ml[hh * 2 + 1] = L;
            }
            continue;
        }
        float r = o / L;
        if (gate) r *= 1.0f / (1.0f + __expf(-gate[static_cast<size_t>(hh) * hd + d]));
        out[static_cast<size_t>(hh) * hd + d] = r;
    }
    if constexpr (EX) {
        __syncthreads();
        const uint32_t epoch = s_epoch;
        exchange_head(ex, epoch, n_heads, hd, hh, M, L, s_o[0], out, gate, status);
        exchange_finish(ex, epoch);
    }
}

// ---------------------------------------------------------------- merge kernel
// Part s of head hh: (m, l) at ml[s*ml_stride + 2*hh], o at o[s*o_stride + hh*hd].
__global__ void k_merge_partials(float* out, const float* ml, const float* o, uint32_t n_parts, uint32_t n_heads,
                                 uint32_t hd, const float* gate, size_t ml_stride, size_t o_stride) {
    const uint32_t hh = blockIdx.x;
    for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x) {
        float M = -INFINITY;
        for (uint32_t s = 0; s < n_parts; ++s) {
            const float* mls = ml + s * ml_stride + 2 * hh;
            if (mls[1] > 0.f) M = fmaxf(M, mls[0]);
        }
        float acc = 0.f, l = 0.f;
        for (uint32_t s = 0; s < n_parts; ++s) {
            const float* mls = ml + s * ml_stride + 2 * hh;
            const float ls = mls[1];
            if (!(ls > 0.f)) continue;
            const float sc = ex2_approx(mls[0] - M);
            acc += sc * o[s * o_stride + static_cast<size_t>(hh) * hd + d];
            l += sc * ls;
        }
        float r = acc / l;
        if (gate) r *= 1.0f / (1.0f + __expf(-gate[static_cast<size_t>(hh) * hd + d]));
        out[static_cast<size_t>(hh) * hd + d] = r;
    }
}

// ------------------------------------------------------------------ dispatch
template <int HD, int G, bool TM, bool ROPE>
int launch_t(const DecodeParams& p, const CUtensorMap& km, const CUtensorMap& vm, const DecodeRope& rope,
             uint32_t grid, cudaStream_t st, char* err, size_t errlen) {
    const size_t smem = DecodeSmem<HD, G, TM, ROPE>::BYTES;
    if (TM && p.hc > static_cast<uint32_t>(DecodeCfg<HD>::HC_TM_MAX)) {
        set_err(err, errlen, "decode: %u kv heads per CTA with tensor copies (max %d)", p.hc, DecodeCfg<HD>::HC_TM_MAX);
        return -1;
    }
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(k_decode<HD, G, TM, ROPE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) {
            set_err(err, errlen, "decode: smem attribute: %s", cudaGetErrorString(e));
            return -1;
        }
        attr_done[dev] = true;
    }
    k_decode<HD, G, TM, ROPE><<<grid, decode_threads<HD, ROPE>(), smem, st>>>(km, vm, p, rope);
    YATTN_CHECK_LAUNCH(err, errlen, "decode");
    return 0;
}

template <int HD, bool TM, bool ROPE>
int launch_hd(const DecodeParams& p, const CUtensorMap& km, const CUtensorMap& vm, const DecodeRope& rope,
              uint32_t gmax, uint32_t grid, cudaStream_t st, char* err, size_t errlen) {
    switch (gmax) {
        case 1: return launch_t<HD, 1, TM, ROPE>(p, km, vm, rope, grid, st, err, errlen);
        case 2: return launch_t<HD, 2, TM, ROPE>(p, km, vm, rope, grid, st, err, errlen);
        case 3: return launch_t<HD, 3, TM, ROPE>(p, km, vm, rope, grid, st, err, errlen);
        case 4: return launch_t<HD, 4, TM, ROPE>(p, km, vm, rope, grid, st, err, errlen);
        case 5: return launch_t<HD, 5, TM, ROPE>(p, km, vm, rope, grid, st, err, errlen);
        case 6: return launch_t<HD, 6, TM, ROPE>(p, km, vm, rope, grid, st, err, errlen);
        case 7: return launch_t<HD, 7, TM, ROPE>(p, km, vm, rope, grid, st, err, errlen);
        case 8: return launch_t<HD, 8, TM, ROPE>(p, km, vm, rope, grid, st, err, errlen);
        default: set_err(err, errlen, "decode: %u query heads per kv head (max 8)", gmax); return -1;
    }
}

// tm: tensor-copy kernels (p.hc must be 1, km / vm valid); otherwise the row-copy kernels.
// rope (tensor-copy kernels only): the fused RoPE + KV store variant.
int launch_decode(const DecodeParams& p, bool tm, const CUtensorMap* km, const CUtensorMap* vm, uint32_t head_dim,
                  uint32_t grid, cudaStream_t st, char* err, size_t errlen, const DecodeRope* rope = nullptr) {
    const uint32_t gmax = (p.n_heads + p.n_kv - 1) / p.n_kv;
    static const CUtensorMap none{};
    static const DecodeRope no_rope{};
    const CUtensorMap& k = km ? *km : none;
    const CUtensorMap& v = vm ? *vm : none;
    if (rope) {
        if (!tm) {
            set_err(err, errlen, "decode: the fused RoPE store needs the pooled (tensor-copy) path");
            return -1;
        }
        switch (head_dim) {
            case 64: return launch_hd<64, true, true>(p, k, v, *rope, gmax, grid, st, err, errlen);
            case 128: return launch_hd<128, true, true>(p, k, v, *rope, gmax, grid, st, err, errlen);
            case 256: return launch_hd<256, true, true>(p, k, v, *rope, gmax, grid, st, err, errlen);
            default: break;
        }
    } else if (tm) {
        switch (head_dim) {
            case 64: return launch_hd<64, true, false>(p, k, v, no_rope, gmax, grid, st, err, errlen);
            case 128: return launch_hd<128, true, false>(p, k, v, no_rope, gmax, grid, st, err, errlen);
            case 256: return launch_hd<256, true, false>(p, k, v, no_rope, gmax, grid, st, err, errlen);
            default: break;
        }
    } else {
        switch (head_dim) {
            case 64: return launch_hd<64, false, false>(p, k, v, no_rope, gmax, grid, st, err, errlen);
            case 128: return launch_hd<128, false, false>(p, k, v, no_rope, gmax, grid, st, err, errlen);
            case 256: return launch_hd<256, false, false>(p, k, v, no_rope, gmax, grid, st, err, errlen);
            default: break;
        }
    }
    set_err(err, errlen, "decode: head_dim %u not supported (64/128/256)", head_dim);
    return -1;
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

// Uniform split length aiming at `target` CTAs for `work` = keys x head groups.
uint32_t auto_split(uint64_t work, uint32_t target) {
    uint64_t len = (work + target - 1) / target;
    len = std::max<uint64_t>(len, 128);
    len = (len + kSplitQuant - 1) / kSplitQuant * kSplitQuant;
    return static_cast<uint32_t>(std::min<uint64_t>(len, 1u << 30));
}

// Workspace: merge counters (one per multi-split (item, head group)), then
// (m, l) and o of every partial slot (one per (item, kv head, split)).
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

// Uniform-split parameters for one query over keys [t_begin, t_end).
struct SinglePlan {
    uint32_t hc, n_groups_kv, split, ns, n_parts, n_groups;
};

// Single queries run the tensor-copy kernels (tm_heads_per_cta heads per CTA).
SinglePlan plan_single(uint32_t ntok, uint32_t n_kv, uint32_t hd, uint32_t target) {
    SinglePlan s{};
    s.hc = tm_heads_per_cta(n_kv, hd);
    s.n_groups_kv = n_kv / s.hc;
    s.split = auto_split(static_cast<uint64_t>(ntok) * s.n_groups_kv, target);
    s.ns = (ntok + s.split - 1) / s.split;
    s.n_parts = s.ns > 1 ? n_kv * s.ns : 0;
    s.n_groups = s.ns > 1 ? s.n_groups_kv : 0;
    return s;
}

DecodeParams single_params(const SinglePlan& sp, float* out, const float* q, const uint16_t* k, const uint16_t* v,
                           const float* gate, uint32_t t_begin, uint32_t t_end, uint32_t n_heads, uint32_t n_kv,
                           uint32_t hd, uint32_t kv_dim) {
    DecodeParams p{};
    p.item0.q = q;
    p.item0.out = out;
    p.item0.k = k;
    p.item0.v = v;
    p.item0.gate = gate;
    p.item0.pos = t_end - 1;
    p.split_len = sp.split;
    p.n_splits0 = sp.ns;
    p.t_base = t_begin;
    p.t_end0 = t_end;
    p.n_heads = n_heads;
    p.n_kv = n_kv;
    p.kv_dim = kv_dim;
    p.hc = sp.hc;
    p.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(hd));
    return p;
}

// Launches a single-query decode; with many splits the merge runs as a
// separate parallel kernel instead of in the last-arriving CTA, and with ex that
// kernel also exchanges the merged heads with the other ranks.
int launch_single(DecodeParams& p, const SinglePlan& sp, uint32_t hd, cudaStream_t st, char* err, size_t errlen,
                  const ExchangeArgs* ex = nullptr) {
    const bool defer = ex || sp.ns > kInKernelMergeMax;
    p.defer_merge = defer ? 1 : 0;
    if (defer && sp.ns > kMergeMaxSplits) {
        set_err(err, errlen, "decode: %u splits per head group (at most %u)", sp.ns, kMergeMaxSplits);
        return -1;
    }
    // K and V maps over keys [0, t_end) of this layer; boxes of one stage (16 tokens per consumer warp)
    CUtensorMap km, vm;
    const uint32_t box_rows = 16u * (hd >= 256 ? DecodeCfg<256>::NCW : DecodeCfg<128>::NCW) / p.hc;
    if (encode_kv_map(&km, p.item0.k, p.kv_dim, p.t_end0, box_rows, err, errlen) ||
        encode_kv_map(&vm, p.item0.v, p.kv_dim, p.t_end0, box_rows, err, errlen))
        return -1;
    p.kmap_base = reinterpret_cast<uint64_t>(p.item0.k);
    p.vmap_base = reinterpret_cast<uint64_t>(p.item0.v);
    p.row_bytes = p.kv_dim * 2;
    if (launch_decode(p, true, &km, &vm, hd, sp.ns * sp.n_groups_kv, st, err, errlen)) return -1;
    if (!defer) return 0;
    const uint32_t G = gmax_of(p.n_heads, p.n_kv);
    if (ex)
        k_merge_splits<true><<<p.n_heads, 256, 0, st>>>(p.part_ml, p.part_o, sp.ns, p.n_heads, p.n_kv, G, hd,
                                                         p.item0.out, p.item0.gate, nullptr, nullptr, *ex, p.status);
    else
        k_merge_splits<false><<<p.n_heads, 256, 0, st>>>(p.part_ml, p.part_o, sp.ns, p.n_heads, p.n_kv, G, hd,
                                                          p.item0.out, p.item0.gate,
                                                          p.partial_only ? p.out_ml : nullptr, p.out_o,
                                                          ExchangeArgs{}, p.status);
    YATTN_CHECK_LAUNCH(err, errlen, "decode merge");
    return 0;
}

}  // namespace

// Single query, uniform splits, internal or given workspace.  Shared by the
// drop-in decode, yattn_attn_decode and yattn_decode_partial.
int decode_single(float* out, const float* q, const uint16_t* k, const uint16_t* v, const float* gate,
                  uint32_t t_begin, uint32_t t_end, uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t kv_dim,
                  float* partial_ml, float* partial_o, void* ws, size_t ws_bytes, cudaStream_t st, char* err,
                  size_t errlen, const ExchangeArgs* ex = nullptr) {
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
    SinglePlan sp = plan_single(t_end - t_begin, n_kv, hd, static_cast<uint32_t>(ctx->num_sms));
    if (ex && sp.ns == 1) {   // the exchange merges split slots: one split per head group still writes one
        sp.n_parts = n_kv;
        sp.n_groups = sp.n_groups_kv;
    }
    DecodeParams p = single_params(sp, out, q, k, v, gate, t_begin, t_end, n_heads, n_kv, hd, kv_dim);
    p.status = ctx->status;
    p.partial_only = partial_ml != nullptr ? 1 : 0;
    p.out_ml = partial_ml;
    p.out_o = partial_o;
    if (sp.n_parts > 0) {
        const size_t need = ws_bytes_for(sp.n_parts, sp.n_groups, gmax, hd);
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
        carve_ws(ws, sp.n_parts, sp.n_groups, gmax, p);
    }
    return launch_single(p, sp, hd, st, err, errlen, ex);
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

namespace {
// tm: heads per CTA of the tensor-copy kernels (pooled run), else of the row-copy kernels.
int decode_plan_impl(const uint32_t* pos_host, uint32_t n_items, uint32_t n_kv_heads, uint32_t head_dim,
                     uint32_t split_tokens, uint32_t target_ctas, bool tm, YattnDecodeWork* work_host,
                     uint32_t work_cap, uint32_t* n_work, uint32_t* n_parts, uint32_t* n_groups, char* err,
                     size_t errlen) {
    if (!pos_host || !work_host || !n_work || !n_parts || !n_groups || n_kv_heads == 0 || n_kv_heads > 65535) {
        set_err(err, errlen, "decode_plan: bad arguments");
        return -1;
    }
    if (head_dim != 64 && head_dim != 128 && head_dim != 256) {
        set_err(err, errlen, "decode_plan: head_dim %u not supported (64/128/256)", head_dim);
        return -1;
    }
    const uint32_t hc = tm ? tm_heads_per_cta(n_kv_heads, head_dim) : heads_per_cta(n_kv_heads, head_dim);
    const uint32_t nkg = n_kv_heads / hc;
    uint64_t total = 0;
    for (uint32_t i = 0; i < n_items; ++i) total += static_cast<uint64_t>(pos_host[i]) + 1;
    total *= nkg;
    if (target_ctas == 0) target_ctas = static_cast<uint32_t>(dev_num_sms());
    std::vector<YattnDecodeWork> w;
    uint32_t parts = 0, groups = 0;
    // uniform splits of `split` keys, one unit per CTA, longest units first
    auto build_uniform = [&](uint32_t split) -> int {
        w.clear();
        parts = groups = 0;
        for (uint32_t i = 0; i < n_items; ++i) {
            const uint32_t ntok = pos_host[i] + 1;
            const uint32_t ns = (ntok + split - 1) / split;
            if (ns > 65535) {
                set_err(err, errlen, "decode_plan: %u splits for item %u (max 65535)", ns, i);
                return -1;
            }
            for (uint32_t kg = 0; kg < nkg; ++kg) {
                for (uint32_t s = 0; s < ns; ++s) {
                    YattnDecodeWork x{};
                    x.item = i;
                    x.kv_head = static_cast<uint16_t>(kg * hc);
                    x.n_splits = static_cast<uint16_t>(ns);
                    x.split = s;
                    x.t_begin = s * split;
                    x.t_end = std::min(ntok, (s + 1) * split);
                    x.part_base = ns > 1 ? parts : 0u;
                    x.group = ns > 1 ? groups : 0u;
                    w.push_back(x);
                }
                if (ns > 1) {
                    parts += hc * ns;     // one slot per (kv head of the group, split)
                    groups += 1;
                }
            }
        }
        std::stable_sort(w.begin(), w.end(), [](const YattnDecodeWork& a, const YattnDecodeWork& b) {
            return (a.t_end - a.t_begin) > (b.t_end - b.t_begin);
        });
        for (size_t u = 0; u < w.size(); ++u) w[u].cta = static_cast<uint32_t>(u);
        return 0;
    };
    if (split_tokens) {
        if (build_uniform((split_tokens + kSplitQuant - 1) / kSplitQuant * kSplitQuant) != 0) return -1;
    } else {
        // Balanced: the (item, head group) key ranges laid end to end, cut into
        // chunks of `chunk` keys; CTA c streams the keys of chunk c as one unit per
        // range it touches.  A CTA's second and later units are charged
        // kUnitCost keys (pipeline drain and refill, descriptor fetch, merge).
        // No piece is shorter than kSplitMin: a cut that would leave a shorter
        // tail moves back so the tail has kSplitMin keys, or to the range end.  Chunks are at least max_tok / kMaxSplits long, so no range
        // has more splits than the last-arriving CTA merges quickly, and grow
        // until the charged plan fits in target_ctas CTAs.
        uint32_t max_tok = 0;
        for (uint32_t i = 0; i < n_items; ++i) max_tok = std::max(max_tok, pos_host[i] + 1);
        uint64_t chunk = (total + target_ctas - 1) / target_ctas;
        chunk = std::max<uint64_t>(chunk, kSplitMin);
        chunk = std::max<uint64_t>(chunk, (max_tok + kMaxSplits - 1) / kMaxSplits);
        for (int attempt = 0;; ++attempt) {
            w.clear();
            parts = groups = 0;
            uint64_t pos = 0;            // keys (plus charges) laid down so far
            uint64_t last_cta = ~0ull;   // CTA of the previous unit
            for (uint32_t i = 0; i < n_items; ++i) {
                const uint32_t ntok = pos_host[i] + 1;
                for (uint32_t kg = 0; kg < nkg; ++kg) {
                    const size_t first = w.size();
                    uint32_t t = 0;
                    while (t < ntok) {
                        uint64_t c = pos / chunk;
                        if (c == last_cta) {                 // another unit for this CTA
                            pos += kUnitCost;
                            if (pos / chunk != c) pos = (c + 1) * chunk;
                            c = pos / chunk;
                        }
                        uint64_t room = (c + 1) * chunk - pos;
                        if (room < kSplitMin && ntok - t > room) {   // too little room left: next CTA
                            pos += room;
                            ++c;
                            room = chunk;
                        }
                        uint32_t len = static_cast<uint32_t>(std::min<uint64_t>(ntok - t, room));
                        const uint32_t rest = ntok - t - len;
                        if (rest > 0 && rest < kSplitMin) {   // no short tail:
                            if (len >= 2 * kSplitMin - rest)
                                len -= kSplitMin - rest;      // leave kSplitMin keys for the next CTA
                            else
                                len = ntok - t;               // or take the tail here
                        }
                        YattnDecodeWork x{};
                        x.item = i;
                        x.kv_head = static_cast<uint16_t>(kg * hc);
                        x.t_begin = t;
                        x.t_end = t + len;
                        x.cta = static_cast<uint32_t>(c);
                        w.push_back(x);
                        t += len;
                        pos += len;
                        last_cta = c;
                    }
                    const uint32_t ns = static_cast<uint32_t>(w.size() - first);
                    if (ns > 65535) {
                        set_err(err, errlen, "decode_plan: %u splits for item %u (max 65535)", ns, i);
                        return -1;
                    }
                    for (uint32_t s = 0; s < ns; ++s) {
                        YattnDecodeWork& x = w[first + s];
                        x.n_splits = static_cast<uint16_t>(ns);
                        x.split = s;
                        x.part_base = ns > 1 ? parts : 0u;
                        x.group = ns > 1 ? groups : 0u;
                    }
                    if (ns > 1) {
                        parts += hc * ns;
                        groups += 1;
                    }
                }
            }
            // dense CTA numbers (a chunk that the cuts skipped holds no unit): the run
            // launches one CTA per unit, so the CTA count must not exceed the unit count
            uint32_t n_cta = 0, prev = ~0u;
            for (YattnDecodeWork& x : w) {
                if (x.cta != prev) {
                    prev = x.cta;
                    ++n_cta;
                }
                x.cta = n_cta - 1;
            }
            if (n_cta <= target_ctas || attempt >= 64) break;
            // the charges pushed units past the last CTA: grow finely first, then faster
            chunk += (attempt < 16 ? chunk / 128 : chunk / 16) + 1;
        }
        // units are already grouped by CTA in increasing order.  When the ranges
        // are few and even (a batch of equal contexts, fewer ranges than CTAs),
        // cutting every range into equal pieces can beat the balanced cut: each
        // CTA then has one unit and every range fewer splits.  The uniform cut is
        // taken when it finishes within one unit charge of the balanced plan's
        // largest charged CTA, since the charge undercounts a unit's cost where
        // the merged rows are wide (qwen35's 8 query heads of 256 dims per kv
        // head: 56 us uniform against 58-61 us balanced at 32 x 4096 keys).
        uint64_t est = 0, cur = 0;
        for (size_t u = 0; u < w.size(); ++u) {
            const bool first_of_cta = u == 0 || w[u].cta != w[u - 1].cta;
            cur = (first_of_cta ? 0 : cur + kUnitCost) + (w[u].t_end - w[u].t_begin);
            est = std::max(est, cur);
        }
        if (static_cast<uint64_t>(n_items) * nkg <= target_ctas) {
            // smallest split (in kSplitQuant steps, at least kSplitMin) whose pieces fit in
            // target_ctas CTAs; the piece count falls as the split grows, and at a split of
            // max_tok every range is one piece
            auto pieces = [&](uint64_t split) {
                uint64_t n = 0;
                for (uint32_t i = 0; i < n_items; ++i) n += (pos_host[i] + split) / split;   // ceil((pos+1)/split)
                return n * nkg;
            };
            uint64_t lo = (std::max<uint32_t>(kSplitMin, kSplitQuant) + kSplitQuant - 1) / kSplitQuant;
            uint64_t hi = std::max<uint64_t>(lo, (static_cast<uint64_t>(max_tok) + kSplitQuant - 1) / kSplitQuant);
            while (lo < hi) {
                const uint64_t mid = (lo + hi) / 2;
                if (pieces(mid * kSplitQuant) <= target_ctas)
                    hi = mid;
                else
                    lo = mid + 1;
            }
            const uint64_t best = lo * kSplitQuant;
            if (pieces(best) <= target_ctas && std::min<uint64_t>(best, max_tok) <= est + kUnitCost &&
                build_uniform(static_cast<uint32_t>(best)) != 0)
                return -1;
        }
    }
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
}  // namespace

extern "C" int yattn_decode_plan(const uint32_t* pos_host, uint32_t n_items, uint32_t n_kv_heads,
                                 uint32_t head_dim, uint32_t split_tokens, uint32_t target_ctas,
                                 YattnDecodeWork* work_host, uint32_t work_cap, uint32_t* n_work, uint32_t* n_parts,
                                 uint32_t* n_groups, char* err, size_t errlen) {
    return decode_plan_impl(pos_host, n_items, n_kv_heads, head_dim, split_tokens, target_ctas, false, work_host, work_cap,
                            n_work, n_parts, n_groups, err, errlen);
}

extern "C" int yattn_decode_plan_pooled(const uint32_t* pos_host, uint32_t n_items, uint32_t n_kv_heads,
                                        uint32_t head_dim, uint32_t split_tokens, uint32_t target_ctas,
                                        YattnDecodeWork* work_host, uint32_t work_cap, uint32_t* n_work,
                                        uint32_t* n_parts, uint32_t* n_groups, char* err, size_t errlen) {
    return decode_plan_impl(pos_host, n_items, n_kv_heads, head_dim, split_tokens, target_ctas, true, work_host, work_cap,
                            n_work, n_parts, n_groups, err, errlen);
}

extern "C" size_t yattn_decode_workspace_bytes(uint32_t n_parts, uint32_t n_groups, uint32_t n_heads,
                                               uint32_t n_kv_heads, uint32_t head_dim) {
    if (n_kv_heads == 0) return 0;
    if (n_parts == 0) return 0;
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

namespace {
// pool == nullptr: row-copy kernels.  pool: every item's K and V rows lie in
// [pool, pool + pool_bytes); one tensor map covers it (tensor-copy kernels, plan
// made by yattn_decode_plan_pooled).
int decode_run_impl(const YattnDecodeItem* items_dev, const YattnDecodeWork* work_dev, uint32_t n_work,
                    uint32_t n_parts, uint32_t n_groups, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                    uint32_t kv_dim, const void* pool, size_t pool_bytes, void* workspace, size_t ws_bytes,
                    void* stream, char* err, size_t errlen, const DecodeRope* rope = nullptr) {
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
    p.n_work = n_work;
    p.n_heads = n_heads;
    p.n_kv = n_kv_heads;
    p.kv_dim = kv_dim;
    p.hc = pool ? tm_heads_per_cta(n_kv_heads, head_dim) : heads_per_cta(n_kv_heads, head_dim);
    p.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(head_dim));
    p.status = ctx->status;
    if (n_parts > 0) carve_ws(workspace, n_parts, n_groups, gmax, p);
    if (!pool)
        return launch_decode(p, false, nullptr, nullptr, head_dim, n_work, static_cast<cudaStream_t>(stream), err,
                             errlen);
    if (reinterpret_cast<uintptr_t>(pool) & 15u) {
        set_err(err, errlen, "decode_run_pooled: pool must be 16-byte aligned");
        return -1;
    }
    const uint64_t rows = pool_bytes / (static_cast<uint64_t>(kv_dim) * 2);
    if (rows == 0) {
        set_err(err, errlen, "decode_run_pooled: pool of %zu bytes holds no row of kv_dim %u", pool_bytes, kv_dim);
        return -1;
    }
    CUtensorMap map;
    const uint32_t box_rows = 16u * (head_dim >= 256 ? DecodeCfg<256>::NCW : DecodeCfg<128>::NCW) / p.hc;
    if (encode_kv_map(&map, pool, kv_dim, rows, box_rows, err, errlen)) return -1;
    p.kmap_base = p.vmap_base = reinterpret_cast<uint64_t>(pool);
    p.row_bytes = kv_dim * 2;
    if (rope) {
        DecodeRope r = *rope;
        r.pool_rows = rows;
        return launch_decode(p, true, &map, &map, head_dim, n_work, static_cast<cudaStream_t>(stream), err, errlen,
                             &r);
    }
    return launch_decode(p, true, &map, &map, head_dim, n_work, static_cast<cudaStream_t>(stream), err, errlen);
}
}  // namespace

extern "C" int yattn_decode_run(const YattnDecodeItem* items_dev, const YattnDecodeWork* work_dev, uint32_t n_work,
                                uint32_t n_parts, uint32_t n_groups, uint32_t n_heads, uint32_t n_kv_heads,
                                uint32_t head_dim, uint32_t kv_dim, void* workspace, size_t ws_bytes, void* stream,
                                char* err, size_t errlen) {
    return decode_run_impl(items_dev, work_dev, n_work, n_parts, n_groups, n_heads, n_kv_heads, head_dim, kv_dim,
                           nullptr, 0, workspace, ws_bytes, stream, err, errlen);
}

extern "C" int yattn_decode_run_pooled(const YattnDecodeItem* items_dev, const YattnDecodeWork* work_dev,
                                       uint32_t n_work, uint32_t n_parts, uint32_t n_groups, uint32_t n_heads,
                                       uint32_t n_kv_heads, uint32_t head_dim, uint32_t kv_dim, const void* pool,
                                       size_t pool_bytes, void* workspace, size_t ws_bytes, void* stream, char* err,
                                       size_t errlen) {
    if (!pool) {
        set_err(err, errlen, "decode_run_pooled: null pool");
        return -1;
    }
    return decode_run_impl(items_dev, work_dev, n_work, n_parts, n_groups, n_heads, n_kv_heads, head_dim, kv_dim,
                           pool, pool_bytes, workspace, ws_bytes, stream, err, errlen);
}

extern "C" int yattn_decode_run_pooled_rope(const YattnDecodeItem* items_dev, const YattnDecodeNewRow* rows_dev,
                                            const YattnDecodeWork* work_dev, uint32_t n_work, uint32_t n_parts,
                                            uint32_t n_groups, uint32_t n_heads, uint32_t n_kv_heads,
                                            uint32_t head_dim, uint32_t kv_dim, const void* pool, size_t pool_bytes,
                                            int rope_kind, uint32_t n_rope_dims, float theta, void* workspace,
                                            size_t ws_bytes, void* stream, char* err, size_t errlen) {
    if (!pool || !rows_dev) {
        set_err(err, errlen, "decode_run_pooled_rope: null pool or rows");
        return -1;
    }
    if (rope_kind < 0 || rope_kind > 2) {
        set_err(err, errlen, "decode_run_pooled_rope: rope_kind %d (0 llama, 1 qwen, 2 mrope)", rope_kind);
        return -1;
    }
    const uint32_t nd = rope_kind == 2 ? n_rope_dims : head_dim;
    if (nd == 0 || (nd & 1) || nd > head_dim || nd / 2 > static_cast<uint32_t>(kRopeMaxPairs)) {
        set_err(err, errlen, "decode_run_pooled_rope: %u rotated dims for head_dim %u", nd, head_dim);
        return -1;
    }
    DecodeRope rope{};
    rope.rows = rows_dev;
    rope.kind = static_cast<uint32_t>(rope_kind);
    rope.n_dims = nd;
    // the reference's expression, in the same fp32 operation order (matvec.c:895, 912, 929)
    for (uint32_t j = 0; j < nd / 2; ++j)
        rope.inv_freq[j] = powf(theta, -2.0f * static_cast<float>(j) / static_cast<float>(nd));
    return decode_run_impl(items_dev, work_dev, n_work, n_parts, n_groups, n_heads, n_kv_heads, head_dim, kv_dim,
                           pool, pool_bytes, workspace, ws_bytes, stream, err, errlen, &rope);
}

extern "C" size_t yattn_decode_partial_workspace_bytes(uint32_t n_tokens, uint32_t n_heads, uint32_t n_kv_heads,
                                                       uint32_t head_dim) {
    if (n_kv_heads == 0 || n_tokens == 0) return 0;
    const SinglePlan sp = plan_single(n_tokens, n_kv_heads, head_dim, static_cast<uint32_t>(dev_num_sms()));
    if (sp.ns <= 1) return 0;
    return ws_bytes_for(sp.n_parts, sp.n_groups, gmax_of(n_heads, n_kv_heads), head_dim);
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
    k_merge_partials<<<n_heads, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        out, ml, o, n_parts, n_heads, head_dim, gate, static_cast<size_t>(n_heads) * 2,
        static_cast<size_t>(n_heads) * head_dim);
    YATTN_CHECK_LAUNCH(err, errlen, "merge_partials");
    return 0;
}

extern "C" int yattn_merge_partials_packed(float* out, const float* parts, uint32_t n_parts, uint32_t n_heads,
                                           uint32_t head_dim, const float* gate, void* stream, char* err,
                                           size_t errlen) {
    if (!out || !parts || n_parts == 0 || n_heads == 0 || head_dim == 0) {
        set_err(err, errlen, "merge_partials_packed: bad arguments");
        return -1;
    }
    const size_t part = static_cast<size_t>(n_heads) * (2 + head_dim);
    k_merge_partials<<<n_heads, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        out, parts, parts + static_cast<size_t>(n_heads) * 2, n_parts, n_heads, head_dim, gate, part, part);
    YATTN_CHECK_LAUNCH(err, errlen, "merge_partials_packed");
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

// ------------------------------------------------------- split-KV decode + exchange
//
// One rank's step of a decode whose key range is split over the GPUs: the
// partial decode of keys [k_begin, k_end) (split-KV over this GPU's SMs), then
// one kernel that merges this GPU's splits per head and exchanges the merged
// heads with every rank over peer memory (exchange.cuh), writing the whole
// range's output on every rank.  Two launches per step; an empty shard
// (k_begin == k_end) takes part in the exchange with l = 0.

extern "C" int yattn_decode_exchange(const float* q, const uint16_t* kcache, const uint16_t* vcache,
                                     uint32_t k_begin, uint32_t k_end, uint32_t n_heads, uint32_t n_kv_heads,
                                     uint32_t head_dim, uint32_t kv_dim, void* const* areas, uint32_t world,
                                     uint32_t rank, float* out, const float* gate, uint64_t wait_limit_ns,
                                     void* workspace, size_t ws_bytes, void* stream, char* err, size_t errlen) {
    if (check_geom(n_heads, n_kv_heads, head_dim, kv_dim, err, errlen)) return -1;
    if (!areas || !out || world == 0 || world > kMaxWorld || rank >= world || k_end < k_begin) {
        set_err(err, errlen, "decode_exchange: bad arguments (world 1..%u, rank < world, k_begin <= k_end)",
                kMaxWorld);
        return -1;
    }
    ExchangeArgs ex{};
    for (uint32_t r = 0; r < world; ++r) {
        if (!areas[r]) {
            set_err(err, errlen, "decode_exchange: null area for rank %u", r);
            return -1;
        }
        ex.area[r] = static_cast<uint8_t*>(areas[r]);
    }
    ex.world = world;
    ex.rank = rank;
    ex.wait_ns = wait_limit_ns ? wait_limit_ns : kWaitLimitNs;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (k_end > k_begin)
        return decode_single(out, q, kcache, vcache, gate, k_begin, k_end, n_heads, n_kv_heads, head_dim, kv_dim,
                             nullptr, nullptr, workspace, ws_bytes, st, err, errlen, &ex);
    // no keys on this rank: its part of every head has l = 0
    DevCtx* ctx = dev_ctx(err, errlen);
    if (!ctx) return -1;
    k_merge_splits<true><<<n_heads, 256, 0, st>>>(nullptr, nullptr, 0, n_heads, n_kv_heads,
                                                   gmax_of(n_heads, n_kv_heads), head_dim, out, gate, nullptr,
                                                   nullptr, ex, ctx->status);
    YATTN_CHECK_LAUNCH(err, errlen, "decode_exchange");
    return 0;
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
//
// The status word (the array's first int) is never cleared by a decode call:
// a bounded wait that gave up, or a malformed item, stays recorded there until
// yattn_device_status(..., clear = 1) reads and resets it, exactly like the
// status word of the allocating entry points.

namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;   // 4 MiB per device
constexpr size_t kNoAllocHeader = 256;              // status word, then 256-aligned counters + partials

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch, looked up once per device by the first
// call on it.  In host code the symbol itself is only a host-side stand-in,
// never a device address.  The cached address belongs to the device's primary
// context: after cudaDeviceReset() the module is loaded again and the cache is
// stale, so a process that resets a device must not call this entry again.
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

namespace yattn {

// The no-alloc status word of the current device, or nullptr if no
// allocation-free call has run on it yet (then nothing can be recorded there).
int* noalloc_status_word() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    return static_cast<int*>(g_noalloc_addr[dev]);
}

}  // namespace yattn

extern "C" int yattn_attn_decode_noalloc(float* att_out, const float* q, const uint16_t* kcache,
                                         const uint16_t* vcache, const float* gate, uint32_t pos, uint32_t n_heads,
                                         uint32_t n_kv_heads, uint32_t head_dim, uint32_t kv_dim, void* stream,
                                         char* err, size_t errlen) {
    if (check_geom(n_heads, n_kv_heads, head_dim, kv_dim, err, errlen)) return -1;
    if (pos == UINT32_MAX) {   // keys [0, pos + 1) would wrap to an empty range
        set_err(err, errlen, "decode: empty key range [0, %u)", 0u);
        return -1;
    }
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
    const uint32_t gmax = gmax_of(n_heads, n_kv_heads);
    const SinglePlan sp = plan_single(pos + 1, n_kv_heads, head_dim, static_cast<uint32_t>(dev_num_sms()));
    const size_t need = sp.ns > 1 ? ws_bytes_for(sp.n_parts, sp.n_groups, gmax, head_dim) : 0;
    if (need > kNoAllocScratchBytes - kNoAllocHeader) {
        set_err(err, errlen,
                "decode_noalloc: this query needs %zu bytes of split-KV scratch, more than the %zu-byte static "
                "scratch (%u splits x %u kv heads x %u q heads x head_dim %u); use yattn_attn_decode",
                need, kNoAllocScratchBytes - kNoAllocHeader, sp.ns, n_kv_heads, gmax, head_dim);
        return -1;
    }
    // First call on a device: looks up the scratch address (no allocation).
    uint8_t* base = static_cast<uint8_t*>(noalloc_scratch(dev, err, errlen));
    if (!base) return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    DecodeParams p = single_params(sp, att_out, q, kcache, vcache, gate, 0, pos + 1, n_heads, n_kv_heads, head_dim,
                                   kv_dim);
    p.status = reinterpret_cast<int*>(base);   // read and reset by yattn_device_status
    if (sp.ns > 1) {
        // The array keeps the previous call's contents: the merge counters must start at
        // zero (a call that gave up can leave them raised), the partials are fully
        // rewritten before use.  The status word is left as it is.
        carve_ws(base + kNoAllocHeader, sp.n_parts, sp.n_groups, gmax, p);
        cudaError_t e = cudaMemsetAsync(base + kNoAllocHeader, 0, static_cast<size_t>(sp.n_groups) * sizeof(uint32_t),
                                        st);
        if (e != cudaSuccess) {
            set_err(err, errlen, "decode_noalloc: clearing the merge counters failed: %s", cudaGetErrorString(e));
            return -1;
        }
    }
    return launch_single(p, sp, head_dim, st, err, errlen);
}
