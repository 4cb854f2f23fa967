// exchange.cuh -- the split-KV partial exchange over peer memory, shared by the
// standalone exchange kernel (exchange.cu) and the decode's fused split merge
// (decode.cu).
//
// Every rank owns one receive area:
//   header  [0, 256)          u32 epoch, u32 finished-CTA counter
//   flags   [256, ...)        u32 [world][n_heads]: flag [r][hh] = last epoch rank r published head hh
//   parts                     f32 [2 parities][world][n_heads][2 + hd]: (m, l, o[hd]) of rank r, head hh
// A launch's epoch is the local header's epoch + 1; parts go to parity epoch & 1.
// A rank can run at most one call ahead of a peer (it cannot finish call e+1
// before the peer pushed e+1, which the peer does only after it merged call e),
// so the other parity's parts are never overwritten early.  The last CTA of a
// launch advances the local epoch, so repeated launches (a CUDA graph replays
// one) need no host-side counter.
//
// No GPU loads another GPU's memory: a rank stores its part and raises its flag
// in every area (plain stores over NVLink) and reads only its own area.
#pragma once

#include "common.cuh"

namespace yattn {

constexpr uint32_t kMaxWorld = 8;
constexpr size_t kExHeader = 256;   // epoch, finished-CTA counter

struct AreaLayout {
    size_t flags;      // u32 [world][n_heads]
    size_t parts;      // f32 [2][world][n_heads][2 + hd]
    size_t bytes;
};

__host__ __device__ inline AreaLayout area_layout(uint32_t world, uint32_t n_heads, uint32_t hd) {
    AreaLayout a{};
    a.flags = kExHeader;
    a.parts = kExHeader + ((static_cast<size_t>(world) * n_heads * 4 + 255) / 256) * 256;
    a.bytes = a.parts + 2ull * world * n_heads * (2 + hd) * 4;
    return a;
}

// Where the exchange goes: every rank's area as mapped in this process.
struct ExchangeArgs {
    uint8_t* area[kMaxWorld];
    uint32_t world, rank;
    unsigned long long wait_ns;      // bound of the flag wait
};

// Release pattern at system scope: the fence orders every access that precedes
// it (this thread's, and by the CTA barrier before it the other threads') before
// the flag store; the peer's acquire load of the flag then sees them.
__device__ __forceinline__ void publish_sys(uint32_t* p, uint32_t v) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// This launch's epoch, read from the local header by thread 0 (published in *s_epoch).
__device__ __forceinline__ void exchange_epoch(const ExchangeArgs& ex, uint32_t* s_epoch) {
    if (threadIdx.x == 0) *s_epoch = *reinterpret_cast<volatile const uint32_t*>(ex.area[ex.rank]) + 1u;
}

// One CTA, head hh: pushes this rank's part (M, L in registers of every thread,
// o[0..hd) in shared memory) into every rank's area, raises flag [rank][hh]
// there, waits (bounded) for every rank's flag of hh in the local area and
// writes the merged head into out (x sigmoid(gate)).  A head whose parts all
// have L == 0 gets 0; on timeout the head is NaN and *status reads 401.
// Every thread of the CTA calls it; blockDim.x >= world.
__device__ __forceinline__ void exchange_head(const ExchangeArgs& ex, uint32_t epoch, uint32_t n_heads, uint32_t hd,
                                              uint32_t hh, float M, float L, const float* s_o, float* out,
                                              const float* gate, int* status) {
    const AreaLayout lay = area_layout(ex.world, n_heads, hd);
    const uint32_t par = epoch & 1u;
    const size_t part_f = 2 + hd;
    __shared__ int s_ok;
    // ---- push this rank's part into every area ----
    for (uint32_t r = 0; r < ex.world; ++r) {
        float* dst = reinterpret_cast<float*>(ex.area[r] + lay.parts) +
                     ((static_cast<size_t>(par) * ex.world + ex.rank) * n_heads + hh) * part_f;
        for (uint32_t i = threadIdx.x; i < part_f; i += blockDim.x) dst[i] = i == 0 ? M : i == 1 ? L : s_o[i - 2];
    }
    if (threadIdx.x == 0) s_ok = 1;
    __syncthreads();
    // ---- publish: flag [rank][hh] of every area = epoch ----
    if (threadIdx.x < ex.world) {
        uint32_t* f = reinterpret_cast<uint32_t*>(ex.area[threadIdx.x] + lay.flags) +
                      static_cast<size_t>(ex.rank) * n_heads + hh;
        publish_sys(f, epoch);
    }
    // ---- wait for every rank's part of head hh (bounded) ----
    if (threadIdx.x < ex.world) {
        const uint32_t* f = reinterpret_cast<const uint32_t*>(ex.area[ex.rank] + lay.flags) +
                            static_cast<size_t>(threadIdx.x) * n_heads + hh;
        const unsigned long long t0 = globaltimer_ns();
        for (uint32_t it = 0;; ++it) {
            if (static_cast<int>(ld_acquire_sys(f) - epoch) >= 0) break;
            if ((it & 255u) == 255u && globaltimer_ns() - t0 > ex.wait_ns) {
                atomicCAS(status, 0, ST_EXCHANGE_TIMEOUT);
                s_ok = 0;
                break;
            }
        }
    }
    __syncthreads();
    const float* parts = reinterpret_cast<const float*>(ex.area[ex.rank] + lay.parts) +
                         static_cast<size_t>(par) * ex.world * n_heads * part_f;
    if (s_ok) {
        // every rank's (m, l) first, all loads in flight, then the o values
        float mr[kMaxWorld], lr[kMaxWorld];
#pragma unroll
        for (uint32_t r = 0; r < kMaxWorld; ++r) {
            mr[r] = -INFINITY;
            lr[r] = 0.f;
            if (r < ex.world) {
                const float* pr = parts + (static_cast<size_t>(r) * n_heads + hh) * part_f;
                mr[r] = __ldcg(pr);
                lr[r] = __ldcg(pr + 1);
            }
        }
        float Mx = -INFINITY;
#pragma unroll
        for (uint32_t r = 0; r < kMaxWorld; ++r)
            if (lr[r] > 0.f) Mx = fmaxf(Mx, mr[r]);
        float w[kMaxWorld], Lx = 0.f;
#pragma unroll
        for (uint32_t r = 0; r < kMaxWorld; ++r) {
            w[r] = lr[r] > 0.f ? ex2_approx(mr[r] - Mx) : 0.f;
            Lx += w[r] * lr[r];
        }
        for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x) {
            float ov[kMaxWorld];
#pragma unroll
            for (uint32_t r = 0; r < kMaxWorld; ++r)
                ov[r] = (r < ex.world && w[r] != 0.f)
                            ? __ldcg(parts + (static_cast<size_t>(r) * n_heads + hh) * part_f + 2 + d)
                            : 0.f;
            float acc = 0.f;
#pragma unroll
            for (uint32_t r = 0; r < kMaxWorld; ++r) acc += w[r] * ov[r];
            // every rank's shard empty: no key was attended, the output is 0 (not 0/0)
            float res = Lx > 0.f ? acc / Lx : 0.f;
            if (gate) res *= 1.0f / (1.0f + __expf(-gate[static_cast<size_t>(hh) * hd + d]));
            out[static_cast<size_t>(hh) * hd + d] = res;
        }
    } else {
        // a peer never published: the output is NaN, so a caller that skips the status
        // poll cannot take a stale result for this call's
        for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x)
            out[static_cast<size_t>(hh) * hd + d] = __int_as_float(0x7fc00000);
    }
}

// The last CTA of the launch advances the local epoch (every thread calls it).
__device__ __forceinline__ void exchange_finish(const ExchangeArgs& ex, uint32_t epoch) {
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t* hdr = reinterpret_cast<uint32_t*>(ex.area[ex.rank]);
        const uint32_t done = atomicAdd(hdr + 1, 1u);
        if (done == gridDim.x - 1) {
            hdr[1] = 0u;
            __threadfence();
            atomicExch(hdr, epoch);
        }
    }
}

}  // namespace yattn
