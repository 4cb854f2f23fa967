// common.cuh -- shared device/host helpers of the sm_100a attention library.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../../include/yllm_attn_sm100.h"

namespace yattn {

// ------------------------------------------------------------------ host side

// Writes a message into (err, errlen) when the caller gave a buffer.
void set_err(char* err, size_t errlen, const char* fmt, ...);
// Records the message for yattn_last_error() (drop-in entry points).
void set_last_error(const char* msg);
// Per-device context: status word, drop-in workspace.  Created on first use.
struct DevCtx {
    int device = -1;
    int num_sms = 0;
    int* status = nullptr;        // device int, bounded-wait timeouts land here
    void* ws = nullptr;           // drop-in workspace (grown on demand)
    size_t ws_bytes = 0;
    void* small = nullptr;        // device scratch for drop-in items/work descriptors
    size_t small_bytes = 0;
    void* gdn_ws = nullptr;       // chunked GDN prefill scratch (grown on demand)
    size_t gdn_ws_bytes = 0;
};
DevCtx* dev_ctx(char* err, size_t errlen);   // current device's context (nullptr on failure)
// Status word of the allocation-free decode on the current device (nullptr before its first call).
int* noalloc_status_word();
int dev_num_sms();

#define YATTN_CHECK_LAUNCH(err, errlen, what)                                            \
    do {                                                                                 \
        cudaError_t e_ = cudaGetLastError();                                             \
        if (e_ != cudaSuccess) {                                                         \
            ::yattn::set_err(err, errlen, "%s: launch failed: %s", what,                 \
                             cudaGetErrorString(e_));                                    \
            return -1;                                                                   \
        }                                                                                \
    } while (0)

// ---------------------------------------------------------------- device side

// Status codes written to the device status word when a bounded wait gives up
// (or a kernel finds a malformed work item and stops).
enum : int {
    ST_OK = 0,
    ST_DECODE_FULL_TIMEOUT = 101,
    ST_DECODE_EMPTY_TIMEOUT = 102,
    ST_DECODE_BAD_ITEM = 103,   // q / gate not 16-byte aligned, or (pooled) K/V not rows of the pool
    ST_PREFILL_TIMEOUT = 201,
    ST_PREFILL_Q_NOT_F16 = 202,  // YATTN_PREFILL_Q_F16 given, but a q value is not an fp16 value
    ST_GDN_TIMEOUT = 301,
    ST_GEMV_TIMEOUT = 501,
    ST_EXCHANGE_TIMEOUT = 401,
};

// Upper bound of any spin in these kernels (ns of %globaltimer).  Far above
// any legitimate wait (a tile copy takes microseconds).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;   // 2 s

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  On timeout: records `code` in *status
// (first writer wins), sets the CTA abort flag and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* status, int code,
                                                  volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    unsigned long long t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 63u) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                if (status) atomicCAS(status, 0, code);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// Warp-uniform form: every lane waits, the warp proceeds only if all lanes saw
// the phase complete (so a timeout never splits a warp before warp-collective code).
__device__ __forceinline__ bool warp_wait_bounded(uint64_t* bar, uint32_t parity, int* status, int code,
                                                  volatile int* abort_flag) {
    const bool ok = mbar_wait_bounded(bar, parity, status, code, abort_flag);
    return __all_sync(0xffffffffu, ok);
}

// One bulk global->shared copy completing on an mbarrier (TMA, non-tensor form).
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ANDs a predicate over the participating threads: every
// thread gets the same answer, so all of them can take the same branch after it.
__device__ __forceinline__ bool named_bar_and(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred p, %2, %3, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"(pred ? 1u : 0u), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// Named barrier that ORs a predicate over the participating threads.
__device__ __forceinline__ bool named_bar_or(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.or.pred p, %2, %3, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"(pred ? 1u : 0u), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// Prefetch [src, src + bytes) into L2 (bulk form; src 16-byte aligned, bytes a multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// The engine's f32_to_f16 (platform.c:340-379): half-up rounding of the
// dropped mantissa bits, f32 subnormals to zero, overflow to inf.
__host__ __device__ __forceinline__ uint16_t engine_f32_to_f16(float f) {
#ifdef __CUDA_ARCH__
    uint32_t x = __float_as_uint(f);
#else
    uint32_t x;
    memcpy(&x, &f, 4);
#endif
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t fexp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    int e = static_cast<int>(fexp) - 112;
    if (fexp == 0) return static_cast<uint16_t>(sign);
    if (fexp == 0xff) return static_cast<uint16_t>(sign | 0x7c00u | (man ? 0x200u : 0u));
    if (e >= 31) return static_cast<uint16_t>(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return static_cast<uint16_t>(sign);
        uint32_t full = man | 0x800000u;
        uint32_t sh = static_cast<uint32_t>(14 - e);
        return static_cast<uint16_t>(sign | ((full + (1u << (sh - 1))) >> sh));
    }
    man += 0x1000u;
    if (man & 0x800000u) {
        e += 1;
        if (e >= 31) return static_cast<uint16_t>(sign | 0x7c00u);
        return static_cast<uint16_t>(sign | (static_cast<uint32_t>(e) << 10));
    }
    return static_cast<uint16_t>(sign | (static_cast<uint32_t>(e) << 10) | (man >> 13));
}

// RoPE rotation of the pair (a, b) of inverse frequency inv_freq at position pos, in the
// reference's fp32 operation order (matvec.c:890-939): angle = one fp32 multiply,
// a*c - b*s and a*s + b*c without FMA contraction.  Shared by the RoPE store and the
// decode with the fused store, so both give the same bits.
__device__ __forceinline__ void rope_sincos(float inv_freq, uint32_t pos, float& s, float& c) {
    sincosf(__fmul_rn(inv_freq, static_cast<float>(pos)), &s, &c);
}
__device__ __forceinline__ void rope_apply(float& a, float& b, float s, float c) {
    const float ra = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    const float rb = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
    a = ra;
    b = rb;
}
__device__ __forceinline__ void rope_rotate(float& a, float& b, float inv_freq, uint32_t pos) {
    float s, c;
    rope_sincos(inv_freq, pos, s, c);
    rope_apply(a, b, s, c);
}

// Element indices (e0, e1) of RoPE pair j inside a head: kind 0 (2j, 2j+1), kind 1
// (j, j + hd/2), kind 2 (j, j + n_dims/2).
__host__ __device__ __forceinline__ void rope_pair(uint32_t kind, uint32_t hd, uint32_t n_dims, uint32_t j,
                                                   uint32_t& e0, uint32_t& e1) {
    if (kind == 0) {
        e0 = 2 * j;
        e1 = 2 * j + 1;
    } else if (kind == 1) {
        e0 = j;
        e1 = j + hd / 2;
    } else {
        e0 = j;
        e1 = j + n_dims / 2;
    }
}

// fp16 bits -> fp32, exact (hardware conversion).
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ float2 h2f2(uint32_t two) {
    return __half22float2(*reinterpret_cast<const __half2*>(&two));
}

}  // namespace yattn
