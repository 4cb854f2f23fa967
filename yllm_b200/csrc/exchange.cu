// exchange.cu -- split-KV partial exchange and merge over peer memory (NVLink).
//
// Long-context decode shards one query's key range over the GPUs (one process
// per GPU); each GPU reduces its range to per-head (m, l, o) partials with
// yattn_decode_partial.  The reference has no multi-GPU attention (its only
// parallelism is pipeline parallelism over TCP, dist.c), so this exchange has no
// reference counterpart; the merge arithmetic is the log-sum-exp merge of
// decode.cu.
//
// One kernel does the exchange and the merge.  CTA hh (one per query head):
//   1. stores this rank's partial of head hh into every rank's receive area
//      (slot [parity][rank][hh]) -- plain stores into peer memory over NVLink;
//   2. raises flag [rank][hh] of every area to this launch's epoch
//      (release, system scope);
//   3. waits, bounded, until the local area's flags [r][hh] of all ranks reach
//      the epoch (acquire, system scope), then merges the parts of head hh from
//      local memory and writes out.
// No GPU loads another GPU's memory.  Payloads are double-buffered by epoch
// parity: a rank can run at most one call ahead of a peer (it cannot finish
// call e+1 before the peer pushed e+1, which the peer does only after it has
// merged call e), so the other parity's payload is never overwritten early.
//
// The epoch lives in the local area's header and advances when the last CTA of
// a launch finishes, so repeated launches (a CUDA graph replays one) need no
// host-side counter.
#include "common.cuh"

namespace yattn {
namespace {

constexpr uint32_t kMaxWorld = 8;
constexpr size_t kHeader = 256;   // epoch, finished-CTA counter

struct AreaLayout {
    size_t flags;      // u32 [world][n_heads]
    size_t parts;      // f32 [2][world][n_heads][2 + hd]
    size_t bytes;
};

__host__ __device__ inline AreaLayout area_layout(uint32_t world, uint32_t n_heads, uint32_t hd) {
    AreaLayout a{};
    a.flags = kHeader;
    a.parts = kHeader + ((static_cast<size_t>(world) * n_heads * 4 + 255) / 256) * 256;
    a.bytes = a.parts + 2ull * world * n_heads * (2 + hd) * 4;
    return a;
}

struct ExParams {
    const float* ml;                 // this rank's (m, l) [n_heads][2]
    const float* o;                  // this rank's o [n_heads][hd]
    uint8_t* area[kMaxWorld];        // every rank's receive area (area[rank] is local)
    float* out;
    const float* gate;
    uint32_t world, rank, n_heads, hd;
    unsigned long long wait_ns;      // bound of the flag wait
    int* status;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(128) k_exchange_merge(const ExParams p) {
    const uint32_t hh = blockIdx.x;
    const AreaLayout L = area_layout(p.world, p.n_heads, p.hd);
    uint8_t* mine = p.area[p.rank];
    uint32_t* hdr = reinterpret_cast<uint32_t*>(mine);
    __shared__ uint32_t s_epoch;
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        s_epoch = *reinterpret_cast<volatile uint32_t*>(hdr) + 1u;   // this launch's epoch
        s_ok = 1;
    }
    __syncthreads();
    const uint32_t epoch = s_epoch;
    const uint32_t par = epoch & 1u;
    const size_t part_f = 2 + p.hd;   // floats per (rank, head) part

    // ---- 1. push this rank's part of head hh into every area ----
    for (uint32_t r = 0; r < p.world; ++r) {
        float* dst = reinterpret_cast<float*>(p.area[r] + L.parts) +
                     ((static_cast<size_t>(par) * p.world + p.rank) * p.n_heads + hh) * part_f;
        for (uint32_t i = threadIdx.x; i < part_f; i += blockDim.x)
            dst[i] = (i < 2) ? p.ml[hh * 2 + i] : p.o[static_cast<size_t>(hh) * p.hd + (i - 2)];
    }
    __syncthreads();
    // ---- 2. publish: flag [rank][hh] of every area = epoch ----
    if (threadIdx.x < p.world) {
        __threadfence_system();
        uint32_t* f = reinterpret_cast<uint32_t*>(p.area[threadIdx.x] + L.flags) +
                      static_cast<size_t>(p.rank) * p.n_heads + hh;
        st_release_sys(f, epoch);
    }
    // ---- 3. wait for every rank's part of head hh (bounded), then merge ----
    if (threadIdx.x < p.world) {
        const uint32_t* f = reinterpret_cast<const uint32_t*>(mine + L.flags) +
                            static_cast<size_t>(threadIdx.x) * p.n_heads + hh;
        const unsigned long long t0 = globaltimer_ns();
        for (uint32_t it = 0;; ++it) {
            if (static_cast<int>(ld_acquire_sys(f) - epoch) >= 0) break;
            if ((it & 255u) == 255u && globaltimer_ns() - t0 > p.wait_ns) {
                atomicCAS(p.status, 0, ST_EXCHANGE_TIMEOUT);
                s_ok = 0;
                break;
            }
        }
    }
    __syncthreads();
    if (s_ok) {
        const float* parts = reinterpret_cast<const float*>(mine + L.parts) +
                             static_cast<size_t>(par) * p.world * p.n_heads * part_f;
        for (uint32_t d = threadIdx.x; d < p.hd; d += blockDim.x) {
            float M = -INFINITY;
            for (uint32_t r = 0; r < p.world; ++r) {
                const float* pr = parts + (static_cast<size_t>(r) * p.n_heads + hh) * part_f;
                if (__ldcg(pr + 1) > 0.f) M = fmaxf(M, __ldcg(pr));
            }
            float acc = 0.f, l = 0.f;
            for (uint32_t r = 0; r < p.world; ++r) {
                const float* pr = parts + (static_cast<size_t>(r) * p.n_heads + hh) * part_f;
                const float lr = __ldcg(pr + 1);
                if (!(lr > 0.f)) continue;
                const float sc = ex2_approx(__ldcg(pr) - M);
                acc += sc * __ldcg(pr + 2 + d);
                l += sc * lr;
            }
            // every rank's shard empty: no key was attended, the output is 0 (not 0/0)
            float res = l > 0.f ? acc / l : 0.f;
            if (p.gate) res *= 1.0f / (1.0f + __expf(-p.gate[static_cast<size_t>(hh) * p.hd + d]));
            p.out[static_cast<size_t>(hh) * p.hd + d] = res;
        }
    } else {
        // a peer never published: the output is NaN, so a caller that skips the status
        // poll cannot take a stale result for this call's
        for (uint32_t d = threadIdx.x; d < p.hd; d += blockDim.x)
            p.out[static_cast<size_t>(hh) * p.hd + d] = __int_as_float(0x7fc00000);
    }
    // ---- the last CTA of the launch advances the local epoch ----
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t done = atomicAdd(hdr + 1, 1u);
        if (done == gridDim.x - 1) {
            hdr[1] = 0u;
            __threadfence();
            atomicExch(hdr, epoch);
        }
    }
}

}  // namespace
}  // namespace yattn

using namespace yattn;

extern "C" size_t yattn_exchange_area_bytes(uint32_t world, uint32_t n_heads, uint32_t head_dim) {
    if (world == 0 || world > kMaxWorld || n_heads == 0 || head_dim == 0) return 0;
    return area_layout(world, n_heads, head_dim).bytes;
}

extern "C" int yattn_exchange_area_alloc(uint32_t world, uint32_t n_heads, uint32_t head_dim, void** area_out,
                                         char* err, size_t errlen) {
    if (!area_out || world == 0 || world > kMaxWorld || n_heads == 0 || head_dim == 0) {
        set_err(err, errlen, "exchange_area_alloc: bad arguments (world 1..%u)", kMaxWorld);
        return -1;
    }
    const size_t bytes = area_layout(world, n_heads, head_dim).bytes;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess || cudaMemset(p, 0, bytes) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        if (p) cudaFree(p);
        set_err(err, errlen, "exchange_area_alloc: cudaMalloc/cudaMemset(%zu) failed", bytes);
        return -1;
    }
    *area_out = p;
    return 0;
}

extern "C" int yattn_exchange_area_free(void* area, char* err, size_t errlen) {
    if (area && cudaFree(area) != cudaSuccess) {
        set_err(err, errlen, "exchange_area_free: cudaFree failed");
        return -1;
    }
    return 0;
}

extern "C" int yattn_ipc_handle(const void* area, void* handle_out, char* err, size_t errlen) {
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(area));
    if (e != cudaSuccess) {
        set_err(err, errlen, "ipc_handle: %s", cudaGetErrorString(e));
        return -1;
    }
    memcpy(handle_out, &h, sizeof(h));
    return 0;
}

extern "C" int yattn_ipc_open(const void* handle, void** ptr_out, char* err, size_t errlen) {
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        set_err(err, errlen, "ipc_open: %s", cudaGetErrorString(e));
        return -1;
    }
    *ptr_out = p;
    return 0;
}

extern "C" int yattn_ipc_close(void* ptr, char* err, size_t errlen) {
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) {
        set_err(err, errlen, "ipc_close: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

extern "C" int yattn_exchange_merge(const float* ml, const float* o, void* const* areas, uint32_t world,
                                    uint32_t rank, uint32_t n_heads, uint32_t head_dim, float* out, const float* gate,
                                    uint64_t wait_limit_ns, void* stream, char* err, size_t errlen) {
    if (!ml || !o || !areas || !out || world == 0 || world > kMaxWorld || rank >= world || n_heads == 0 ||
        head_dim == 0) {
        set_err(err, errlen, "exchange_merge: bad arguments (world 1..%u, rank < world)", kMaxWorld);
        return -1;
    }
    DevCtx* ctx = dev_ctx(err, errlen);
    if (!ctx) return -1;
    ExParams p{};
    p.ml = ml;
    p.o = o;
    for (uint32_t r = 0; r < world; ++r) {
        if (!areas[r]) {
            set_err(err, errlen, "exchange_merge: null area for rank %u", r);
            return -1;
        }
        p.area[r] = static_cast<uint8_t*>(areas[r]);
    }
    p.out = out;
    p.gate = gate;
    p.world = world;
    p.rank = rank;
    p.n_heads = n_heads;
    p.hd = head_dim;
    p.wait_ns = wait_limit_ns ? wait_limit_ns : kWaitLimitNs;
    p.status = ctx->status;
    k_exchange_merge<<<n_heads, 128, 0, static_cast<cudaStream_t>(stream)>>>(p);
    YATTN_CHECK_LAUNCH(err, errlen, "exchange_merge");
    return 0;
}
