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
#include "exchange.cuh"

namespace yattn {
namespace {

struct ExParams {
    const float* ml;                 // this rank's (m, l) [n_heads][2]
    const float* o;                  // this rank's o [n_heads][hd]
    ExchangeArgs ex;
    float* out;
    const float* gate;
    uint32_t n_heads, hd;
    int* status;
};

// CTA hh: this rank's part of head hh from (ml, o), then the exchange of that head.
__global__ void __launch_bounds__(128) k_exchange_merge(const ExParams p) {
    const uint32_t hh = blockIdx.x;
    __shared__ uint32_t s_epoch;
    __shared__ float s_o[256];
    exchange_epoch(p.ex, &s_epoch);
    for (uint32_t d = threadIdx.x; d < p.hd; d += blockDim.x) s_o[d] = p.o[static_cast<size_t>(hh) * p.hd + d];
    const float M = p.ml[hh * 2], L = p.ml[hh * 2 + 1];
    __syncthreads();
    const uint32_t epoch = s_epoch;
    exchange_head(p.ex, epoch, p.n_heads, p.hd, hh, M, L, s_o, p.out, p.gate, p.status);
    exchange_finish(p.ex, epoch);
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
        head_dim == 0 || head_dim > 256) {
        set_err(err, errlen, "exchange_merge: bad arguments (world 1..%u, rank < world, head_dim <= 256)", kMaxWorld);
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
        p.ex.area[r] = static_cast<uint8_t*>(areas[r]);
    }
    p.ex.world = world;
    p.ex.rank = rank;
    p.ex.wait_ns = wait_limit_ns ? wait_limit_ns : kWaitLimitNs;
    p.out = out;
    p.gate = gate;
    p.n_heads = n_heads;
    p.hd = head_dim;
    p.status = ctx->status;
    k_exchange_merge<<<n_heads, 128, 0, static_cast<cudaStream_t>(stream)>>>(p);
    YATTN_CHECK_LAUNCH(err, errlen, "exchange_merge");
    return 0;
}
