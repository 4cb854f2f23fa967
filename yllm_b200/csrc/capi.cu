// capi.cu -- status, error strings and the per-device context of the C ABI.
#include "common.cuh"
#include "tcgen05.cuh"

#include <cudaTypedefs.h>

#include <mutex>
#include <stdarg.h>
#include <string>

namespace yattn {

namespace {
thread_local std::string g_last_error;
std::mutex g_ctx_mu;
DevCtx g_ctx[64];
}  // namespace

void set_err(char* err, size_t errlen, const char* fmt, ...) {
    if (!err || errlen == 0) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, errlen, fmt, ap);
    va_end(ap);
}

void set_last_error(const char* msg) { g_last_error = msg ? msg : "unknown error"; }

DevCtx* dev_ctx(char* err, size_t errlen) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) {
        set_err(err, errlen, "no usable CUDA device: %s", cudaGetErrorString(e));
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_ctx_mu);
    DevCtx& c = g_ctx[dev];
    if (c.device == dev) return &c;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    int* st = nullptr;
    if (cudaMalloc(&st, 256) != cudaSuccess || cudaMemset(st, 0, 256) != cudaSuccess) {
        set_err(err, errlen, "device %d: status word allocation failed", dev);
        return nullptr;
    }
    c.num_sms = sms;
    c.status = st;
    c.device = dev;
    return &c;
}

// ------------------------------------------------------------- tensor maps

namespace {
PFN_cuTensorMapEncodeTiled_v12000 get_encode(char* err, size_t errlen) {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn) return fn;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !ptr) {
        set_err(err, errlen, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(e));
        return nullptr;
    }
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    return fn;
}
}  // namespace

int encode_kv_map(CUtensorMap* map, const void* base, uint32_t kv_dim, uint64_t n_rows, uint32_t box_rows, char* err,
                  size_t errlen) {
    auto enc = get_encode(err, errlen);
    if (!enc) return -1;
    cuuint64_t dims[2] = {kv_dim, n_rows};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(kv_dim) * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_err(err, errlen, "cuTensorMapEncodeTiled failed (%d): kv_dim %u, %llu rows, box %u", static_cast<int>(r),
                kv_dim, static_cast<unsigned long long>(n_rows), box_rows);
        return -1;
    }
    return 0;
}

int encode_f32_store_map(CUtensorMap* map, void* base, uint32_t cols, uint32_t stride_elems, uint64_t n_rows,
                         uint32_t box_rows, char* err, size_t errlen) {
    auto enc = get_encode(err, errlen);
    if (!enc) return -1;
    cuuint64_t dims[2] = {cols, n_rows};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride_elems) * 4};
    cuuint32_t box[2] = {32, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_err(err, errlen, "cuTensorMapEncodeTiled (fp32 store map) failed (%d): %u cols, stride %u, %llu rows",
                static_cast<int>(r), cols, stride_elems, static_cast<unsigned long long>(n_rows));
        return -1;
    }
    return 0;
}

int dev_num_sms() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) return 148;
    return sms;
}

}  // namespace yattn

using namespace yattn;

extern "C" int yattn_version(void) { return 1 * 10000 + 0 * 100 + 0; }

extern "C" const char* yattn_last_error(void) { return g_last_error.c_str(); }

extern "C" void yattn_clear_error(void) { g_last_error.clear(); }

extern "C" int yattn_device_status(int* status_out, int clear, char* err, size_t errlen) {
    // Two words can hold a code: the context's (every allocating entry point) and the
    // allocation-free decode's, inside its static scratch.  Neither is created here if it
    // does not exist yet, so a caller that only uses the allocation-free entry point
    // allocates nothing by polling.
    int* words[2] = {nullptr, noalloc_status_word()};
    {
        int dev = -1;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
            set_err(err, errlen, "device_status: no usable CUDA device");
            return -1;
        }
        std::lock_guard<std::mutex> lk(g_ctx_mu);
        if (g_ctx[dev].device == dev) words[0] = g_ctx[dev].status;
    }
    int v = 0;
    for (int* w : words) {
        if (!w) continue;
        int x = 0;
        cudaError_t e = cudaMemcpy(&x, w, sizeof(int), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) {
            set_err(err, errlen, "device_status: %s", cudaGetErrorString(e));
            return -1;
        }
        if (v == 0) v = x;
        if (clear && x != 0 && cudaMemset(w, 0, sizeof(int)) != cudaSuccess) {
            set_err(err, errlen, "device_status: clear failed");
            return -1;
        }
    }
    if (status_out) *status_out = v;
    return 0;
}
