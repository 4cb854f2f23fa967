// capi.cu -- status, error strings and the per-device context of the C ABI.
#include "common.cuh"

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
    DevCtx* c = dev_ctx(err, errlen);
    if (!c) return -1;
    int v = 0;
    cudaError_t e = cudaMemcpy(&v, c->status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        set_err(err, errlen, "device_status: %s", cudaGetErrorString(e));
        return -1;
    }
    if (clear && cudaMemset(c->status, 0, sizeof(int)) != cudaSuccess) {
        set_err(err, errlen, "device_status: clear failed");
        return -1;
    }
    if (status_out) *status_out = v;
    return 0;
}
