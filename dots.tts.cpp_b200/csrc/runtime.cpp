// Host runtime helpers (see runtime.h).
#include "runtime.h"

#include <algorithm>
#include <chrono>
#include <cstdarg>
#include <cstring>
#include <thread>

namespace dtts {

namespace {
thread_local char g_err[512] = "";
}

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

const char *last_error() { return g_err; }

int cuda_status(cudaError_t e, const char *what) {
    set_error("%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
    if (e == cudaErrorMemoryAllocation) return DTTS_ERR_OOM;
    if (e == cudaErrorNoDevice || e == cudaErrorInvalidDevice || e == cudaErrorInsufficientDriver)
        return DTTS_ERR_NO_DEVICE;
    return DTTS_ERR_CUDA;
}

static inline uint16_t bf16_rne(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);  // quiet NaN
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return static_cast<uint16_t>(u >> 16);
}

void f32_to_bf16_host(const float *src, uint16_t *dst, size_t n) {
    const size_t chunk = size_t(1) << 22;
    if (n <= chunk) {
        for (size_t i = 0; i < n; i++) dst[i] = bf16_rne(src[i]);
        return;
    }
    unsigned nt = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    std::vector<std::thread> th;
    const size_t per = (n + nt - 1) / nt;
    for (unsigned t = 0; t < nt; t++) {
        const size_t b = t * per, e = std::min(n, b + per);
        if (b >= e) break;
        th.emplace_back([=] {
            for (size_t i = b; i < e; i++) dst[i] = bf16_rne(src[i]);
        });
    }
    for (auto &x : th) x.join();
}

int check_device(int device, int *num_sms) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        cudaGetLastError();
        set_error("no CUDA device available (%s)", e == cudaSuccess ? "count 0" : cudaGetErrorString(e));
        return DTTS_ERR_NO_DEVICE;
    }
    if (device < 0 || device >= n) {
        set_error("device %d out of range (%d visible)", device, n);
        return DTTS_ERR_NO_DEVICE;
    }
    cudaDeviceProp p;
    DTTS_CUDA(cudaGetDeviceProperties(&p, device));
    if (p.major != 10) {
        set_error("device %d is sm_%d%d; this engine is built for sm_100a only", device, p.major, p.minor);
        return DTTS_ERR_NO_DEVICE;
    }
    if (num_sms) *num_sms = p.multiProcessorCount;
    return DTTS_OK;
}

int stream_wait(cudaStream_t s, double limit_s) {
    const auto t0 = std::chrono::steady_clock::now();
    int spins = 0;
    while (true) {
        cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return DTTS_OK;
        if (e != cudaErrorNotReady) return cuda_status(e, "cudaStreamQuery");
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > limit_s) {
            set_error("stream did not finish within %.0f s", limit_s);
            return DTTS_ERR_TIMEOUT;
        }
        if (++spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

}  // namespace dtts
