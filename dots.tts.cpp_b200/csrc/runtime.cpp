// Host runtime helpers (see runtime.h).
#include "runtime.h"

#include <cmath>

#include <algorithm>
#include <chrono>
#include <cstdarg>
#include <cstring>
#include <mutex>
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

// e4m3: 1 sign bit, 4 exponent bits (bias 7), 3 mantissa bits, largest finite
// 448, subnormals m * 2^-9, no infinities.  Round to nearest even, saturating.
uint8_t e4m3_encode_host(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    const uint8_t sign = static_cast<uint8_t>((u >> 24) & 0x80u);
    const uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return sign | 0x7f;    // NaN
    if (a >= 0x43e00000u) return sign | 0x7e;   // |x| >= 448 (or inf): saturate
    if (a < 0x3c800000u) {                      // |x| < 2^-6: multiples of 2^-9
        float f;
        std::memcpy(&f, &a, 4);
        return sign | static_cast<uint8_t>(std::nearbyint(f * 512.0f));   // 8 = 2^-6, the smallest normal
    }
    // keep 3 of the 23 mantissa bits, rounding to nearest even at bit 20 (a
    // carry moves into the exponent), then rebias the exponent from 127 to 7
    const uint32_t r = (a + 0x7ffffu + ((a >> 20) & 1u)) >> 20;
    return sign | static_cast<uint8_t>(r - (120u << 3));
}

float e4m3_decode_host(uint8_t b) {
    const int E = (b >> 3) & 15, m = b & 7;
    if (E == 15 && m == 7) return std::nanf("");
    const float v = E == 0 ? std::ldexp(static_cast<float>(m), -9) : std::ldexp(static_cast<float>(8 + m), E - 10);
    return (b & 0x80) ? -v : v;
}

void e4m3_quantize_rows(const float *w, size_t rows, size_t cols, uint8_t *q, float *scale, float *row_norm) {
    float dec[256];
    for (int i = 0; i < 256; i++) dec[i] = e4m3_decode_host(static_cast<uint8_t>(i));
    auto work = [&](size_t r0, size_t r1) {
        for (size_t r = r0; r < r1; r++) {
            const float *src = w + r * cols;
            uint8_t *dst = q + r * cols;
            float amax = 0.f;
            for (size_t c = 0; c < cols; c++) amax = std::max(amax, std::fabs(src[c]));
            if (amax == 0.f) {
                std::memset(dst, 0, cols);
                scale[r] = 0.f;
                if (row_norm) row_norm[r] = 0.f;
                continue;
            }
            const float inv = 448.0f / amax, s = amax / 448.0f;
            float ss = 0.f;
            for (size_t c = 0; c < cols; c++) {
                dst[c] = e4m3_encode_host(src[c] * inv);
                const float d = dec[dst[c]] * s;
                ss += d * d;
            }
            scale[r] = s;
            if (row_norm) row_norm[r] = std::sqrt(ss);
        }
    };
    const size_t total = rows * cols;
    unsigned nt = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    if (total < (size_t(1) << 20) || nt == 1) { work(0, rows); return; }
    std::vector<std::thread> th;
    const size_t per = (rows + nt - 1) / nt;
    for (unsigned t = 0; t < nt; t++) {
        const size_t b = t * per, e = std::min(rows, b + per);
        if (b >= e) break;
        th.emplace_back(work, b, e);
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

namespace {
struct L2Persist {
    int refs = 0;
    size_t orig = 0, cur = 0;
};
std::mutex g_l2_mutex;
L2Persist g_l2[64];
}  // namespace

size_t l2_persist_acquire(int dev, size_t want) {
    if (dev < 0 || dev >= 64) return 0;
    std::lock_guard<std::mutex> lock(g_l2_mutex);
    L2Persist &p = g_l2[dev];
    int max_persist = 0;
    if (cudaDeviceGetAttribute(&max_persist, cudaDevAttrMaxPersistingL2CacheSize, dev) != cudaSuccess ||
        max_persist <= 0) {
        cudaGetLastError();
        return 0;
    }
    if (p.refs == 0) {
        size_t orig = 0;
        if (cudaDeviceGetLimit(&orig, cudaLimitPersistingL2CacheSize) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        p.orig = p.cur = orig;
    }
    const size_t target = std::min(want, (size_t)max_persist);
    if (target > p.cur) {
        if (cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, target) != cudaSuccess) {
            cudaGetLastError();
            if (p.refs == 0) return 0;
        } else {
            p.cur = target;
        }
    }
    p.refs++;
    return p.cur;
}

void l2_persist_release(int dev) {
    if (dev < 0 || dev >= 64) return;
    std::lock_guard<std::mutex> lock(g_l2_mutex);
    L2Persist &p = g_l2[dev];
    if (p.refs <= 0) return;
    if (--p.refs == 0) {
        cudaCtxResetPersistingL2Cache();
        cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, p.orig);
        cudaGetLastError();
        p.cur = p.orig;
    }
}

}  // namespace dtts
