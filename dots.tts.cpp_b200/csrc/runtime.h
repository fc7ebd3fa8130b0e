// Host runtime shared by the engines: status/error reporting, device guard,
// owned device allocations, bf16 conversion of host weights.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

#include "../../include/dtts.h"

namespace dtts {

void set_error(const char *fmt, ...);
const char *last_error();

// Records the CUDA error (with the call site) and returns DTTS_ERR_CUDA / OOM.
int cuda_status(cudaError_t e, const char *what);

#define DTTS_CUDA(call)                                          \
    do {                                                         \
        cudaError_t _e = (call);                                 \
        if (_e != cudaSuccess) return ::dtts::cuda_status(_e, #call); \
    } while (0)

#define DTTS_CHECK(cond, code, ...)          \
    do {                                     \
        if (!(cond)) {                       \
            ::dtts::set_error(__VA_ARGS__);  \
            return (code);                   \
        }                                    \
    } while (0)

// Makes `dev` current for the scope and restores the caller's device.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// Owns device allocations of one engine.
struct DeviceArena {
    std::vector<void *> ptrs;
    size_t bytes = 0;
    void *alloc(size_t n) {
        void *p = nullptr;
        if (n == 0) n = 16;
        if (cudaMalloc(&p, n) != cudaSuccess) return nullptr;
        ptrs.push_back(p);
        bytes += n;
        return p;
    }
    void release(void *p) {
        for (auto &q : ptrs)
            if (q == p) { cudaFree(q); q = nullptr; }
    }
    void free_all() {
        for (void *p : ptrs)
            if (p) cudaFree(p);
        ptrs.clear();
        bytes = 0;
    }
};

// Host fp32 -> bf16 (round to nearest even), multithreaded for large arrays.
void f32_to_bf16_host(const float *src, uint16_t *dst, size_t n);

// e4m3 (round to nearest even, saturating at +-448) on the host.
uint8_t e4m3_encode_host(float x);
float e4m3_decode_host(uint8_t b);
// Per-row (output-channel) e4m3 quantisation of w [rows][cols]:
// scale[r] = amax_r / 448, q = e4m3(w * 448 / amax_r); row_norm (optional)
// receives the L2 norm of each dequantised row.
void e4m3_quantize_rows(const float *w, size_t rows, size_t cols, uint8_t *q, float *scale, float *row_norm);

// Checks that a device with this ordinal exists and is sm_100; fills num_sms.
int check_device(int device, int *num_sms);

// Bounded host wait on a stream: polls cudaStreamQuery until done or limit.
int stream_wait(cudaStream_t s, double limit_s);

// L2 set-aside for persisting accesses on the current device, shared by the
// engines of this process: l2_persist_acquire raises the set-aside to at least
// `want` bytes (capped by the device maximum) and takes a reference;
// l2_persist_release drops it, and the last release flushes the persisting
// lines and restores the limit the process had before.  Returns the bytes set
// aside (0 where the device or the driver offers none).  The limit belongs to
// this process's context and ends with it.
size_t l2_persist_acquire(int dev, size_t want);
void l2_persist_release(int dev);

}  // namespace dtts
