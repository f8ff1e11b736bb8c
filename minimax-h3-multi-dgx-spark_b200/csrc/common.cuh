// Shared device/host helpers for libh3b (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/h3b.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libh3b is built for sm_100a only"
#endif

namespace h3b {

// ---------------------------------------------------------------------------
// Error reporting.  Host entry points return H3B_OK or a negative code and
// leave a message retrievable with h3b_last_error().  Kernels report
// exhausted waits through a device status word (first error wins).

int set_error(int code, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what);

#define H3B_CUDA_TRY(expr)                                   \
    do {                                                     \
        cudaError_t _e = (expr);                             \
        if (_e != cudaSuccess) return ::h3b::cuda_error(_e, #expr); \
    } while (0)

#define H3B_REQUIRE(cond, ...)                                          \
    do {                                                                \
        if (!(cond)) return ::h3b::set_error(H3B_ERR_ARG, __VA_ARGS__); \
    } while (0)

// The device status word lives in status.cu; kernels in other translation
// units reach it through this pointer (relocatable device code is not used).
struct DeviceStatus {
    int* word;  // device address of the status word
};
int device_status(DeviceStatus* out);

__device__ __forceinline__ void report(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------
// bf16 helpers

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// float -> bf16 round-to-nearest-even (== __float2bfloat16_rn for finite values)
__device__ __forceinline__ uint32_t f2bf_bits(float f) {
    return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(f));
}
// Two floats -> packed bf16x2 (lo in bits 0-15), round-to-nearest-even, one
// paired conversion instead of two scalar ones.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}
// round to bf16 precision and return as float (the reference's _rbf16)
__device__ __forceinline__ float rbf16(float f) { return __uint_as_float(f2bf_bits(f) << 16); }

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline bool aligned(const void* p, uintptr_t a) { return ((uintptr_t)p % a) == 0; }

}  // namespace h3b
