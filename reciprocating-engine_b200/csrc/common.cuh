// Shared device/host helpers for libreng_cuda (sm_100a only).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>

#include "../../include/reng_cuda.h"

namespace reng {

// ---------------------------------------------------------------- errors --
// The C ABI never throws: every entry point returns RENG_OK or a negative
// code and leaves a message in thread-local storage (reng_last_error()).
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);

#define RENG_CUDA_TRY(expr)                                                         \
    do {                                                                            \
        cudaError_t e__ = (expr);                                                   \
        if (e__ != cudaSuccess)                                                     \
            return ::reng::fail(RENG_E_CUDA, std::string(#expr) + ": " +            \
                                                 cudaGetErrorString(e__));          \
    } while (0)

#define RENG_CHECK_ARG(cond, msg)                                                   \
    do {                                                                            \
        if (!(cond)) return ::reng::fail(RENG_E_INVAL, (msg));                      \
    } while (0)

// Up to four CUDA events, destroyed on every return path of the host call
// that made them.
struct EventSet {
    cudaEvent_t e[4] = {};
    int n = 0;
    cudaError_t create(int k) {
        for (; n < k && n < 4; n++) {
            cudaError_t r = cudaEventCreate(&e[n]);
            if (r != cudaSuccess) return r;
        }
        return cudaSuccess;
    }
    ~EventSet() {
        for (int i = 0; i < n; i++) cudaEventDestroy(e[i]);
    }
};

// ------------------------------------------------------------ bf16 bits --
__host__ __device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(b << 16);
#else
    uint32_t u = b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}

// f32 -> bf16 bits, round to nearest even, NaN -> 0x7fc0 (the reference's
// conversion, reng-synapse/src/lib.rs:10-19).
__host__ __device__ __forceinline__ uint16_t f32_to_bf16_bits(float x) {
#ifdef __CUDA_ARCH__
    uint32_t u = __float_as_uint(x);
#else
    uint32_t u;
    memcpy(&u, &x, 4);
#endif
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
    uint32_t rb = 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)((u + rb) >> 16);
}

// Round an f32 to the nearest bf16 value (RNE), returned as f32.
__device__ __forceinline__ float round_bf16(float x) {
    return bf16_bits_to_f32(f32_to_bf16_bits(x));
}

// Two bf16 packed in a u32 (low half first in memory) -> two f32.
__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
}

// ------------------------------------------------------------ PTX forms --
// 16-byte streaming load that does not allocate in L1 (weights are read
// exactly once per step; keep L1 for the activations).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// 16-byte read-only load through L1 (activations shared by many warps).
__device__ __forceinline__ uint4 ldg_nc(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Programmatic dependent launch: wait for the previous grid's memory, and
// let the next grid start its independent prologue early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// D(16x8 f32) += A(16x16 bf16, row) * B(16x8 bf16, col).
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col).
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two E4M3 codes (low byte first) -> two f16 (low half first).  Exact: every
// E4M3 value is an f16 value.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_codes) {
    uint32_t r;
    asm("{\n .reg .b16 t;\n cvt.u16.u32 t, %1;\n cvt.rn.f16x2.e4m3x2 %0, t;\n}\n" : "=r"(r) : "r"(two_codes));
    return r;
}

// bf16 pair -> f16 pair (activations are far inside the f16 range).
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t v) {
    __half2 h = __floats2half2_rn(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Device properties cached per device ordinal.
int num_sms(int device);

}  // namespace reng
