// Shared helpers for the B200 Mamba kernels: status/error reporting, dtype
// conversion, async copy (LDGSTS) primitives and small math helpers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/mamba_b200.h"

namespace mb2 {

// ---------------------------------------------------------------- errors ---
void set_error(const char *fmt, ...);
int fail(int code, const char *fmt, ...);
int check_launch(const char *what);

#define MB2_REQUIRE(cond, code, ...)                                        \
    do {                                                                    \
        if (!(cond)) return ::mb2::fail((code), __VA_ARGS__);               \
    } while (0)

#define MB2_TRY(expr)                                                       \
    do {                                                                    \
        int _rc = (expr);                                                   \
        if (_rc != MB2_OK) return _rc;                                      \
    } while (0)

inline bool aligned(const void *p, size_t bytes) {
    return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ inline int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

inline size_t dtype_size(int dtype) { return dtype == MB2_BF16 ? 2 : 4; }

// ------------------------------------------------------------- dtype I/O ---
template <typename T> struct io;
template <> struct io<float> {
    static __device__ __forceinline__ float load(const float *p) { return *p; }
    static __device__ __forceinline__ float cvt(float v) { return v; }
    static __device__ __forceinline__ float to_f(float v) { return v; }
    static __device__ __forceinline__ float from_f(float v) { return v; }
    // value after a round trip through the storage type (identity for fp32)
    static __device__ __forceinline__ float round(float v) { return v; }
};
template <> struct io<__nv_bfloat16> {
    static __device__ __forceinline__ float load(const __nv_bfloat16 *p) {
        return __bfloat162float(*p);
    }
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) {
        return __bfloat162float(v);
    }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) {
        return __float2bfloat16_rn(v);
    }
    static __device__ __forceinline__ float round(float v) {
        return __bfloat162float(__float2bfloat16_rn(v));
    }
};

// ------------------------------------------------------------ async copy ---
// Ampere-style LDGSTS: 4-byte copies work for any 4-byte aligned address, so
// they stage arbitrary (unpadded) layouts; the TMA path is used where the
// layout is under this library's control.
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async4(void *smem, const void *gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(smem)),
                 "l"(gmem));
}
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)),
                 "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;\n" ::);
}
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// ------------------------------------------------------------------ math ---
constexpr float kLog2e = 1.4426950408889634f;

// torch.nn.functional.softplus with beta=1, threshold=20.
__device__ __forceinline__ float softplus_f(float v) {
    return v > 20.0f ? v : log1pf(expf(v));
}
// SiLU v * sigmoid(v) as v / (1 + e^-v).
// fp32 -> TF32 (10 explicit mantissa bits), rounded to nearest, ties away
__device__ __forceinline__ float tf32_round(float v) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return __uint_as_float(r);
}

__device__ __forceinline__ float silu_f(float v) {
    return __fdividef(v, 1.0f + __expf(-v));
}

}  // namespace mb2
