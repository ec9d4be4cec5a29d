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

// ----------------------------------------- programmatic dependent launch ---
// The decode step is a chain of short dependent kernels.  Launched with
// programmatic stream serialisation, a kernel may start while the kernel
// before it still runs: it does what needs nothing from that kernel first
// (barrier and TMEM set-up, weight tiles, state that kernel does not write),
// then pdl_wait() blocks until that kernel has completed and its writes are
// visible, and pdl_trigger() lets the next kernel start.  Every kernel of the
// chain triggers only after its own wait, so at most two are in flight: the
// part before a kernel's wait runs beside the previous kernel only, and reads
// nothing that kernel writes.  Without the launch attribute both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// kern<<<grid, block, smem, st>>>(args...), with programmatic stream
// serialisation when pdl is set.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block,
                                 size_t smem, cudaStream_t st, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl ? attr : nullptr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

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

__device__ __forceinline__ float ex2(float v) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}

// torch.nn.functional.softplus with beta 1: max(v, 0) + log1p(e), e = exp(-|v|)
// (for v > 20 the sum rounds to v, torch's threshold branch).
//   e: Cody-Waite range reduction (n = rint(-|v| log2 e), r = -|v| - n ln2 with
//      ln2 split into a 16-significant-bit head and a tail), e = 2^n 2^(r log2 e)
//      with 2^n built exactly in the exponent field.  n comes from adding
//      1.5 * 2^23, which leaves rint(-|v| log2 e) in the low bits of the sum
//      (|n| <= 126), so no float-to-integer conversion occupies the MUFU pipe:
//      the function issues two MUFU operations (ex2, rcp);
//   log1p(e) = 2 atanh(u), u = e / (2 + e) in [0, 1/3], and atanh(u) / u is a
//      degree-4 polynomial in u^2 fitted (relative-error least squares,
//      float64) for this library: max relative error 4e-9 on [0, 1/9].
// fp32 result within ~4 ulp of log1p(exp(v)) (float64) for all v; about a
// third of the instructions of log1pf(expf(v)).  Every kernel of the library
// that applies dt_proj's softplus uses this one function, so the tensor-core
// epilogues, the CUDA-core GEMM and the scans agree bit for bit.
__device__ __forceinline__ float softplus_f(float v) {
    constexpr float kLn2Hi = 0.693145751953125f;      // 16 significant bits of ln 2
    constexpr float kLn2Lo = 1.428606765330187e-06f;  // ln 2 - kLn2Hi
    constexpr float c0 = 1.0f, c1 = 0.3333315849304199f, c2 = 0.20012454688549042f,
                    c3 = 0.13980302214622498f, c4 = 0.1408916562795639f;
    constexpr float kRound = 12582912.0f;             // 1.5 * 2^23
    const float a = fminf(fabsf(v), 87.0f);
    const float t = fmaf(-a, kLog2e, kRound);         // kRound + n, n = rint(-a log2 e)
    const float n = t - kRound;                       // exact
    float r = fmaf(n, -kLn2Hi, -a);
    r = fmaf(n, -kLn2Lo, r);
    const float e = ex2(r * kLog2e) *
                    __int_as_float((__float_as_int(t) - __float_as_int(kRound) + 127) << 23);
    const float u = __fdividef(e, 2.0f + e);
    const float w = u * u;
    float P = fmaf(w, c4, c3);
    P = fmaf(w, P, c2);
    P = fmaf(w, P, c1);
    P = fmaf(w, P, c0);
    return fmaxf(v, 0.0f) + (2.0f * u) * P;
}

// fp32 -> TF32 (10 explicit mantissa bits), rounded to nearest, ties away
__device__ __forceinline__ float tf32_round(float v) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return __uint_as_float(r);
}

// SiLU v * sigmoid(v) as v / (1 + e^-v).
__device__ __forceinline__ float silu_f(float v) {
    return __fdividef(v, 1.0f + __expf(-v));
}

}  // namespace mb2
