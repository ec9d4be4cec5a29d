// Causal depthwise conv1d + bias + SiLU (src/cpu_mamba/_mamba.py:211-215):
//   xc[b,t,d] = silu(bias[d] + sum_k w[d,k] * x[b, t-(K-1)+k, d]),  x[b,<0,d] = 0
// reading the x half of in_proj's output in place (row stride ld_in) and
// writing xc token-major.  Optionally also writes the conv tail of
// forward_with_final_state (_mamba.py:180): the last K-1 pre-conv inputs per
// (b, d), zero-left-padded for short sequences.
//
// HBM-bound: each thread owns one channel (two adjacent channels in bf16, so
// that a warp still moves 128 bytes per row access) and CONV_TT consecutive
// timesteps, keeping the K-1 history in registers; consecutive threads are
// consecutive channels, so every row access is one coalesced segment.
#include "internal.cuh"

namespace mb2 {

constexpr int CONV_TT = 32;   // timesteps per thread
constexpr int CONV_KMAX = 8;  // max supported d_conv

template <typename T, int K>
__device__ __forceinline__ void conv_channel(const T *__restrict__ x, int64_t ld_in,
                                             const T *__restrict__ w, const T *__restrict__ bias,
                                             T *__restrict__ xc, int64_t ld_out,
                                             T *__restrict__ tail, int64_t seqlen,
                                             int64_t d_inner, int64_t d, int64_t t0, int64_t b,
                                             float &vmax);

// amax (or null): fused maxima of |xc| for the F16X3 GEMM that reads xc next
// (AMAX_SLOTS slots, zeroed beforehand)
template <typename T, int K>
__global__ void __launch_bounds__(128)
conv1d_silu_kernel(const T *__restrict__ x, int64_t ld_in, const T *__restrict__ w,
                   const T *__restrict__ bias, T *__restrict__ xc, int64_t ld_out,
                   T *__restrict__ tail, int64_t seqlen, int64_t d_inner,
                   unsigned *__restrict__ amax) {
    const int64_t d = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t t0 = (int64_t)blockIdx.y * CONV_TT;
    const int64_t b = blockIdx.z;
    float vmax = 0.0f;
    if (d < d_inner) conv_channel<T, K>(x, ld_in, w, bias, xc, ld_out, tail, seqlen, d_inner, d,
                                        t0, b, vmax);
    if (amax) amax_publish(amax, vmax);      // block-uniform branch
}

template <typename T, int K>
__device__ __forceinline__ void conv_channel(const T *__restrict__ x, int64_t ld_in,
                                             const T *__restrict__ w, const T *__restrict__ bias,
                                             T *__restrict__ xc, int64_t ld_out,
                                             T *__restrict__ tail, int64_t seqlen,
                                             int64_t d_inner, int64_t d, int64_t t0, int64_t b,
                                             float &vmax) {
    float wk[K];
#pragma unroll
    for (int k = 0; k < K; ++k) wk[k] = io<T>::to_f(w[d * K + k]);
    const float bv = bias ? io<T>::to_f(bias[d]) : 0.0f;
    const int64_t row0 = b * seqlen;
    float hist[K];  // hist[K-1] is the current input
#pragma unroll
    for (int k = 0; k < K - 1; ++k) {
        const int64_t t = t0 - (K - 1) + k;
        hist[k] = (t >= 0) ? io<T>::to_f(x[(row0 + t) * ld_in + d]) : 0.0f;
    }
    const int64_t t_end = (t0 + CONV_TT < seqlen) ? t0 + CONV_TT : seqlen;
#pragma unroll 4
    for (int64_t t = t0; t < t_end; ++t) {
        hist[K - 1] = io<T>::to_f(x[(row0 + t) * ld_in + d]);
        float acc = bv;
#pragma unroll
        for (int k = 0; k < K; ++k) acc = fmaf(wk[k], hist[k], acc);
        const float v = io<T>::round(acc);
        const float o = silu_f(v);
        vmax = fmaxf(vmax, fabsf(o));
        xc[(row0 + t) * ld_out + d] = io<T>::from_f(o);
#pragma unroll
        for (int k = 0; k < K - 1; ++k) hist[k] = hist[k + 1];
    }
    if (tail && t_end == seqlen) {
        // after the loop hist[0..K-2] hold x[T-K+1 .. T-1] (zeros before t=0)
#pragma unroll
        for (int k = 0; k < K - 1; ++k)
            tail[(b * d_inner + d) * (K - 1) + k] = io<T>::from_f(hist[k]);
    }
}

// bf16, two channels per thread: one 4-byte load / store per row
template <int K>
__global__ void __launch_bounds__(128)
conv1d_silu_bf16x2_kernel(const __nv_bfloat16 *__restrict__ x, int64_t ld_in,
                          const __nv_bfloat16 *__restrict__ w, const __nv_bfloat16 *__restrict__ bias,
                          __nv_bfloat16 *__restrict__ xc, int64_t ld_out,
                          __nv_bfloat16 *__restrict__ tail, int64_t seqlen, int64_t d_inner) {
    using T = __nv_bfloat16;
    const int64_t d = 2 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x);
    const int64_t t0 = (int64_t)blockIdx.y * CONV_TT;
    const int64_t b = blockIdx.z;
    if (d >= d_inner) return;
    float wk[2][K];
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int k = 0; k < K; ++k) wk[c][k] = io<T>::to_f(w[(d + c) * K + k]);
    const float bv0 = bias ? io<T>::to_f(bias[d]) : 0.0f;
    const float bv1 = bias ? io<T>::to_f(bias[d + 1]) : 0.0f;
    const int64_t row0 = b * seqlen;
    auto ld2 = [&](int64_t t, float &a, float &c) {
        const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162 *>(x + (row0 + t) * ld_in + d);
        a = __low2float(v);
        c = __high2float(v);
    };
    float h0[K], h1[K];
#pragma unroll
    for (int k = 0; k < K - 1; ++k) {
        const int64_t t = t0 - (K - 1) + k;
        if (t >= 0) ld2(t, h0[k], h1[k]);
        else h0[k] = h1[k] = 0.0f;
    }
    const int64_t t_end = (t0 + CONV_TT < seqlen) ? t0 + CONV_TT : seqlen;
#pragma unroll 4
    for (int64_t t = t0; t < t_end; ++t) {
        ld2(t, h0[K - 1], h1[K - 1]);
        float a0 = bv0, a1 = bv1;
#pragma unroll
        for (int k = 0; k < K; ++k) {
            a0 = fmaf(wk[0][k], h0[k], a0);
            a1 = fmaf(wk[1][k], h1[k], a1);
        }
        const float v0 = silu_f(io<T>::round(a0)), v1 = silu_f(io<T>::round(a1));
        *reinterpret_cast<__nv_bfloat162 *>(xc + (row0 + t) * ld_out + d) =
            __floats2bfloat162_rn(v0, v1);
#pragma unroll
        for (int k = 0; k < K - 1; ++k) {
            h0[k] = h0[k + 1];
            h1[k] = h1[k + 1];
        }
    }
    if (tail && t_end == seqlen) {
#pragma unroll
        for (int k = 0; k < K - 1; ++k) {
            tail[(b * d_inner + d) * (K - 1) + k] = io<T>::from_f(h0[k]);
            tail[(b * d_inner + d + 1) * (K - 1) + k] = io<T>::from_f(h1[k]);
        }
    }
}

template <typename T, int K>
static int launch_conv(const void *x, int64_t ld_in, const void *w, const void *bias, void *xc,
                       int64_t ld_out, void *tail, int64_t batch, int64_t seqlen, int64_t di,
                       cudaStream_t st, unsigned *amax) {
    if constexpr (sizeof(T) == 2) {
        // pairs of channels: even d_inner, 4-byte aligned rows
        if (di % 2 == 0 && ld_in % 2 == 0 && ld_out % 2 == 0 && aligned(x, 4) && aligned(xc, 4)) {
            dim3 g2((unsigned)ceil_div(di / 2, 128), (unsigned)ceil_div(seqlen, CONV_TT),
                    (unsigned)batch);
            conv1d_silu_bf16x2_kernel<K><<<g2, 128, 0, st>>>(
                static_cast<const __nv_bfloat16 *>(x), ld_in, static_cast<const __nv_bfloat16 *>(w),
                static_cast<const __nv_bfloat16 *>(bias), static_cast<__nv_bfloat16 *>(xc), ld_out,
                static_cast<__nv_bfloat16 *>(tail), seqlen, di);
            return check_launch("conv1d_silu_bf16x2_kernel");
        }
    }
    dim3 grid((unsigned)ceil_div(di, 128), (unsigned)ceil_div(seqlen, CONV_TT), (unsigned)batch);
    conv1d_silu_kernel<T, K><<<grid, 128, 0, st>>>(
        static_cast<const T *>(x), ld_in, static_cast<const T *>(w), static_cast<const T *>(bias),
        static_cast<T *>(xc), ld_out, static_cast<T *>(tail), seqlen, di,
        sizeof(T) == 4 ? amax : nullptr);
    return check_launch("conv1d_silu_kernel");
}

template <typename T>
static int dispatch_conv(int K, const void *x, int64_t ld_in, const void *w, const void *bias,
                         void *xc, int64_t ld_out, void *tail, int64_t batch, int64_t seqlen,
                         int64_t di, cudaStream_t st, unsigned *amax) {
    switch (K) {
#define MB2_CONV_CASE(KK) \
    case KK: return launch_conv<T, KK>(x, ld_in, w, bias, xc, ld_out, tail, batch, seqlen, di, st, amax);
        MB2_CONV_CASE(2) MB2_CONV_CASE(3) MB2_CONV_CASE(4) MB2_CONV_CASE(5)
        MB2_CONV_CASE(6) MB2_CONV_CASE(7) MB2_CONV_CASE(8)
#undef MB2_CONV_CASE
    }
    return fail(MB2_ERR_UNSUPPORTED, "conv1d: d_conv %d not in [2, %d]", K, CONV_KMAX);
}

// Zero the conv tail when the sequence is empty (the loop above never runs).
template <typename T>
__global__ void zero_kernel(T *p, int64_t n) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = io<T>::from_f(0.0f);
}

int conv1d_silu(int dtype, const void *x_in, int64_t ld_in, const void *w, const void *bias,
                void *xc, int64_t ld_out, void *tail, int64_t batch, int64_t seqlen,
                int64_t d_inner, int64_t d_conv, cudaStream_t st, unsigned *amax) {
    MB2_REQUIRE(dtype == MB2_F32 || dtype == MB2_BF16, MB2_ERR_ARG, "conv1d: bad dtype");
    MB2_REQUIRE(batch >= 0 && seqlen >= 0 && d_inner >= 0, MB2_ERR_SHAPE, "conv1d: negative size");
    MB2_REQUIRE(d_conv >= 2 && d_conv <= CONV_KMAX, MB2_ERR_UNSUPPORTED,
                "conv1d: d_conv %lld not in [2, %d]", (long long)d_conv, CONV_KMAX);
    MB2_REQUIRE(batch < 65536 && ceil_div(seqlen, CONV_TT) < 65536, MB2_ERR_SHAPE,
                "conv1d: batch or seqlen too large");
    if (batch == 0 || d_inner == 0) return MB2_OK;
    MB2_REQUIRE(w, MB2_ERR_ARG, "conv1d: null weight");
    if (seqlen == 0) {
        if (tail) {
            const int64_t n = batch * d_inner * (d_conv - 1);
            if (dtype == MB2_F32)
                zero_kernel<float><<<(unsigned)ceil_div(n, 256), 256, 0, st>>>((float *)tail, n);
            else
                zero_kernel<__nv_bfloat16><<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(
                    (__nv_bfloat16 *)tail, n);
            return check_launch("zero_kernel");
        }
        return MB2_OK;
    }
    MB2_REQUIRE(x_in && xc, MB2_ERR_ARG, "conv1d: null pointer");
    MB2_REQUIRE(ld_in >= d_inner && ld_out >= d_inner, MB2_ERR_SHAPE, "conv1d: leading dim too small");
    if (dtype == MB2_F32)
        return dispatch_conv<float>((int)d_conv, x_in, ld_in, w, bias, xc, ld_out, tail, batch,
                                    seqlen, d_inner, st, amax);
    return dispatch_conv<__nv_bfloat16>((int)d_conv, x_in, ld_in, w, bias, xc, ld_out, tail,
                                        batch, seqlen, d_inner, st, nullptr);
}

}  // namespace mb2

extern "C" int mb2_conv1d_silu(int dtype, const void *x_in, int64_t ld_in, const void *w,
                               const void *bias, void *xc, int64_t ld_out, void *conv_tail,
                               int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_conv,
                               mb2_stream_t stream) {
    return mb2::conv1d_silu(dtype, x_in, ld_in, w, bias, xc, ld_out, conv_tail, batch, seqlen,
                            d_inner, d_conv, (cudaStream_t)stream);
}
