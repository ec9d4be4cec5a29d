// CUDA-core GEMM: y[m, n] = sum_k x[m, k] * W[n, k] (+ bias[n]), fp32 FMA
// accumulation, with the weight tile produced by a loader policy:
//   dense  -- W in the activation dtype (nn.Linear, _mamba.py:67,74,75,84)
//   int8 / int4 / nf4 -- W dequantised on the fly from weight_q + scale with
//            exactly quant.py's arithmetic (q.float() * scale, :68-69, :90-101,
//            :124-134), then rounded to the activation dtype like
//            QuantizedLinear.forward's w.to(x.dtype) (:188-190).
// Used where the tensor-core kernel does not apply (small M: the single-token
// step; quantised weights) and as the exact-fp32 path.
//
// Tile 128 x 64 x 16, 256 threads, 8 x 4 outputs per thread, register-prefetch
// double buffer.  An optional column remap writes x_proj's three output
// segments (dt_low | B | C) to separately aligned column offsets.
#include "internal.cuh"

namespace mb2 {

constexpr int SG_BM = 128, SG_BN = 64, SG_BK = 16, SG_THREADS = 256;

enum BMode { BM_DENSE = 0, BM_INT8 = 1, BM_INT4 = 2, BM_NF4 = 3 };

struct GemmArgs {
    const void *x; int64_t ld_x;
    const void *w;                 // dense W (N, K) or codes
    const float *scale;            // per-row scale (quantised)
    const void *bias;
    void *y; int64_t ld_y;
    int64_t M, N, K;
    int64_t n1, n2, off1, off2;    // output column remap
    int epi;                       // MB2_EPI_NONE / MB2_EPI_SOFTPLUS
    float lut[16];                 // nf4 code book (quant.py:35-40), by value
    const float *row_scale;        // EpiExtra terms
    const void *resid; int64_t ld_r;
};

// quant.py:35-40: a tuple of Python floats turned into a float32 tensor, i.e.
// decimal -> double -> float; casting double literals reproduces it exactly.
void nf4_lut(float *out16) {
    static const double lut_d[16] = {
        -1.0, -0.6961928, -0.5250730, -0.39491748, -0.28444138, -0.18477343,
        -0.09105602, 0.0, 0.07958029, 0.16093020, 0.24611230, 0.33791524,
        0.44070983, 0.56261897, 0.72295684, 1.0};
    for (int i = 0; i < 16; ++i) out16[i] = (float)lut_d[i];
}

template <typename T, int MODE>
__device__ __forceinline__ float load_w(const GemmArgs &a, int64_t n, int64_t k) {
    if (MODE == BM_DENSE) return io<T>::to_f(static_cast<const T *>(a.w)[n * a.K + k]);
    const float s = a.scale[n];
    if (MODE == BM_INT8) {
        const int8_t q = static_cast<const int8_t *>(a.w)[n * a.K + k];
        return io<T>::round((float)q * s);
    }
    const int64_t pcols = (a.K + 1) >> 1;
    const uint8_t byte = static_cast<const uint8_t *>(a.w)[n * pcols + (k >> 1)];
    const int nib = (k & 1) ? (byte & 0x0F) : (byte >> 4);
    if (MODE == BM_INT4) return io<T>::round((float)(nib - 7) * s);
    return io<T>::round(a.lut[nib] * s);
}

template <typename T, int MODE>
__global__ void __launch_bounds__(SG_THREADS)
gemm_simt_kernel(const GemmArgs a) {
    __shared__ __align__(16) float As[2][SG_BK][SG_BM];
    __shared__ __align__(16) float Bs[2][SG_BK][SG_BN];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = (int64_t)blockIdx.y * SG_BM;
    const int64_t n0 = (int64_t)blockIdx.x * SG_BN;
    const T *X = static_cast<const T *>(a.x);

    // A loader: row = tid / 2, 8 consecutive k at (tid & 1) * 8
    const int a_row = tid >> 1, a_k = (tid & 1) * 8;
    // B loader: row = tid / 4, 4 consecutive k at (tid & 3) * 4
    const int b_row = tid >> 2, b_k = (tid & 3) * 4;
    float ra[8], rb[4];

    auto load_tile = [&](int64_t k0) {
        const int64_t m = m0 + a_row;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t k = k0 + a_k + i;
            ra[i] = (m < a.M && k < a.K) ? io<T>::to_f(X[m * a.ld_x + k]) : 0.0f;
        }
        const int64_t n = n0 + b_row;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t k = k0 + b_k + i;
            rb[i] = (n < a.N && k < a.K) ? load_w<T, MODE>(a, n, k) : 0.0f;
        }
    };
    auto store_tile = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 8; ++i) As[buf][a_k + i][a_row] = ra[i];
#pragma unroll
        for (int i = 0; i < 4; ++i) Bs[buf][b_k + i][b_row] = rb[i];
    };

    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[i][jj] = 0.0f;

    const int64_t nk = ceil_div(a.K, SG_BK);
    load_tile(0);
    store_tile(0);
    __syncthreads();
    for (int64_t kt = 0; kt < nk; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < nk) load_tile((kt + 1) * SG_BK);
#pragma unroll
        for (int k = 0; k < SG_BK; ++k) {
            const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][k][ty * 8]);
            const float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][k][ty * 8 + 4]);
            const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][k][tx * 4]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float bv[4] = {b0.x, b0.y, b0.z, b0.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) acc[i][jj] = fmaf(av[i], bv[jj], acc[i][jj]);
        }
        if (kt + 1 < nk) store_tile(buf ^ 1);
        __syncthreads();
    }

    T *Y = static_cast<T *>(a.y);
    const T *bias = static_cast<const T *>(a.bias);
    // optional terms, each behind one branch for the whole 8 x 4 block (a
    // per-element test of the softplus would spread its inlined body over
    // 32 instruction-cache lines)
    if (a.row_scale) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t m = m0 + ty * 8 + i;
            const float rs = m < a.M ? a.row_scale[m] : 1.0f;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) acc[i][jj] *= rs;
        }
    }
    if (bias) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int64_t n = n0 + tx * 4 + jj;
            const float bv = n < a.N ? io<T>::to_f(bias[n]) : 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i][jj] += bv;
        }
    }
    if (a.epi == MB2_EPI_SOFTPLUS) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) acc[i][jj] = softplus_f(io<T>::round(acc[i][jj]));
    }
    if (a.resid) {
        const T *R = static_cast<const T *>(a.resid);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t m = m0 + ty * 8 + i;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int64_t n = n0 + tx * 4 + jj;
                if (m < a.M && n < a.N) acc[i][jj] += io<T>::to_f(R[m * a.ld_r + n]);
            }
        }
    }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
        const int64_t n = n0 + tx * 4 + jj;
        if (n >= a.N) continue;
        const int64_t col = n + (n >= a.n1 ? a.off1 : 0) + (n >= a.n2 ? a.off2 : 0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t m = m0 + ty * 8 + i;
            if (m < a.M) Y[m * a.ld_y + col] = io<T>::from_f(acc[i][jj]);
        }
    }
}

template <typename T, int MODE>
static int launch_simt(const GemmArgs &a, cudaStream_t st) {
    dim3 grid((unsigned)ceil_div(a.N, SG_BN), (unsigned)ceil_div(a.M, SG_BM));
    gemm_simt_kernel<T, MODE><<<grid, SG_THREADS, 0, st>>>(a);
    return check_launch("gemm_simt_kernel");
}

// Internal: dense or quantised CUDA-core GEMM with optional column remap.
int gemm_simt(int dtype, int scheme, const void *x, int64_t ld_x, const void *w,
              const float *scale, const void *bias, void *y, int64_t ld_y, int64_t M,
              int64_t N, int64_t K, int64_t n1, int64_t off1, int64_t n2, int64_t off2,
              int epi, cudaStream_t st, const EpiExtra &ex) {
    MB2_REQUIRE(M >= 0 && N >= 0 && K >= 0, MB2_ERR_SHAPE, "linear: negative size");
    MB2_REQUIRE(ceil_div(M, SG_BM) <= 65535, MB2_ERR_SHAPE, "linear: M too large");
    if (M == 0 || N == 0) return MB2_OK;
    MB2_REQUIRE(x && w && y, MB2_ERR_ARG, "linear: null pointer");
    MB2_REQUIRE(scheme == MB2_Q_NONE || scale, MB2_ERR_ARG, "linear: quantised weight needs scale");
    GemmArgs a{x, ld_x, w, scale, bias, y, ld_y, M, N, K, n1, n2, off1, off2, epi, {},
               ex.row_scale, ex.resid, ex.ld_r};
    nf4_lut(a.lut);
    const bool f32 = dtype == MB2_F32;
    switch (scheme) {
        case MB2_Q_NONE: return f32 ? launch_simt<float, BM_DENSE>(a, st) : launch_simt<__nv_bfloat16, BM_DENSE>(a, st);
        case MB2_Q_INT8: return f32 ? launch_simt<float, BM_INT8>(a, st) : launch_simt<__nv_bfloat16, BM_INT8>(a, st);
        case MB2_Q_INT4: return f32 ? launch_simt<float, BM_INT4>(a, st) : launch_simt<__nv_bfloat16, BM_INT4>(a, st);
        case MB2_Q_NF4: return f32 ? launch_simt<float, BM_NF4>(a, st) : launch_simt<__nv_bfloat16, BM_NF4>(a, st);
    }
    return fail(MB2_ERR_ARG, "linear: unknown scheme %d", scheme);
}

}  // namespace mb2
