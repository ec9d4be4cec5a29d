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
// Tile BMT x 64 x 16 (BMT = 128, or 64 for the few-row GEMMs of the decode
// step), 256 threads, (BMT/16) x 4 outputs per thread, register-prefetch
// double buffer.  With scratch from the caller the K range is split over
// blockIdx.z (the decode step's projections have too few output tiles to fill
// the GPU): each split writes fp32 partial sums and splitk_reduce_kernel adds
// them in a fixed order (deterministic) and applies the epilogue.  An optional
// column remap writes x_proj's three output segments (dt_low | B | C) to
// separately aligned column offsets.
#include "internal.cuh"

namespace mb2 {

constexpr int SG_BM = 128, SG_BN = 64, SG_BK = 16, SG_THREADS = 256;

enum BMode { BM_DENSE = 0, BM_INT8 = 1, BM_INT4 = 2, BM_NF4 = 3 };

struct GemmArgs {
    const void *x; int64_t ld_x;
    const void *w;                 // dense W (N, K) or codes
    const float *scale;            // scale per row, or per (row, group) (quantised)
    int64_t group, ngroups;        // columns per scale group (0: one scale per row)
    const void *bias;
    void *y; int64_t ld_y;
    int64_t M, N, K;
    int64_t n1, n2, off1, off2;    // output column remap
    int epi;                       // MB2_EPI_NONE / MB2_EPI_SOFTPLUS
    float lut[16];                 // nf4 code book (quant.py:35-40), by value
    const float *row_scale;        // EpiExtra terms
    const void *resid; int64_t ld_r;
    float *partial;                // split-K: (splits, M, N) fp32 partial sums, or null
    int64_t kchunk;                // K range per split (multiple of SG_BK)
    int vec;                       // dense rows of x and W start 4-element aligned: vector loads
    int64_t silu_from;             // columns >= silu_from get SiLU (EpiExtra), < 0: none
};

// 4 consecutive elements of a row as floats, one 16-byte (fp32) or 8-byte
// (bf16) load
template <typename T>
__device__ __forceinline__ void load4(const T *p, float (&v)[4]);
template <>
__device__ __forceinline__ void load4<float>(const float *p, float (&v)[4]) {
    const float4 q = *reinterpret_cast<const float4 *>(p);
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
}
template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16 *p, float (&v)[4]) {
    const uint2 q = *reinterpret_cast<const uint2 *>(p);
    v[0] = __uint_as_float(q.x << 16); v[1] = __uint_as_float(q.x & 0xFFFF0000u);
    v[2] = __uint_as_float(q.y << 16); v[3] = __uint_as_float(q.y & 0xFFFF0000u);
}

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
    const float s = a.group ? a.scale[n * a.ngroups + k / a.group] : a.scale[n];
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

template <typename T, int MODE, int BMT>
__global__ void __launch_bounds__(SG_THREADS)
gemm_simt_kernel(const GemmArgs a) {
    constexpr int TM = BMT / 16;                       // output rows per thread
    constexpr int AL = BMT * SG_BK / SG_THREADS;       // A elements loaded per thread
    __shared__ __align__(16) float As[2][SG_BK][BMT];
    __shared__ __align__(16) float Bs[2][SG_BK][SG_BN];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = (int64_t)blockIdx.y * BMT;
    const int64_t n0 = (int64_t)blockIdx.x * SG_BN;
    const T *X = static_cast<const T *>(a.x);
    // this split's K range
    const int64_t kbeg = (int64_t)blockIdx.z * a.kchunk;
    const int64_t kend = (kbeg + a.kchunk < a.K) ? kbeg + a.kchunk : a.K;

    // A loader: row = tid / (SG_BK / AL), AL consecutive k
    const int a_row = tid / (SG_BK / AL), a_k = (tid % (SG_BK / AL)) * AL;
    // B loader: row = tid / 4, 4 consecutive k at (tid & 3) * 4
    const int b_row = tid >> 2, b_k = (tid & 3) * 4;
    float ra[AL], rb[4];

    auto load_tile = [&](int64_t k0) {
        const int64_t m = m0 + a_row;
        if (a.vec) {
            // K % 4 == 0: every 4-element group is wholly inside or outside [0, kend)
#pragma unroll
            for (int i = 0; i < AL; i += 4) {
                const int64_t k = k0 + a_k + i;
                float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (m < a.M && k < kend) load4<T>(X + m * a.ld_x + k, v);
#pragma unroll
                for (int e = 0; e < 4; ++e) ra[i + e] = v[e];
            }
        } else {
#pragma unroll
            for (int i = 0; i < AL; ++i) {
                const int64_t k = k0 + a_k + i;
                ra[i] = (m < a.M && k < kend) ? io<T>::to_f(X[m * a.ld_x + k]) : 0.0f;
            }
        }
        const int64_t n = n0 + b_row;
        if (MODE == BM_DENSE && a.vec) {
            float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const int64_t k = k0 + b_k;
            if (n < a.N && k < kend) load4<T>(static_cast<const T *>(a.w) + n * a.K + k, v);
#pragma unroll
            for (int e = 0; e < 4; ++e) rb[e] = v[e];
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int64_t k = k0 + b_k + i;
                rb[i] = (n < a.N && k < kend) ? load_w<T, MODE>(a, n, k) : 0.0f;
            }
        }
    };
    auto store_tile = [&](int buf) {
#pragma unroll
        for (int i = 0; i < AL; ++i) As[buf][a_k + i][a_row] = ra[i];
#pragma unroll
        for (int i = 0; i < 4; ++i) Bs[buf][b_k + i][b_row] = rb[i];
    };

    float acc[TM][4];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[i][jj] = 0.0f;

    const int64_t nk = kend > kbeg ? ceil_div(kend - kbeg, (int64_t)SG_BK) : 0;
    if (nk > 0) {
        load_tile(kbeg);
        store_tile(0);
    }
    __syncthreads();
    for (int64_t kt = 0; kt < nk; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < nk) load_tile(kbeg + (kt + 1) * SG_BK);
#pragma unroll
        for (int k = 0; k < SG_BK; ++k) {
            float av[TM];
#pragma unroll
            for (int h = 0; h < TM / 4; ++h) {
                const float4 a4 = *reinterpret_cast<const float4 *>(&As[buf][k][ty * TM + 4 * h]);
                av[4 * h] = a4.x; av[4 * h + 1] = a4.y; av[4 * h + 2] = a4.z; av[4 * h + 3] = a4.w;
            }
            const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][k][tx * 4]);
            const float bv[4] = {b0.x, b0.y, b0.z, b0.w};
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) acc[i][jj] = fmaf(av[i], bv[jj], acc[i][jj]);
        }
        if (kt + 1 < nk) store_tile(buf ^ 1);
        __syncthreads();
    }

    if (a.partial) {
        // split-K: raw partial sums; splitk_reduce_kernel finishes the outputs
        float *P = a.partial + (int64_t)blockIdx.z * a.M * a.N;
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const int64_t m = m0 + ty * TM + i;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int64_t n = n0 + tx * 4 + jj;
                if (m < a.M && n < a.N) P[m * a.N + n] = acc[i][jj];
            }
        }
        return;
    }

    T *Y = static_cast<T *>(a.y);
    const T *bias = static_cast<const T *>(a.bias);
    // optional terms, each behind one branch for the whole 8 x 4 block (a
    // per-element test of the softplus would spread its inlined body over
    // 32 instruction-cache lines)
    if (a.row_scale) {
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const int64_t m = m0 + ty * TM + i;
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
            for (int i = 0; i < TM; ++i) acc[i][jj] += bv;
        }
    }
    if (a.epi == MB2_EPI_SOFTPLUS) {
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) acc[i][jj] = softplus_f(io<T>::round(acc[i][jj]));
    }
    if (a.silu_from >= 0 && n0 + tx * 4 + 3 >= a.silu_from) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const bool act = n0 + tx * 4 + jj >= a.silu_from;
#pragma unroll
            for (int i = 0; i < TM; ++i)
                acc[i][jj] = act ? silu_f(io<T>::round(acc[i][jj])) : acc[i][jj];
        }
    }
    if (a.resid) {
        const T *R = static_cast<const T *>(a.resid);
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const int64_t m = m0 + ty * TM + i;
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
        for (int i = 0; i < TM; ++i) {
            const int64_t m = m0 + ty * TM + i;
            if (m < a.M) Y[m * a.ld_y + col] = io<T>::from_f(acc[i][jj]);
        }
    }
}

// Sum of the split-K partials in split order, then the epilogue terms in the
// same order as the single-pass kernel; one output element per thread.
template <typename T>
__global__ void splitk_reduce_kernel(const GemmArgs a, int splits) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.M * a.N) return;
    const int64_t m = i / a.N, n = i - m * a.N;
    const int64_t mn = a.M * a.N;
    // four loads in flight; fixed combination order (deterministic)
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    int z = 0;
    // unrolled so that up to 32 partial loads are in flight at once
#pragma unroll 8
    for (; z + 4 <= splits; z += 4) {
        a0 += a.partial[(z + 0) * mn + i];
        a1 += a.partial[(z + 1) * mn + i];
        a2 += a.partial[(z + 2) * mn + i];
        a3 += a.partial[(z + 3) * mn + i];
    }
    for (; z < splits; ++z) a0 += a.partial[z * mn + i];
    float v = (a0 + a1) + (a2 + a3);
    if (a.row_scale) v *= a.row_scale[m];
    if (a.bias) v += io<T>::to_f(static_cast<const T *>(a.bias)[n]);
    if (a.epi == MB2_EPI_SOFTPLUS) v = softplus_f(io<T>::round(v));
    if (a.silu_from >= 0 && n >= a.silu_from) v = silu_f(io<T>::round(v));
    if (a.resid) v += io<T>::to_f(static_cast<const T *>(a.resid)[m * a.ld_r + n]);
    const int64_t col = n + (n >= a.n1 ? a.off1 : 0) + (n >= a.n2 ? a.off2 : 0);
    static_cast<T *>(a.y)[m * a.ld_y + col] = io<T>::from_f(v);
}

static int g_simt_sms = 0;

template <typename T, int MODE>
static int launch_simt(GemmArgs a, const EpiExtra &ex, cudaStream_t st) {
    const bool small = a.M <= 64;
    const int bmt = small ? 64 : SG_BM;
    const int64_t tiles = ceil_div(a.N, (int64_t)SG_BN) * ceil_div(a.M, (int64_t)bmt);
    if (g_simt_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_simt_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_simt_sms <= 0) g_simt_sms = 148;
    }
    // split K when the output tiles leave the GPU idle and scratch is given:
    // aim at two CTAs per SM, at least two K tiles per split
    int64_t splits = 1;
    if (ex.scratch && a.M > 0 && a.N > 0) {
        const int64_t want = ceil_div((int64_t)2 * g_simt_sms, tiles);
        int64_t kmax = a.K / (2 * SG_BK);
        kmax = kmax < 16 ? kmax : 16;      // the reduction reads splits x M x N
        const int64_t cap = (int64_t)(ex.scratch_bytes / ((size_t)a.M * a.N * sizeof(float)));
        splits = want < kmax ? want : kmax;
        splits = splits < cap ? splits : cap;
        if (splits < 1) splits = 1;
    }
    a.kchunk = round_up(ceil_div(a.K, splits), (int64_t)SG_BK);
    splits = a.kchunk > 0 ? ceil_div(a.K, a.kchunk) : 1;
    if (splits < 1) splits = 1;
    a.partial = splits > 1 ? ex.scratch : nullptr;
    MB2_REQUIRE(splits <= 65535, MB2_ERR_SHAPE, "linear: too many K splits");
    dim3 grid((unsigned)ceil_div(a.N, (int64_t)SG_BN), (unsigned)ceil_div(a.M, (int64_t)bmt),
              (unsigned)splits);
    if (small)
        gemm_simt_kernel<T, MODE, 64><<<grid, SG_THREADS, 0, st>>>(a);
    else
        gemm_simt_kernel<T, MODE, SG_BM><<<grid, SG_THREADS, 0, st>>>(a);
    MB2_TRY(check_launch("gemm_simt_kernel"));
    if (splits > 1) {
        const int64_t n = a.M * a.N;
        splitk_reduce_kernel<T><<<(unsigned)ceil_div(n, (int64_t)256), 256, 0, st>>>(a, (int)splits);
        MB2_TRY(check_launch("splitk_reduce_kernel"));
    }
    return MB2_OK;
}

// Internal: dense or quantised CUDA-core GEMM with optional column remap.
int gemm_simt(int dtype, int scheme, const void *x, int64_t ld_x, const void *w,
              const float *scale, const void *bias, void *y, int64_t ld_y, int64_t M,
              int64_t N, int64_t K, int64_t n1, int64_t off1, int64_t n2, int64_t off2,
              int epi, cudaStream_t st, const EpiExtra &ex, int64_t group) {
    MB2_REQUIRE(M >= 0 && N >= 0 && K >= 0, MB2_ERR_SHAPE, "linear: negative size");
    MB2_REQUIRE(group >= 0, MB2_ERR_ARG, "linear: negative group size");
    MB2_REQUIRE(ceil_div(M, (int64_t)64) <= 65535, MB2_ERR_SHAPE, "linear: M too large");
    if (M == 0 || N == 0) return MB2_OK;
    MB2_REQUIRE(x && w && y, MB2_ERR_ARG, "linear: null pointer");
    MB2_REQUIRE(scheme == MB2_Q_NONE || scale, MB2_ERR_ARG, "linear: quantised weight needs scale");
    const size_t es = dtype == MB2_F32 ? 4 : 2;
    // 4-element groups of x rows (and of dense W rows) as single loads
    const int vec = K % 4 == 0 && ld_x % 4 == 0 && aligned(x, 4 * es) &&
                    (scheme != MB2_Q_NONE || aligned(w, 4 * es));
    GemmArgs a{x, ld_x, w, scale, group, group ? ceil_div(K, group) : 1, bias, y, ld_y, M, N, K,
               n1, n2, off1, off2, epi, {},
               ex.row_scale, ex.resid, ex.ld_r, nullptr, K, vec, ex.silu_from};
    nf4_lut(a.lut);
    const bool f32 = dtype == MB2_F32;
    switch (scheme) {
        case MB2_Q_NONE: return f32 ? launch_simt<float, BM_DENSE>(a, ex, st) : launch_simt<__nv_bfloat16, BM_DENSE>(a, ex, st);
        case MB2_Q_INT8: return f32 ? launch_simt<float, BM_INT8>(a, ex, st) : launch_simt<__nv_bfloat16, BM_INT8>(a, ex, st);
        case MB2_Q_INT4: return f32 ? launch_simt<float, BM_INT4>(a, ex, st) : launch_simt<__nv_bfloat16, BM_INT4>(a, ex, st);
        case MB2_Q_NF4: return f32 ? launch_simt<float, BM_NF4>(a, ex, st) : launch_simt<__nv_bfloat16, BM_NF4>(a, ex, st);
    }
    return fail(MB2_ERR_ARG, "linear: unknown scheme %d", scheme);
}

}  // namespace mb2
