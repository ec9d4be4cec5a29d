// Weight-only quantisation kernels, bit-exact with src/cpu_mamba/quant.py.
//
//   int8 (quant.py:60-65): scale = max(amax_row|w|, 1e-8) / 127,
//        q = clamp(round_half_even(w / scale), -127, 127)
//   int4 (quant.py:72-87): scale = max(amax, 1e-8) / 7, q in [-7, 7], stored
//        u = q + 7, byte = u[2j] << 4 | u[2j+1]; odd rows padded with q = 0
//   nf4  (quant.py:104-121): scale = max(amax, 1e-8), w_n = clamp(w/scale, -1, 1),
//        code = first argmin_k |w_n - LUT[k]|, packed like int4 (pad code 0)
//   dequant (quant.py:68-69, 90-101, 124-134): q.float() * scale / LUT[code] * scale
//
// Blockwise (grouped) variants -- the reference's roadmap item "blockwise NF4
// (group_size=64, as in QLoRA)", README.md:115, :201 -- apply the same
// formulas to each run of `group` consecutive input columns of a row, with
// one scale per (row, group): scale is (rows, ceil(cols / group)).  group = 0
// means the reference's one scale per row.
//
// This file is compiled WITHOUT fast-math: w / scale is an IEEE
// round-to-nearest division (__fdiv_rn) as in torch, rintf rounds half to
// even as torch.round does.
#include "internal.cuh"

namespace mb2 {

void nf4_lut(float *out16);  // gemm_simt.cu

struct Lut16 { float v[16]; };

constexpr int Q_THREADS = 256;

__device__ __forceinline__ float nan_max(float m, float a) {
    return (a > m || isnan(a)) ? a : m;
}

__device__ float block_amax(const float *w, int64_t cols) {
    __shared__ float red[Q_THREADS / 32];
    float m = 0.0f;
    for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) m = nan_max(m, fabsf(w[j]));
    for (int o = 16; o > 0; o >>= 1) m = nan_max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
        for (int o = 16; o > 0; o >>= 1) v = nan_max(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float r = red[0];
    __syncthreads();
    return r;
}

__device__ __forceinline__ float clamp_min_eps(float v) {
    const float eps = 1e-8f;  // torch casts the Python scalar 1e-8 to float32
    return v < eps ? eps : v;
}

__device__ __forceinline__ int q_sym(float w, float s, float qmax) {
    float v = rintf(__fdiv_rn(w, s));
    v = fminf(fmaxf(v, -qmax), qmax);
    return (int)v;
}

__device__ __forceinline__ int nf4_code(float w, float s, const Lut16 &lut) {
    float wn = __fdiv_rn(w, s);
    wn = fminf(fmaxf(wn, -1.0f), 1.0f);
    int best = 0;
    float bd = fabsf(wn - lut.v[0]);
#pragma unroll
    for (int i = 1; i < 16; ++i) {
        const float dd = fabsf(wn - lut.v[i]);
        if (dd < bd) { bd = dd; best = i; }
    }
    return best;
}

template <int SCHEME>
__global__ void __launch_bounds__(Q_THREADS)
quantize_kernel(const float *__restrict__ w, int64_t cols, void *__restrict__ out,
                float *__restrict__ scale, const Lut16 lut) {
    const int64_t r = blockIdx.x;
    const float *wr = w + r * cols;
    const float amax = clamp_min_eps(block_amax(wr, cols));
    const float s = SCHEME == MB2_Q_INT8 ? __fdiv_rn(amax, 127.0f)
                  : SCHEME == MB2_Q_INT4 ? __fdiv_rn(amax, 7.0f) : amax;
    if (threadIdx.x == 0) scale[r] = s;
    if (SCHEME == MB2_Q_INT8) {
        int8_t *q = static_cast<int8_t *>(out) + r * cols;
        for (int64_t j = threadIdx.x; j < cols; j += blockDim.x)
            q[j] = (int8_t)q_sym(wr[j], s, 127.0f);
    } else {
        const int64_t pcols = (cols + 1) >> 1;
        uint8_t *q = static_cast<uint8_t *>(out) + r * pcols;
        for (int64_t p = threadIdx.x; p < pcols; p += blockDim.x) {
            int nib[2];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int64_t j = 2 * p + k;
                if (SCHEME == MB2_Q_INT4)
                    nib[k] = (j < cols ? q_sym(wr[j], s, 7.0f) : 0) + 7;
                else
                    nib[k] = j < cols ? nf4_code(wr[j], s, lut) : 0;
            }
            q[p] = (uint8_t)((nib[0] << 4) | nib[1]);
        }
    }
}

// One warp per (row, group): the group's amax (NaN-propagating like torch's
// amax), its scale, then its codes; 4-bit groups are even so pairs never
// straddle two groups.
template <int SCHEME>
__global__ void __launch_bounds__(Q_THREADS)
quantize_grouped_kernel(const float *__restrict__ w, int64_t cols, int64_t group,
                        void *__restrict__ out, float *__restrict__ scale, const Lut16 lut) {
    const int64_t r = blockIdx.x;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t ng = (cols + group - 1) / group;
    const float *wr = w + r * cols;
    for (int64_t g = wid; g < ng; g += Q_THREADS / 32) {
        const int64_t j0 = g * group;
        const int64_t j1 = (j0 + group < cols) ? j0 + group : cols;
        float m = 0.0f;
        for (int64_t j = j0 + lane; j < j1; j += 32) m = nan_max(m, fabsf(wr[j]));
        for (int o = 16; o > 0; o >>= 1) m = nan_max(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float amax = clamp_min_eps(m);
        const float sg = SCHEME == MB2_Q_INT8 ? __fdiv_rn(amax, 127.0f)
                       : SCHEME == MB2_Q_INT4 ? __fdiv_rn(amax, 7.0f) : amax;
        if (lane == 0) scale[r * ng + g] = sg;
        if (SCHEME == MB2_Q_INT8) {
            int8_t *q = static_cast<int8_t *>(out) + r * cols;
            for (int64_t j = j0 + lane; j < j1; j += 32) q[j] = (int8_t)q_sym(wr[j], sg, 127.0f);
        } else {
            uint8_t *q = static_cast<uint8_t *>(out) + r * ((cols + 1) >> 1);
            for (int64_t pp = (j0 >> 1) + lane; 2 * pp < j1; pp += 32) {
                int nib[2];
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const int64_t j = 2 * pp + k;
                    if (SCHEME == MB2_Q_INT4)
                        nib[k] = (j < cols ? q_sym(wr[j], sg, 7.0f) : 0) + 7;
                    else
                        nib[k] = j < cols ? nf4_code(wr[j], sg, lut) : 0;
                }
                q[pp] = (uint8_t)((nib[0] << 4) | nib[1]);
            }
        }
    }
}

template <int SCHEME>
__global__ void dequantize_kernel(const void *__restrict__ wq, const float *__restrict__ scale,
                                  int64_t rows, int64_t in_dim, int64_t group,
                                  float *__restrict__ out, const Lut16 lut) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * in_dim) return;
    const int64_t r = i / in_dim, j = i - r * in_dim;
    const float s = group ? scale[r * ((in_dim + group - 1) / group) + j / group] : scale[r];
    if (SCHEME == MB2_Q_INT8) {
        out[i] = (float)static_cast<const int8_t *>(wq)[i] * s;
    } else {
        const int64_t pcols = (in_dim + 1) >> 1;
        const uint8_t byte = static_cast<const uint8_t *>(wq)[r * pcols + (j >> 1)];
        const int nib = (j & 1) ? (byte & 0x0F) : (byte >> 4);
        out[i] = SCHEME == MB2_Q_INT4 ? (float)(nib - 7) * s : lut.v[nib] * s;
    }
}

// The tensor-core GEMM's weight operand from quantised codes: deq(W) formed
// exactly as dequantize_kernel (q.float() * scale, quant.py:68-69, :90-101,
// :124-134) and as QuantizedLinear.forward casts it (.to(x.dtype), :188-190),
// then, for fp32, split into TF32 planes out[0:n] = hi, out[n:2n] = lo (as
// mb2_split_tf32), for bf16 rounded to bf16.
template <int SCHEME, bool BF16>
__global__ void dequant_operand_kernel(const void *__restrict__ wq,
                                       const float *__restrict__ scale, int64_t rows,
                                       int64_t in_dim, int64_t group, void *__restrict__ out,
                                       const Lut16 lut) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t n = rows * in_dim;
    if (i >= n) return;
    const int64_t r = i / in_dim, j = i - r * in_dim;
    const float s = group ? scale[r * ((in_dim + group - 1) / group) + j / group] : scale[r];
    float w;
    if (SCHEME == MB2_Q_INT8) {
        w = (float)static_cast<const int8_t *>(wq)[i] * s;
    } else {
        const int64_t pcols = (in_dim + 1) >> 1;
        const uint8_t byte = static_cast<const uint8_t *>(wq)[r * pcols + (j >> 1)];
        const int nib = (j & 1) ? (byte & 0x0F) : (byte >> 4);
        w = SCHEME == MB2_Q_INT4 ? (float)(nib - 7) * s : lut.v[nib] * s;
    }
    if (BF16) {
        static_cast<__nv_bfloat16 *>(out)[i] = __float2bfloat16_rn(w);
    } else {
        const float hi = tf32_round(w);
        static_cast<float *>(out)[i] = hi;
        static_cast<float *>(out)[n + i] = tf32_round(w - hi);
    }
}

// The integer codes themselves as fp16 (exact), the operand of the F16X3
// kernel's CODES form, which applies the scale in its epilogue.
template <int SCHEME>
__global__ void codes_f16_kernel(const void *__restrict__ wq, int64_t rows, int64_t in_dim,
                                 __half *__restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * in_dim) return;
    int q;
    if (SCHEME == MB2_Q_INT8) {
        q = static_cast<const int8_t *>(wq)[i];
    } else {
        const int64_t r = i / in_dim, j = i - r * in_dim;
        const int64_t pcols = (in_dim + 1) >> 1;
        const uint8_t byte = static_cast<const uint8_t *>(wq)[r * pcols + (j >> 1)];
        q = ((j & 1) ? (byte & 0x0F) : (byte >> 4)) - 7;
    }
    out[i] = __int2half_rn(q);
}

int codes_f16(int scheme, const void *wq, int64_t rows, int64_t in_dim, void *out, cudaStream_t st) {
    const int64_t n = rows * in_dim;
    if (n == 0) return MB2_OK;
    const unsigned grid = (unsigned)ceil_div(n, (int64_t)256);
    __half *o = static_cast<__half *>(out);
    if (scheme == MB2_Q_INT8) codes_f16_kernel<MB2_Q_INT8><<<grid, 256, 0, st>>>(wq, rows, in_dim, o);
    else if (scheme == MB2_Q_INT4) codes_f16_kernel<MB2_Q_INT4><<<grid, 256, 0, st>>>(wq, rows, in_dim, o);
    else return fail(MB2_ERR_ARG, "codes_f16: scheme %d has no integer codes", scheme);
    return check_launch("codes_f16_kernel");
}

size_t dequant_operand_bytes(int dtype, int64_t rows, int64_t in_dim) {
    if (dtype == MB2_BF16) return (size_t)rows * in_dim * 2;
    // TF32 planes (8 B per weight), or the F16X3 split (4096 + 4 B per weight,
    // rounded to 256) plus the fp32 weight it is made from (4 B per weight)
    const size_t split = (split_f16_bytes(rows, in_dim) + 255) & ~size_t(255);
    const size_t f16x3 = split + (size_t)rows * in_dim * 4;
    const size_t tf32 = (size_t)rows * in_dim * 8;
    return f16x3 > tf32 ? f16x3 : tf32;
}

int dequant_operand(int dtype, int scheme, const void *wq, const float *scale, int64_t rows,
                    int64_t in_dim, int64_t group, void *out, cudaStream_t st) {
    const int64_t n = rows * in_dim;
    if (n == 0) return MB2_OK;
    Lut16 lut;
    nf4_lut(lut.v);
    const unsigned grid = (unsigned)ceil_div(n, (int64_t)256);
    const bool bf = dtype == MB2_BF16;
#define MB2_DQ(S)                                                                              \
    (bf ? (dequant_operand_kernel<S, true><<<grid, 256, 0, st>>>(wq, scale, rows, in_dim, group, out, lut), 0) \
        : (dequant_operand_kernel<S, false><<<grid, 256, 0, st>>>(wq, scale, rows, in_dim, group, out, lut), 0))
    switch (scheme) {
        case MB2_Q_INT8: MB2_DQ(MB2_Q_INT8); break;
        case MB2_Q_INT4: MB2_DQ(MB2_Q_INT4); break;
        case MB2_Q_NF4: MB2_DQ(MB2_Q_NF4); break;
        default: return fail(MB2_ERR_ARG, "unknown scheme %d", scheme);
    }
#undef MB2_DQ
    return check_launch("dequant_operand_kernel");
}

// group 0: one scale per row (quant.py); else one per (row, group of columns)
static int quantize_any(int scheme, const float *w, int64_t rows, int64_t cols, int64_t group,
                        void *weight_q, float *scale, cudaStream_t st) {
    MB2_REQUIRE(scheme == MB2_Q_INT8 || scheme == MB2_Q_INT4 || scheme == MB2_Q_NF4,
                MB2_ERR_ARG, "unknown scheme %d", scheme);
    MB2_REQUIRE(rows >= 0 && cols >= 0 && rows <= 0x7fffffff, MB2_ERR_SHAPE, "quantize: bad shape");
    MB2_REQUIRE(group >= 0 && (group == 0 || scheme == MB2_Q_INT8 || group % 2 == 0),
                MB2_ERR_ARG, "quantize: group size must be >= 0 (even for 4-bit schemes)");
    if (rows == 0) return MB2_OK;
    MB2_REQUIRE(w && weight_q && scale, MB2_ERR_ARG, "quantize: null pointer");
    Lut16 lut;
    nf4_lut(lut.v);
    const unsigned grid = (unsigned)rows;
    if (group == 0) {
        switch (scheme) {
            case MB2_Q_INT8: quantize_kernel<MB2_Q_INT8><<<grid, Q_THREADS, 0, st>>>(w, cols, weight_q, scale, lut); break;
            case MB2_Q_INT4: quantize_kernel<MB2_Q_INT4><<<grid, Q_THREADS, 0, st>>>(w, cols, weight_q, scale, lut); break;
            default: quantize_kernel<MB2_Q_NF4><<<grid, Q_THREADS, 0, st>>>(w, cols, weight_q, scale, lut); break;
        }
    } else {
        switch (scheme) {
            case MB2_Q_INT8: quantize_grouped_kernel<MB2_Q_INT8><<<grid, Q_THREADS, 0, st>>>(w, cols, group, weight_q, scale, lut); break;
            case MB2_Q_INT4: quantize_grouped_kernel<MB2_Q_INT4><<<grid, Q_THREADS, 0, st>>>(w, cols, group, weight_q, scale, lut); break;
            default: quantize_grouped_kernel<MB2_Q_NF4><<<grid, Q_THREADS, 0, st>>>(w, cols, group, weight_q, scale, lut); break;
        }
    }
    return check_launch("quantize_kernel");
}

static int dequantize_any(int scheme, const void *weight_q, const float *scale, int64_t rows,
                          int64_t in_dim, int64_t group, float *w_out, cudaStream_t st) {
    MB2_REQUIRE(scheme == MB2_Q_INT8 || scheme == MB2_Q_INT4 || scheme == MB2_Q_NF4,
                MB2_ERR_ARG, "unknown scheme %d", scheme);
    MB2_REQUIRE(rows >= 0 && in_dim >= 0 && group >= 0, MB2_ERR_SHAPE, "dequantize: bad shape");
    const int64_t n = rows * in_dim;
    if (n == 0) return MB2_OK;
    MB2_REQUIRE(weight_q && scale && w_out, MB2_ERR_ARG, "dequantize: null pointer");
    Lut16 lut;
    nf4_lut(lut.v);
    const unsigned grid = (unsigned)ceil_div(n, 256);
    switch (scheme) {
        case MB2_Q_INT8: dequantize_kernel<MB2_Q_INT8><<<grid, 256, 0, st>>>(weight_q, scale, rows, in_dim, group, w_out, lut); break;
        case MB2_Q_INT4: dequantize_kernel<MB2_Q_INT4><<<grid, 256, 0, st>>>(weight_q, scale, rows, in_dim, group, w_out, lut); break;
        default: dequantize_kernel<MB2_Q_NF4><<<grid, 256, 0, st>>>(weight_q, scale, rows, in_dim, group, w_out, lut); break;
    }
    return check_launch("dequantize_kernel");
}

int dequantize_f32(int scheme, const void *wq, const float *scale, int64_t rows, int64_t in_dim,
                   int64_t group, float *out, cudaStream_t st) {
    return dequantize_any(scheme, wq, scale, rows, in_dim, group, out, st);
}

}  // namespace mb2

using namespace mb2;

extern "C" int mb2_quantize(int scheme, const float *w, int64_t rows, int64_t cols,
                            void *weight_q, float *scale, mb2_stream_t stream) {
    return quantize_any(scheme, w, rows, cols, 0, weight_q, scale, (cudaStream_t)stream);
}

extern "C" int mb2_quantize_grouped(int scheme, const float *w, int64_t rows, int64_t cols,
                                    int64_t group_size, void *weight_q, float *scale,
                                    mb2_stream_t stream) {
    return quantize_any(scheme, w, rows, cols, group_size, weight_q, scale, (cudaStream_t)stream);
}

extern "C" int mb2_dequantize(int scheme, const void *weight_q, const float *scale,
                              int64_t rows, int64_t in_dim, float *w_out, mb2_stream_t stream) {
    return dequantize_any(scheme, weight_q, scale, rows, in_dim, 0, w_out, (cudaStream_t)stream);
}

extern "C" int mb2_dequantize_grouped(int scheme, const void *weight_q, const float *scale,
                                      int64_t rows, int64_t in_dim, int64_t group_size,
                                      float *w_out, mb2_stream_t stream) {
    return dequantize_any(scheme, weight_q, scale, rows, in_dim, group_size, w_out,
                          (cudaStream_t)stream);
}
