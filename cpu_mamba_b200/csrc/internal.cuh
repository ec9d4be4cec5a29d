// Internal launchers shared between the library's translation units (not part
// of the C ABI).
#pragma once

#include "common.cuh"

namespace mb2 {

// Optional terms of a projection's epilogue, applied to each output element
// y[m, n] in this order:
//   v  = acc * row_scale[m]          (pre-norm folded into the projection:
//                                     row_scale = 1 / rms(x_m), the norm weight
//                                     folded into W's columns)
//   v += bias[n];  softplus if asked
//   v = silu(v) for columns n >= silu_from, on v rounded to the output dtype
//                                    (in_proj's z half: the gate SiLU(z) of
//                                     _mamba.py:264 applied where z is produced)
//   v += resid[m * ld_r + n]          (residual add; resid may alias y)
struct EpiExtra {
    const float *row_scale = nullptr;
    const void *resid = nullptr;
    int64_t ld_r = 0;
    int64_t silu_from = -1;            // < 0: no SiLU columns
    // not an epilogue term: device scratch for the projection -- the
    // dequantised operand of a quantised weight on the tensor-core path, or
    // the CUDA-core GEMM's split-K partial sums (few-row GEMMs) -- or null
    float *scratch = nullptr;
    size_t scratch_bytes = 0;
    // not an epilogue term: partial maxima of |x| that the F16X3 fp32 GEMM
    // scales x by.  amax_n > 0: amax_parts already holds amax_n of them (the
    // kernel that wrote x computed them); amax_n == 0: amax_parts is scratch of
    // AMAX_PARTS (512) floats that the GEMM fills with a pass over x first;
    // null: no F16X3.
    float *amax_parts = nullptr;
    int amax_n = 0;
    // not an epilogue term: when non-null and the fp32 tensor-core split-K
    // path runs (few rows), the raw partial sums are left in `scratch` as
    // (splits, M, N) fp32 without any epilogue term and *defer_splits = the
    // split count, for the consumer kernel to reduce; 0 when the output was
    // written as usual
    int *defer_splits = nullptr;
    // not an epilogue term: launch the few-row tensor-core GEMM and its
    // reduction as links of a programmatic chain (common.cuh): PDL_CHAIN
    // waits for the previous kernel before any load; PDL_WEIGHTS_EARLY also
    // loads its first weight tiles before that wait (the previous kernel
    // writes no weights)
    int pdl = 0;
    // not an epilogue term: scratch where an fp32 projection with many
    // 256-wide column tiles may place x split into fp16 halves once (M·K·4
    // bytes + M·4 for the row scales) instead of splitting it in every
    // column tile; null: split inside the GEMM
    void *xsplit = nullptr;
    size_t xsplit_bytes = 0;
};
enum { PDL_NONE = 0, PDL_CHAIN = 1, PDL_WEIGHTS_EARLY = 2 };

// Slots of the fused maxima: a kernel writing a GEMM's input takes
// atomicMax(slot[block % AMAX_SLOTS], |value| bits) over the slots, zeroed
// beforehand; the GEMM reduces the slots.
constexpr int AMAX_SLOTS = 64;
__device__ __forceinline__ void amax_publish(unsigned *slots, float m) {
    // m >= 0 (or NaN): its bits order like the value; one atomic per block
    // (call with every thread of the block, after its last value)
    __shared__ float red[32];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[wid] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        const int nw = (int)((blockDim.x * blockDim.y + 31) >> 5);
        for (int w = 1; w < nw; ++w) m = fmaxf(m, red[w]);
        const unsigned b = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
        atomicMax(slots + b % AMAX_SLOTS, __float_as_uint(m));
    }
}

int gemm_simt(int dtype, int scheme, const void *x, int64_t ld_x, const void *w,
              const float *scale, const void *bias, void *y, int64_t ld_y, int64_t M,
              int64_t N, int64_t K, int64_t n1, int64_t off1, int64_t n2, int64_t off2,
              int epi, cudaStream_t st, const EpiExtra &ex = EpiExtra{}, int64_t group = 0);
int gemm_tc(int dtype, const void *x, int64_t ld_x, const void *w, const float *w_split,
            const void *bias, void *y, int64_t ld_y, int64_t M, int64_t N, int64_t K,
            int64_t n1, int64_t off1, int64_t n2, int64_t off2, int epi, cudaStream_t st,
            bool *used, const EpiExtra &ex = EpiExtra{});
// fp32 GEMM on the fp16 tensor cores (scaled fp16 split of x and of W, W from
// mb2_split_f16); *used reports whether it ran (aligned operands, K % 8 == 0).
int gemm_f16x3(const float *x, int64_t ld_x, const void *w16, const void *bias, float *y,
               int64_t ld_y, int64_t M, int64_t N, int64_t K, int64_t n1, int64_t off1,
               int64_t n2, int64_t off2, int epi, cudaStream_t st, bool *used,
               const EpiExtra &ex, float *parts, int pair = -1);
// The same kernel on a quantised weight's codes (int8 / int4, one scale per
// row) given as exact fp16 (codes_f16), the scale applied in the epilogue.
int gemm_f16x3_codes(const float *x, int64_t ld_x, const void *codes16, const float *col_scale,
                     const void *bias, float *y, int64_t ld_y, int64_t M, int64_t N, int64_t K,
                     int64_t n1, int64_t off1, int64_t n2, int64_t off2, int epi, cudaStream_t st,
                     bool *used, const EpiExtra &ex, float *parts);
// int8 / int4 codes (rows, in_dim) as fp16 integers q (int4: nibble - 7, the
// packing of quant.py:90-101), exact
int codes_f16(int scheme, const void *wq, int64_t rows, int64_t in_dim, void *out, cudaStream_t st);
size_t split_f16_bytes(int64_t rows, int64_t cols);
// W (rows, cols) fp32 -> mb2_split_f16's layout at out (256-byte aligned)
int split_f16(const float *w, int64_t rows, int64_t cols, void *out, cudaStream_t st);
// quant.py's dequantised weight (bit-exact), fp32 (rows, in_dim)
int dequantize_f32(int scheme, const void *wq, const float *scale, int64_t rows, int64_t in_dim,
                   int64_t group, float *out, cudaStream_t st);
int conv1d_silu(int dtype, const void *x_in, int64_t ld_in, const void *w, const void *bias,
                void *xc, int64_t ld_out, void *tail, int64_t batch, int64_t seqlen,
                int64_t d_inner, int64_t d_conv, cudaStream_t st, unsigned *amax = nullptr);
// `act` (SCAN_* bits): which inputs their producer already activated -- dt =
// softplus(dt_proj output), SiLU(z) in in_proj's epilogue; the scan applies
// the others itself.  SCAN_DT_SCRATCH: the dt rows are the caller's scratch,
// which a T-segmented scan may overwrite with softplus(dt) in its first pass.
enum { SCAN_DT_ACT = 1, SCAN_Z_ACT = 2, SCAN_DT_SCRATCH = 4 };
int scan_fused(int dtype, const void *xc, int64_t ld_xc, const void *dl, int64_t ld_dl,
               const void *bm, int64_t ld_b, const void *cm, int64_t ld_c, const void *z,
               int64_t ld_z, const void *w_dt, const void *b_dt, const void *A_log,
               const void *D, const float *h0, float *h_last, void *y, int64_t ld_y,
               int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state, int64_t dt_rank,
               cudaStream_t stream, unsigned *amax = nullptr, int act = 0);

int scan_gated(int dtype, const void *xc, int64_t ld_xc, const void *dt, int64_t ld_dt,
               const void *bm, int64_t ld_b, const void *cm, int64_t ld_c, const void *z,
               int64_t ld_z, const void *A_log, const void *D, const float *h0, float *h_last,
               void *y, int64_t ld_y, int64_t batch, int64_t seqlen, int64_t d_inner,
               int64_t d_state, cudaStream_t stream, float *seg_ws = nullptr,
               size_t seg_bytes = 0, unsigned *amax = nullptr, int act = 0);
// Long sequences over few (batch, channel) chains: the number of T segments
// scan_gated runs in parallel (1 = none) and the scratch it needs for them.
int scan_segments(int64_t batch, int64_t d_inner, int64_t seqlen, int64_t d_state);
size_t scan_segment_bytes(int64_t batch, int64_t d_inner, int64_t seqlen, int64_t d_state);

// The decode step's dt_proj (fp32 dot products of dt_low with W_dt's rows),
// softplus and state update in one kernel; y may alias xc.
int scan_step_dt(int dtype, const void *xc, int64_t ld_x, const void *dt_low, int64_t ld_dl,
                 const void *w_dt, const void *b_dt, const void *bm, const void *cm,
                 int64_t ld_bc, const void *z, int64_t ld_z, const void *A_log, const void *D,
                 float *h, void *y, int64_t ld_y, int64_t batch, int64_t d_inner, int64_t d_state,
                 int64_t dt_rank, cudaStream_t st, bool pdl = false);

// Quantised weights as the tensor-core GEMM's operand (bit-exact dequantised
// values; fp32: TF32 hi / lo planes, bf16: rounded) and its size in bytes --
// for fp32 also large enough for the F16X3 operand: mb2_split_f16's layout of
// the dequantised weight followed by that fp32 weight itself.
size_t dequant_operand_bytes(int dtype, int64_t rows, int64_t in_dim);
int dequant_operand(int dtype, int scheme, const void *wq, const float *scale, int64_t rows,
                    int64_t in_dim, int64_t group, void *out, cudaStream_t st);

// Dense or quantised linear y = x W^T (+ bias, + extras): the tensor-core
// kernel where it applies, the CUDA-core kernel otherwise.  n1/off1/n2/off2
// remap output columns (column n is written at n + off1 [n >= n1] + off2 [n >= n2]).
int linear_any(int dtype, const mb2_linear_w &L, const void *x, int64_t ld_x, void *y,
               int64_t ld_y, int64_t M, int64_t N, int64_t K, int epi, cudaStream_t st,
               int64_t n1 = -1, int64_t off1 = 0, int64_t n2 = -1, int64_t off2 = 0,
               const EpiExtra &ex = EpiExtra{});

}  // namespace mb2
