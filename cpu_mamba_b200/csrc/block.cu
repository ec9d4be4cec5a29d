// Block-level composition of the Mamba S6 forward (src/cpu_mamba/_mamba.py:204-265),
// the forward_with_final_state state outputs (:165-202) and the single-token
// step (:103-163), plus the linear-layer entry points.
//
// Forward pipeline (6 launches, caller-provided workspace, no allocation):
//   1. in_proj            x (N, dm)          -> xz (N, 2di): x | SiLU(z), the
//                                               gate's SiLU applied in the epilogue
//   2. conv1d + SiLU      xz[:, :di]         -> xc (N, di)   [+ conv tail]
//   3. x_proj             xc                 -> xdbl (N, ldx): dt_low | B | C, each
//                                               segment on an 8-element boundary
//   4. dt_proj            xdbl[:, :R]        -> over xz[:, :di] (the conv's
//                                               input, dead by now)
//   5. gated scan         xc, dt_proj out, xdbl, SiLU(z) -> y (N, di)
//      [+ h_last] (softplus + exp(dt A) + recurrence + D skip + cast + gate;
//       y overwrites xc in place).  Where the dt GEMM cannot run on the tensor
//       cores, steps 4 and 5 are one fused scan that also computes dt.
//   6. out_proj           y                  -> out (N, dm)
#include "internal.cuh"

namespace mb2 {

int linear_any(int dtype, const mb2_linear_w &L, const void *x, int64_t ld_x, void *y,
               int64_t ld_y, int64_t M, int64_t N, int64_t K, int epi, cudaStream_t st,
               int64_t n1, int64_t off1, int64_t n2, int64_t off2, const EpiExtra &ex) {
    if (n1 < 0) n1 = N;
    if (n2 < 0) n2 = N;
    if (L.scheme != MB2_Q_NONE) {
        // many rows: dequantise the weight into scratch as the tensor-core
        // operand (bit-exact values, as QuantizedLinear.forward forms them on
        // every call) and run the tensor-core GEMM; else the CUDA-core GEMM
        // dequantises tile by tile in its loader
        if (M >= 256 && ex.scratch &&
            ex.scratch_bytes >= dequant_operand_bytes(dtype, N, K)) {
            if (dtype == MB2_F32 && ex.amax_parts && K % 8 == 0 && L.group_size == 0 &&
                (L.scheme == MB2_Q_INT8 || L.scheme == MB2_Q_INT4)) {
                // int8 / int4 with one scale per row: the integer codes, exact
                // in fp16, are the tensor-core operand and the scale is applied
                // per output column in the epilogue (two MMAs per K step)
                MB2_TRY(codes_f16(L.scheme, L.weight_q, N, K, ex.scratch, st));
                bool used = false;
                MB2_TRY(gemm_f16x3_codes(static_cast<const float *>(x), ld_x, ex.scratch, L.scale,
                                         L.bias, static_cast<float *>(y), ld_y, M, N, K, n1, off1,
                                         n2, off2, epi, st, &used, ex, ex.amax_parts));
                if (used) return MB2_OK;
            }
            if (dtype == MB2_F32 && ex.amax_parts && K % 8 == 0) {
                // fp32: the dequantised weight (quant.py's values, bit-exact),
                // its scaled fp16 split, then the F16X3 GEMM
                const size_t split = (split_f16_bytes(N, K) + 255) & ~size_t(255);
                float *deq = reinterpret_cast<float *>(reinterpret_cast<char *>(ex.scratch) + split);
                MB2_TRY(dequantize_f32(L.scheme, L.weight_q, L.scale, N, K, L.group_size, deq, st));
                MB2_TRY(split_f16(deq, N, K, ex.scratch, st));
                bool used = false;
                MB2_TRY(gemm_f16x3(static_cast<const float *>(x), ld_x, ex.scratch, L.bias,
                                   static_cast<float *>(y), ld_y, M, N, K, n1, off1, n2, off2, epi,
                                   st, &used, ex, ex.amax_parts));
                if (used) return MB2_OK;
            }
            MB2_TRY(dequant_operand(dtype, L.scheme, L.weight_q, L.scale, N, K, L.group_size,
                                    ex.scratch, st));
            const bool bf = dtype == MB2_BF16;
            bool used = false;
            EpiExtra ex2 = ex;
            ex2.scratch = nullptr;
            ex2.scratch_bytes = 0;
            MB2_TRY(gemm_tc(dtype, x, ld_x, bf ? (const void *)ex.scratch : nullptr,
                            bf ? nullptr : ex.scratch, L.bias, y, ld_y, M, N, K, n1, off1, n2,
                            off2, epi, st, &used, ex2));
            if (used) return MB2_OK;
        }
        return gemm_simt(dtype, L.scheme, x, ld_x, L.weight_q, L.scale, L.bias, y, ld_y, M, N, K,
                         n1, off1, n2, off2, epi, st, ex, L.group_size);
    }
    MB2_REQUIRE(L.weight, MB2_ERR_ARG, "linear: null weight");
    bool used = false;
    if (dtype == MB2_F32 && L.weight_f16 && M >= 256 && ex.amax_parts) {
        MB2_TRY(gemm_f16x3(static_cast<const float *>(x), ld_x, L.weight_f16, L.bias,
                           static_cast<float *>(y), ld_y, M, N, K, n1, off1, n2, off2, epi, st,
                           &used, ex, ex.amax_parts));
        if (used) return MB2_OK;
    }
    MB2_TRY(gemm_tc(dtype, x, ld_x, L.weight, L.weight_split, L.bias, y, ld_y, M, N, K, n1, off1,
                    n2, off2, epi, st, &used, ex));
    if (used) return MB2_OK;
    return gemm_simt(dtype, MB2_Q_NONE, x, ld_x, L.weight, nullptr, L.bias, y, ld_y, M, N, K,
                     n1, off1, n2, off2, epi, st, ex);
}

struct Layout {
    int64_t N, di, dm, S, R, K;
    int64_t RB, RC, ldx;   // x_dbl segment offsets and row length
    size_t es;
    size_t off_xz, off_xc, off_xdbl, total;   // y reuses the xc buffer
    size_t off_part, part_bytes;              // step: split-K partial sums
    size_t off_seg, seg_bytes;                // forward: scan T-segment state
    size_t off_deq, deq_bytes;                // forward: a quantised weight, dequantised
    size_t off_aux;                           // forward: partial maxima for F16X3 (2 KB)
};

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Workspace of a forward over `rows` tokens, or (step) of a decode step: the
// step's projections have few rows and split K, so it adds room for four
// splits' partial sums of its widest projection.
static Layout make_layout(const mb2_block *b, int64_t rows, bool step = false,
                          int64_t batch = 0, int64_t seqlen = 0) {
    Layout l{};
    l.N = rows;
    l.di = b->d_inner; l.dm = b->d_model; l.S = b->d_state; l.R = b->dt_rank; l.K = b->d_conv;
    l.RB = round_up(l.R, 8);
    l.RC = l.RB + round_up(l.S, 8);
    l.ldx = l.RC + round_up(l.S, 8);
    l.es = dtype_size(b->dtype);
    size_t off = 0;
    l.off_xz = off; off = align256(off + (size_t)rows * 2 * l.di * l.es);
    l.off_xc = off; off = align256(off + (size_t)rows * l.di * l.es);
    l.off_xdbl = off; off = align256(off + (size_t)rows * l.ldx * l.es);
    l.off_part = off;
    l.part_bytes = 0;
    if (step) {
        int64_t wide = 2 * l.di > l.dm ? 2 * l.di : l.dm;
        wide = wide > l.R + 2 * l.S ? wide : l.R + 2 * l.S;
        l.part_bytes = (size_t)rows * wide * sizeof(float) * 4;
        off = align256(off + l.part_bytes);
    }
    l.off_seg = off;
    l.seg_bytes = step ? 0 : scan_segment_bytes(batch, l.di, seqlen, l.S);
    off = align256(off + l.seg_bytes);
    l.off_deq = off;
    l.deq_bytes = 0;
    if (!step && rows >= 256) {   // the tensor-core path of quantised projections
        auto need = [&](const mb2_linear_w &w, int64_t n, int64_t k) {
            const size_t v = w.scheme != MB2_Q_NONE ? dequant_operand_bytes(b->dtype, n, k) : 0;
            l.deq_bytes = v > l.deq_bytes ? v : l.deq_bytes;
        };
        need(b->in_proj, 2 * l.di, l.dm);
        need(b->x_proj, l.R + 2 * l.S, l.di);
        need(b->out_proj, l.dm, l.di);
        off = align256(off + l.deq_bytes);
    }
    // forward: x's partial maxima for in_proj (512 floats), then the fused
    // maxima slots of x_proj's input (written by the conv) and out_proj's
    // input (written by the scan)
    l.off_aux = off;
    if (!step) off = align256(off + (512 + 2 * AMAX_SLOTS) * sizeof(float));
    l.total = off;
    return l;
}

// dt_proj's weight as the fused scan reads it: dense rows in the activation
// dtype (a quantised dt_proj supplies its dequantised weight in .weight).
static const void *dt_weight(const mb2_block &b) { return b.dt_proj.weight; }

static int check_block(const mb2_block *b) {
    MB2_REQUIRE(b, MB2_ERR_ARG, "block: null descriptor");
    MB2_REQUIRE(b->dtype == MB2_F32 || b->dtype == MB2_BF16, MB2_ERR_ARG, "block: bad dtype");
    MB2_REQUIRE(b->d_model > 0 && b->d_inner > 0 && b->d_state >= 1 && b->d_state <= 256 &&
                    b->dt_rank >= 1 && b->d_conv >= 2,
                MB2_ERR_SHAPE, "block: bad dimensions");
    MB2_REQUIRE(b->conv_w && b->A_log, MB2_ERR_ARG, "block: missing conv1d.weight / A_log");
    MB2_REQUIRE(b->dt_proj.weight, MB2_ERR_ARG,
                "block: dt_proj.weight (dense; the dequantised weight when quantised) is required");
    if (b->dtype == MB2_BF16)
        MB2_REQUIRE(b->d_inner % 2 == 0 && b->dt_rank % 2 == 0 && b->d_state % 2 == 0,
                    MB2_ERR_UNSUPPORTED, "block(bf16): d_inner, dt_rank, d_state must be even");
    return MB2_OK;
}

// ------------------------------------------------------------- step conv ---
// forward_step's conv (_mamba.py:128-139): window = [conv_state | x], output
// silu(bias + sum_k w[k] * window[k]), conv_state <- window[1:] (in place).
template <typename T, int K>
__global__ void conv_step_kernel(const T *__restrict__ xz, int64_t ld_xz, const T *__restrict__ w,
                                 const T *__restrict__ bias, T *__restrict__ conv_state,
                                 T *__restrict__ xc, int64_t batch, int64_t d_inner) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch * d_inner) return;
    const int64_t b = i / d_inner, d = i - b * d_inner;
    T *cs = conv_state + i * (K - 1);
    float win[K];
#pragma unroll
    for (int k = 0; k < K - 1; ++k) win[k] = io<T>::to_f(cs[k]);
    win[K - 1] = io<T>::to_f(xz[b * ld_xz + d]);
    float acc = bias ? io<T>::to_f(bias[d]) : 0.0f;
#pragma unroll
    for (int k = 0; k < K; ++k) acc = fmaf(io<T>::to_f(w[d * K + k]), win[k], acc);
    xc[b * d_inner + d] = io<T>::from_f(silu_f(io<T>::round(acc)));
#pragma unroll
    for (int k = 0; k < K - 1; ++k) cs[k] = io<T>::from_f(win[k + 1]);
}

// The same conv step taking in_proj's raw split-K partial sums (fp32, (ks, B,
// 2 d_inner)) instead of its output: each thread sums its x element's splits
// in the fixed order of the split-K reduction (four interleaved partial sums),
// applies in_proj's row scale and bias, runs the conv ring, and also sums its
// z element (the other half of in_proj's row) into xz for the scan.  Saves the
// reduction's launch.
template <int K>
__global__ void conv_step_reduce_kernel(const float *__restrict__ P, int ks,
                                        const float *__restrict__ row_scale,
                                        const float *__restrict__ in_bias, float *__restrict__ xz,
                                        int64_t ld_xz, const float *__restrict__ w,
                                        const float *__restrict__ bias,
                                        float *__restrict__ conv_state, float *__restrict__ xc,
                                        int64_t batch, int64_t d_inner) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch * d_inner) return;
    const int64_t b = i / d_inner, d = i - b * d_inner;
    const int64_t N = 2 * d_inner, mn = batch * N;
    auto total = [&](int64_t n) {
        const float *q = P + b * N + n;
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        int z = 0;
        // unrolled so that up to 32 partial loads are in flight at once
#pragma unroll 8
        for (; z + 4 <= ks; z += 4) {
            a0 += q[(z + 0) * mn];
            a1 += q[(z + 1) * mn];
            a2 += q[(z + 2) * mn];
            a3 += q[(z + 3) * mn];
        }
        for (; z < ks; ++z) a0 += q[z * mn];
        float v = (a0 + a1) + (a2 + a3);
        if (row_scale) v *= row_scale[b];
        if (in_bias) v += in_bias[n];
        return v;
    };
    xz[b * ld_xz + d_inner + d] = total(d_inner + d);      // z, for the scan
    float *cs = conv_state + i * (K - 1);
    float win[K];
#pragma unroll
    for (int k = 0; k < K - 1; ++k) win[k] = cs[k];
    win[K - 1] = total(d);
    float acc = bias ? bias[d] : 0.0f;
#pragma unroll
    for (int k = 0; k < K; ++k) acc = fmaf(w[d * K + k], win[k], acc);
    xc[b * d_inner + d] = silu_f(acc);
#pragma unroll
    for (int k = 0; k < K - 1; ++k) cs[k] = win[k + 1];
}

template <typename T>
static int launch_conv_step(int K, const void *xz, int64_t ld_xz, const void *w, const void *bias,
                            void *conv_state, void *xc, int64_t batch, int64_t di,
                            cudaStream_t st) {
    const unsigned grid = (unsigned)ceil_div(batch * di, 256);
    switch (K) {
#define MB2_CS(KK)                                                                          \
    case KK:                                                                                \
        conv_step_kernel<T, KK><<<grid, 256, 0, st>>>(                                      \
            (const T *)xz, ld_xz, (const T *)w, (const T *)bias, (T *)conv_state, (T *)xc, \
            batch, di);                                                                     \
        return check_launch("conv_step_kernel");
        MB2_CS(2) MB2_CS(3) MB2_CS(4) MB2_CS(5) MB2_CS(6) MB2_CS(7) MB2_CS(8)
#undef MB2_CS
    }
    return fail(MB2_ERR_UNSUPPORTED, "step: d_conv %d not in [2, 8]", K);
}

}  // namespace mb2

using namespace mb2;

extern "C" int mb2_linear(int dtype, const void *x, int64_t ld_x, const void *w,
                          const float *w_split, const void *bias, void *y, int64_t ld_y,
                          int64_t M, int64_t N, int64_t K, int epilogue, mb2_stream_t stream) {
    MB2_REQUIRE(dtype == MB2_F32 || dtype == MB2_BF16, MB2_ERR_ARG, "linear: bad dtype");
    MB2_REQUIRE(epilogue == MB2_EPI_NONE || epilogue == MB2_EPI_SOFTPLUS, MB2_ERR_ARG,
                "linear: bad epilogue");
    MB2_REQUIRE(ld_x >= K && ld_y >= N, MB2_ERR_SHAPE, "linear: leading dimension too small");
    mb2_linear_w L{w, w_split, nullptr, nullptr, bias, MB2_Q_NONE, 0, nullptr};
    return linear_any(dtype, L, x, ld_x, y, ld_y, M, N, K, epilogue, (cudaStream_t)stream);
}

static int qlinear_any(int scheme, int64_t group, int dtype, const void *x, int64_t ld_x,
                       const void *weight_q, const float *scale, const void *bias, void *y,
                       int64_t ld_y, int64_t M, int64_t N, int64_t K, int epilogue,
                       mb2_stream_t stream) {
    MB2_REQUIRE(dtype == MB2_F32 || dtype == MB2_BF16, MB2_ERR_ARG, "qlinear: bad dtype");
    MB2_REQUIRE(scheme == MB2_Q_INT8 || scheme == MB2_Q_INT4 || scheme == MB2_Q_NF4, MB2_ERR_ARG,
                "unknown scheme %d", scheme);
    MB2_REQUIRE(ld_x >= K && ld_y >= N, MB2_ERR_SHAPE, "qlinear: leading dimension too small");
    MB2_REQUIRE(epilogue == MB2_EPI_NONE || epilogue == MB2_EPI_SOFTPLUS, MB2_ERR_ARG,
                "qlinear: bad epilogue");
    return gemm_simt(dtype, scheme, x, ld_x, weight_q, scale, bias, y, ld_y, M, N, K, N, 0, N, 0,
                     epilogue, (cudaStream_t)stream, EpiExtra{}, group);
}

extern "C" int mb2_qlinear(int scheme, int dtype, const void *x, int64_t ld_x,
                           const void *weight_q, const float *scale, const void *bias, void *y,
                           int64_t ld_y, int64_t M, int64_t N, int64_t K, int epilogue,
                           mb2_stream_t stream) {
    return qlinear_any(scheme, 0, dtype, x, ld_x, weight_q, scale, bias, y, ld_y, M, N, K,
                       epilogue, stream);
}

extern "C" int mb2_qlinear_grouped(int scheme, int64_t group_size, int dtype, const void *x,
                                   int64_t ld_x, const void *weight_q, const float *scale,
                                   const void *bias, void *y, int64_t ld_y, int64_t M, int64_t N,
                                   int64_t K, int epilogue, mb2_stream_t stream) {
    return qlinear_any(scheme, group_size, dtype, x, ld_x, weight_q, scale, bias, y, ld_y, M, N,
                       K, epilogue, stream);
}

// One block forward over N = batch * seqlen rows runs as a head (in_proj ->
// conv -> x_proj, leaving x_dbl in the workspace) and a tail (dt_proj -> scan
// -> gate -> out_proj).  A channel-sharded block all-reduces x_dbl between
// the two (x_proj contracts over the sharded channels).
// row_scale (N floats) scales in_proj's output rows (a pre-norm folded into
// in_proj); resid (N, d_model) is added to out_proj's output (may alias out).
static EpiExtra scratch_extra(const Layout &l, char *ws) {
    EpiExtra e;    // scratch for dequantised weights (quantised projections)
    e.scratch = l.deq_bytes ? reinterpret_cast<float *>(ws + l.off_deq) : nullptr;
    e.scratch_bytes = l.deq_bytes;
    e.amax_parts = reinterpret_cast<float *>(ws + l.off_aux);
    return e;
}

// The fused maxima slots of x_proj's (which = 0) or out_proj's (1) input,
// zeroed for the kernel that writes that input, or null where no F16X3 GEMM
// can read them (bf16, or too few rows).
static unsigned *fused_amax(const Layout &l, char *ws, int dtype, int which, cudaStream_t st) {
    if (dtype != MB2_F32 || l.N < 256) return nullptr;
    unsigned *slots = reinterpret_cast<unsigned *>(ws + l.off_aux) + 512 + which * AMAX_SLOTS;
    cudaMemsetAsync(slots, 0, AMAX_SLOTS * sizeof(unsigned), st);
    return slots;
}

// Stage boundaries for mb2_block_forward_profile: ev[0] before in_proj,
// ev[i] after stage i (in_proj, conv, x_proj, dt_proj, scan, out_proj), or
// null (no events).
static void mark(cudaEvent_t *ev, int i, cudaStream_t st) {
    if (ev) cudaEventRecord(ev[i], st);
}

// Where the gate's SiLU(z) is applied: in in_proj's epilogue (fp32) or in the
// scan's output pass (bf16).
static bool z_in_proj(const mb2_block &b) { return b.dtype == MB2_F32; }

static int pipeline_head(const mb2_block &b, const Layout &l, const void *x, int64_t batch,
                         int64_t seqlen, void *conv_tail, char *ws, cudaStream_t st,
                         const float *row_scale, cudaEvent_t *ev = nullptr) {
    void *xz = ws + l.off_xz, *xc = ws + l.off_xc, *xdbl = ws + l.off_xdbl;
    const int64_t N = l.N, di = l.di, S = l.S, R = l.R;
    EpiExtra in_ex = scratch_extra(l, ws), mid_ex = scratch_extra(l, ws);
    in_ex.row_scale = row_scale;
    // fp32: the z half leaves in_proj as SiLU(z), the gate (:264); the bf16
    // GEMM's four epilogue warps are the slower place for it (the scan gates)
    in_ex.silu_from = z_in_proj(b) ? di : -1;
    in_ex.xsplit = ws + l.off_xc;   // free until the conv writes xc
    in_ex.xsplit_bytes = l.off_xdbl - l.off_xc;
    mark(ev, 0, st);
    if (N > 0)
        MB2_TRY(linear_any(b.dtype, b.in_proj, x, l.dm, xz, 2 * di, N, 2 * di, l.dm, MB2_EPI_NONE,
                           st, -1, 0, -1, 0, in_ex));
    mark(ev, 1, st);
    unsigned *xc_max = fused_amax(l, ws, b.dtype, 0, st);
    MB2_TRY(check_launch("block: maxima clear"));
    MB2_TRY(conv1d_silu(b.dtype, xz, 2 * di, b.conv_w, b.conv_b, xc, di, conv_tail, batch, seqlen,
                        di, b.d_conv, st, xc_max));
    mark(ev, 2, st);
    if (xc_max) {
        mid_ex.amax_parts = reinterpret_cast<float *>(xc_max);
        mid_ex.amax_n = AMAX_SLOTS;
    }
    if (N > 0)
        MB2_TRY(linear_any(b.dtype, b.x_proj, xc, di, xdbl, l.ldx, N, R + 2 * S, di, MB2_EPI_NONE,
                           st, R, l.RB - R, R + S, l.RC - l.RB - S, mid_ex));
    mark(ev, 3, st);
    return MB2_OK;
}

static int pipeline_tail(const mb2_block &b, const Layout &l, void *out, int64_t batch,
                         int64_t seqlen, float *h_last, char *ws, cudaStream_t st,
                         const void *resid, cudaEvent_t *ev = nullptr) {
    void *xz = ws + l.off_xz, *xc = ws + l.off_xc, *xdbl = ws + l.off_xdbl;
    const int64_t N = l.N, di = l.di, S = l.S, R = l.R;
    const size_t es = l.es;
    EpiExtra out_ex = scratch_extra(l, ws);
    out_ex.resid = resid;
    out_ex.ld_r = l.dm;
    // dt_proj (_mamba.py:219) on the tensor cores, bias in the epilogue,
    // written over the x half of xz (dead once the conv has run); the gated
    // scan applies the softplus (:220) once per token and channel (in T
    // segments, the first pass writes it back over these rows for the
    // second).  (Softplus in the GEMM epilogue measured slower: dt_proj's
    // K = R GEMM is bound by its epilogue already.)  A quantised dt_proj
    // passes its dequantised weight in .weight (as the fused scan needs it).
    // Where that GEMM does not apply (an unsplit fp32 weight, fewer than 256
    // rows) the fused scan computes dt itself from W_dt's rows in registers.
    // Either scan reads z as SiLU(z), which in_proj's epilogue formed.
    bool dt_done = false;
    if (N >= 256 && b.dtype == MB2_F32 && b.dt_proj.weight_f16) {
        EpiExtra dt_ex;                  // x's maxima by a pass over dt_low (N x R)
        dt_ex.amax_parts = reinterpret_cast<float *>(ws + l.off_aux);
        MB2_TRY(gemm_f16x3(static_cast<const float *>(xdbl), l.ldx, b.dt_proj.weight_f16,
                           b.dt_proj.bias, static_cast<float *>(xz), 2 * di, N, di, R, di, 0, di,
                           0, MB2_EPI_NONE, st, &dt_done, dt_ex, dt_ex.amax_parts));
    }
    if (N > 0 && !dt_done)
        MB2_TRY(gemm_tc(b.dtype, xdbl, l.ldx, b.dt_proj.weight, b.dt_proj.weight_split,
                        b.dt_proj.bias, xz, 2 * di, N, di, R, di, 0, di, 0, MB2_EPI_NONE, st,
                        &dt_done));
    mark(ev, 4, st);
    unsigned *y_max = fused_amax(l, ws, b.dtype, 1, st);
    MB2_TRY(check_launch("block: maxima clear"));
    if (dt_done)
        MB2_TRY(scan_gated(b.dtype, xc, di, xz, 2 * di, (char *)xdbl + l.RB * es, l.ldx,
                           (char *)xdbl + l.RC * es, l.ldx, (char *)xz + di * es, 2 * di, b.A_log,
                           b.D, nullptr, h_last, xc, di, batch, seqlen, di, S, st,
                           reinterpret_cast<float *>(ws + l.off_seg), l.seg_bytes, y_max,
                           (z_in_proj(b) ? SCAN_Z_ACT : 0) | SCAN_DT_SCRATCH));
    else
        MB2_TRY(scan_fused(b.dtype, xc, di, xdbl, l.ldx, (char *)xdbl + l.RB * es, l.ldx,
                           (char *)xdbl + l.RC * es, l.ldx, (char *)xz + di * es, 2 * di,
                           dt_weight(b), b.dt_proj.bias, b.A_log, b.D, nullptr, h_last, xc, di,
                           batch, seqlen, di, S, R, st, y_max, z_in_proj(b) ? SCAN_Z_ACT : 0));
    mark(ev, 5, st);
    if (y_max) {
        out_ex.amax_parts = reinterpret_cast<float *>(y_max);
        out_ex.amax_n = AMAX_SLOTS;
    }
    if (N > 0)
        MB2_TRY(linear_any(b.dtype, b.out_proj, xc, di, out, l.dm, N, l.dm, di, MB2_EPI_NONE, st,
                           -1, 0, -1, 0, out_ex));
    mark(ev, 6, st);
    return MB2_OK;
}

static int block_pipeline(const mb2_block &b, const Layout &l, const void *x, void *out,
                          int64_t batch, int64_t seqlen, float *h_last, void *conv_tail,
                          char *ws, cudaStream_t st, const float *row_scale,
                          const void *resid) {
    MB2_TRY(pipeline_head(b, l, x, batch, seqlen, conv_tail, ws, st, row_scale));
    return pipeline_tail(b, l, out, batch, seqlen, h_last, ws, st, resid);
}

extern "C" size_t mb2_block_workspace_bytes(const mb2_block *blk, int64_t batch, int64_t seqlen) {
    if (!blk || batch < 0 || seqlen < 0) return 0;
    return make_layout(blk, batch * seqlen, false, batch, seqlen).total;
}

extern "C" int mb2_block_forward(const mb2_block *blk, const void *x, void *out, int64_t batch,
                                 int64_t seqlen, float *h_last, void *conv_tail, void *workspace,
                                 size_t workspace_bytes, mb2_stream_t stream) {
    MB2_TRY(check_block(blk));
    MB2_REQUIRE(batch >= 0 && seqlen >= 0, MB2_ERR_SHAPE, "block: negative size");
    const mb2_block &b = *blk;
    cudaStream_t st = (cudaStream_t)stream;
    const Layout l = make_layout(blk, batch * seqlen, false, batch, seqlen);
    MB2_REQUIRE(workspace_bytes >= l.total, MB2_ERR_WORKSPACE,
                "block: workspace %zu < required %zu", workspace_bytes, l.total);
    if (batch == 0) return MB2_OK;
    if (l.N > 0) MB2_REQUIRE(x && out && workspace, MB2_ERR_ARG, "block: null pointer");
    return block_pipeline(b, l, x, out, batch, seqlen, h_last, conv_tail,
                          static_cast<char *>(workspace), st, nullptr, nullptr);
}

extern "C" int mb2_block_forward_profile(const mb2_block *blk, const void *x, void *out,
                                         int64_t batch, int64_t seqlen, void *workspace,
                                         size_t workspace_bytes, float *stage_ms,
                                         mb2_stream_t stream) {
    MB2_TRY(check_block(blk));
    MB2_REQUIRE(batch > 0 && seqlen > 0, MB2_ERR_SHAPE, "block profile: empty batch");
    MB2_REQUIRE(x && out && workspace && stage_ms, MB2_ERR_ARG, "block profile: null pointer");
    cudaStream_t st = (cudaStream_t)stream;
    const Layout l = make_layout(blk, batch * seqlen, false, batch, seqlen);
    MB2_REQUIRE(workspace_bytes >= l.total, MB2_ERR_WORKSPACE,
                "block profile: workspace %zu < required %zu", workspace_bytes, l.total);
    cudaEvent_t ev[7] = {};
    int rc = MB2_OK;
    for (int i = 0; i < 7 && rc == MB2_OK; ++i)
        if (cudaEventCreate(&ev[i]) != cudaSuccess)
            rc = fail(MB2_ERR_CUDA, "block profile: cudaEventCreate failed");
    char *ws = static_cast<char *>(workspace);
    if (rc == MB2_OK) rc = pipeline_head(*blk, l, x, batch, seqlen, nullptr, ws, st, nullptr, ev);
    if (rc == MB2_OK) rc = pipeline_tail(*blk, l, out, batch, seqlen, nullptr, ws, st, nullptr, ev);
    if (rc == MB2_OK && cudaEventSynchronize(ev[6]) != cudaSuccess)
        rc = fail(MB2_ERR_CUDA, "block profile: %s", cudaGetErrorString(cudaGetLastError()));
    for (int i = 0; i < 6 && rc == MB2_OK; ++i)
        if (cudaEventElapsedTime(&stage_ms[i], ev[i], ev[i + 1]) != cudaSuccess)
            rc = fail(MB2_ERR_CUDA, "block profile: cudaEventElapsedTime failed");
    for (int i = 0; i < 7; ++i)
        if (ev[i]) cudaEventDestroy(ev[i]);
    return rc;
}

extern "C" size_t mb2_step_workspace_bytes(const mb2_block *blk, int64_t batch) {
    if (!blk || batch < 0) return 0;
    return make_layout(blk, batch, true).total;
}

// A decode step as a head (in_proj -> ring conv -> x_proj) and a tail
// (dt_proj -> one scan step -> gate -> out_proj), split like the forward.
// The fp32 step's kernels are launched as a programmatic chain (common.cuh):
// each starts while the one before it finishes, the x_proj and out_proj
// GEMMs loading their first weight tiles and the state update staging W_dt
// and prefetching h before their inputs are ready.
static int step_head(const mb2_block &b, const Layout &l, const void *x, void *conv_state,
                     int64_t batch, char *ws, cudaStream_t st, const float *row_scale = nullptr) {
    void *xz = ws + l.off_xz, *xc = ws + l.off_xc, *xdbl = ws + l.off_xdbl;
    const int64_t di = l.di, S = l.S, R = l.R;
    EpiExtra sk;                    // split-K scratch for the few-row projections
    sk.scratch = reinterpret_cast<float *>(ws + l.off_part);
    sk.scratch_bytes = l.part_bytes;
    sk.pdl = PDL_WEIGHTS_EARLY;     // x_proj follows the conv step, which writes no weights
    EpiExtra in_ex = sk;
    in_ex.row_scale = row_scale;
    in_ex.pdl = PDL_CHAIN;          // the kernel before in_proj is not known
    int splits = 0;                 // fp32 split-K in_proj: its partials, reduced by the conv
    if (b.dtype == MB2_F32) in_ex.defer_splits = &splits;
    MB2_TRY(linear_any(b.dtype, b.in_proj, x, l.dm, xz, 2 * di, batch, 2 * di, l.dm, MB2_EPI_NONE,
                       st, -1, 0, -1, 0, in_ex));
    if (splits > 0) {
        const unsigned grid = (unsigned)ceil_div(batch * di, (int64_t)256);
        cudaError_t le = cudaSuccess;
        switch (b.d_conv) {
#define MB2_CSR(KK)                                                                            \
    case KK:                                                                                   \
        le = launch_kernel(true, conv_step_reduce_kernel<KK>, dim3(grid), dim3(256), 0, st,   \
                           sk.scratch, splits, row_scale,                                     \
                           static_cast<const float *>(b.in_proj.bias), static_cast<float *>(xz), \
                           2 * di, static_cast<const float *>(b.conv_w),                      \
                           static_cast<const float *>(b.conv_b),                              \
                           static_cast<float *>(conv_state), static_cast<float *>(xc), batch, \
                           di);                                                               \
        break;
            MB2_CSR(2) MB2_CSR(3) MB2_CSR(4) MB2_CSR(5) MB2_CSR(6) MB2_CSR(7) MB2_CSR(8)
#undef MB2_CSR
            default: return fail(MB2_ERR_UNSUPPORTED, "step: d_conv %lld not in [2, 8]",
                                 (long long)b.d_conv);
        }
        if (le != cudaSuccess)
            return fail(MB2_ERR_CUDA, "conv_step_reduce_kernel launch: %s", cudaGetErrorString(le));
        MB2_TRY(check_launch("conv_step_reduce_kernel"));
    } else if (b.dtype == MB2_F32)
        MB2_TRY(launch_conv_step<float>((int)b.d_conv, xz, 2 * di, b.conv_w, b.conv_b, conv_state,
                                        xc, batch, di, st));
    else
        MB2_TRY(launch_conv_step<__nv_bfloat16>((int)b.d_conv, xz, 2 * di, b.conv_w, b.conv_b,
                                                conv_state, xc, batch, di, st));
    return linear_any(b.dtype, b.x_proj, xc, di, xdbl, l.ldx, batch, R + 2 * S, di, MB2_EPI_NONE,
                      st, R, l.RB - R, R + S, l.RC - l.RB - S, sk);
}

static int step_tail(const mb2_block &b, const Layout &l, void *out, float *h, int64_t batch,
                     char *ws, cudaStream_t st, const void *resid = nullptr) {
    void *xz = ws + l.off_xz, *xc = ws + l.off_xc, *xdbl = ws + l.off_xdbl;
    const int64_t di = l.di, S = l.S, R = l.R;
    const size_t es = l.es;
    EpiExtra sk;
    sk.scratch = reinterpret_cast<float *>(ws + l.off_part);
    sk.scratch_bytes = l.part_bytes;
    sk.pdl = PDL_WEIGHTS_EARLY;     // out_proj follows the state update, which writes no weights
    // one timestep: dt_proj (W_dt's dense rows; a quantised dt_proj supplies
    // its dequantised weight) + softplus, exp(dt A), h updated in place,
    // y = C.h + D x, gate -- one kernel
    MB2_TRY(scan_step_dt(b.dtype, xc, di, xdbl, l.ldx, b.dt_proj.weight, b.dt_proj.bias,
                         (char *)xdbl + l.RB * es, (char *)xdbl + l.RC * es, l.ldx,
                         (char *)xz + di * es, 2 * di, b.A_log, b.D, h, xc, di, batch, di, S, R,
                         st, true));
    EpiExtra out_ex = sk;
    out_ex.resid = resid;
    out_ex.ld_r = l.dm;
    return linear_any(b.dtype, b.out_proj, xc, di, out, l.dm, batch, l.dm, di, MB2_EPI_NONE, st,
                      -1, 0, -1, 0, out_ex);
}

extern "C" int mb2_block_step(const mb2_block *blk, const void *x, void *out, float *h,
                              void *conv_state, int64_t batch, void *workspace,
                              size_t workspace_bytes, mb2_stream_t stream) {
    MB2_TRY(check_block(blk));
    MB2_REQUIRE(batch >= 0, MB2_ERR_SHAPE, "step: negative batch");
    const mb2_block &b = *blk;
    cudaStream_t st = (cudaStream_t)stream;
    const Layout l = make_layout(blk, batch, true);
    MB2_REQUIRE(workspace_bytes >= l.total, MB2_ERR_WORKSPACE,
                "step: workspace %zu < required %zu", workspace_bytes, l.total);
    if (batch == 0) return MB2_OK;
    MB2_REQUIRE(x && out && h && conv_state && workspace, MB2_ERR_ARG, "step: null pointer");
    char *ws = static_cast<char *>(workspace);
    MB2_TRY(step_head(b, l, x, conv_state, batch, ws, st));
    return step_tail(b, l, out, h, batch, ws, st);
}

// ------------------------------------------------------- channel shards ---
// A block whose d_inner channels are split over ranks: every rank runs the
// head on its channels, the caller all-reduces x_dbl (x_proj contracts over
// d_inner), every rank runs the tail, and the caller all-reduces out
// (out_proj contracts over d_inner too).  x_dbl's pad columns are zeroed in
// the head so the reduced buffer holds no uninitialised values.

extern "C" int mb2_block_shard_xdbl(const mb2_block *blk, int64_t rows, int step, size_t *offset,
                                    int64_t *ld) {
    MB2_TRY(check_block(blk));
    MB2_REQUIRE(rows >= 0 && offset && ld, MB2_ERR_ARG, "shard_xdbl: bad argument");
    const Layout l = make_layout(blk, rows, step != 0);
    *offset = l.off_xdbl;
    *ld = l.ldx;
    return MB2_OK;
}

extern "C" int mb2_block_forward_shard(const mb2_block *blk, int phase, const void *x, void *out,
                                       int64_t batch, int64_t seqlen, float *h_last,
                                       void *conv_tail, void *workspace, size_t workspace_bytes,
                                       mb2_stream_t stream) {
    MB2_TRY(check_block(blk));
    MB2_REQUIRE(phase == 1 || phase == 2, MB2_ERR_ARG, "forward_shard: phase must be 1 or 2");
    MB2_REQUIRE(batch >= 0 && seqlen >= 0, MB2_ERR_SHAPE, "forward_shard: negative size");
    cudaStream_t st = (cudaStream_t)stream;
    const Layout l = make_layout(blk, batch * seqlen, false, batch, seqlen);
    MB2_REQUIRE(workspace_bytes >= l.total, MB2_ERR_WORKSPACE,
                "forward_shard: workspace %zu < required %zu", workspace_bytes, l.total);
    if (l.N == 0) return MB2_OK;
    MB2_REQUIRE(workspace && (phase == 1 ? x != nullptr : out != nullptr), MB2_ERR_ARG,
                "forward_shard: null pointer");
    char *ws = static_cast<char *>(workspace);
    if (phase == 2) return pipeline_tail(*blk, l, out, batch, seqlen, h_last, ws, st, nullptr);
    cudaMemsetAsync(ws + l.off_xdbl, 0, (size_t)l.N * l.ldx * l.es, st);
    MB2_TRY(check_launch("forward_shard: x_dbl clear"));
    return pipeline_head(*blk, l, x, batch, seqlen, conv_tail, ws, st, nullptr);
}

extern "C" int mb2_block_step_shard(const mb2_block *blk, int phase, const void *x, void *out,
                                    float *h, void *conv_state, int64_t batch, void *workspace,
                                    size_t workspace_bytes, mb2_stream_t stream) {
    MB2_TRY(check_block(blk));
    MB2_REQUIRE(phase == 1 || phase == 2, MB2_ERR_ARG, "step_shard: phase must be 1 or 2");
    MB2_REQUIRE(batch >= 0, MB2_ERR_SHAPE, "step_shard: negative batch");
    cudaStream_t st = (cudaStream_t)stream;
    const Layout l = make_layout(blk, batch, true);
    MB2_REQUIRE(workspace_bytes >= l.total, MB2_ERR_WORKSPACE,
                "step_shard: workspace %zu < required %zu", workspace_bytes, l.total);
    if (batch == 0) return MB2_OK;
    MB2_REQUIRE(workspace && (phase == 1 ? (x && conv_state) : (out && h)), MB2_ERR_ARG,
                "step_shard: null pointer");
    char *ws = static_cast<char *>(workspace);
    if (phase == 2) return step_tail(*blk, l, out, h, batch, ws, st);
    cudaMemsetAsync(ws + l.off_xdbl, 0, (size_t)batch * l.ldx * l.es, st);
    MB2_TRY(check_launch("step_shard: x_dbl clear"));
    return step_head(*blk, l, x, conv_state, batch, ws, st);
}

// ------------------------------------------------------------------ stack ---
// A residual stack of pre-norm blocks, x <- x + block(RMSNorm(x)) per layer
// (the Mamba-130M-style composition; the reference has no stack: its block is
// composed with torch.nn.RMSNorm around CPUMamba.forward).  RMSNorm(x) =
// x / rms(x) * g with rms(x) = sqrt(mean(x^2) + eps).  Its weight g is folded
// into in_proj's columns once (mb2_fold_norm), and 1 / rms(x_m) is one float
// per token that in_proj's epilogue multiplies in, so the normalised
// activations are never written.  out_proj's epilogue adds the residual and
// writes the stream in place.  Per layer: row-rms pass + the block's five
// launches.

// one warp per row: r[m] = 1 / sqrt(mean(x[m, :]^2) + eps), fp32 accumulation
template <typename T>
__global__ void rms_scale_kernel(const T *__restrict__ x, int64_t ld, int64_t rows, int64_t D,
                                 float eps, float *__restrict__ r, int vec) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const T *xr = x + row * ld;
    float ss = 0.0f;
    if (vec) {
        constexpr int V = 16 / (int)sizeof(T);
        for (int64_t c = (int64_t)lane * V; c < D; c += 32 * V) {
            const uint4 u = *reinterpret_cast<const uint4 *>(xr + c);
            const T *e = reinterpret_cast<const T *>(&u);
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const float f = io<T>::to_f(e[k]);
                ss = fmaf(f, f, ss);
            }
        }
    } else {
        for (int64_t c = lane; c < D; c += 32) {
            const float f = io<T>::to_f(xr[c]);
            ss = fmaf(f, f, ss);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) r[row] = 1.0f / sqrtf(ss / (float)D + eps);
}

static int rms_scale(int dtype, const void *x, int64_t rows, int64_t D, float eps, float *r,
                     cudaStream_t st) {
    if (rows == 0) return MB2_OK;
    const size_t es = dtype_size(dtype);
    const int vec = aligned(x, 16) && (D * (int64_t)es) % 16 == 0;
    const unsigned grid = (unsigned)ceil_div(rows, (int64_t)8);
    if (dtype == MB2_F32)
        rms_scale_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float *>(x), D, rows, D,
                                                      eps, r, vec);
    else
        rms_scale_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
            static_cast<const __nv_bfloat16 *>(x), D, rows, D, eps, r, vec);
    return check_launch("rms_scale_kernel");
}

template <typename T>
__global__ void fold_norm_kernel(const T *__restrict__ w, const T *__restrict__ g,
                                 T *__restrict__ out, int64_t rows, int64_t cols) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * cols) return;
    out[i] = io<T>::from_f(io<T>::to_f(w[i]) * io<T>::to_f(g[i % cols]));
}

extern "C" int mb2_fold_norm(int dtype, const void *w, const void *norm_weight, void *out,
                             int64_t rows, int64_t cols, mb2_stream_t stream) {
    MB2_REQUIRE(dtype == MB2_F32 || dtype == MB2_BF16, MB2_ERR_ARG, "fold_norm: bad dtype");
    MB2_REQUIRE(rows >= 0 && cols >= 0, MB2_ERR_SHAPE, "fold_norm: negative size");
    if (rows * cols == 0) return MB2_OK;
    MB2_REQUIRE(w && norm_weight && out, MB2_ERR_ARG, "fold_norm: null pointer");
    const unsigned grid = (unsigned)ceil_div(rows * cols, (int64_t)256);
    cudaStream_t st = (cudaStream_t)stream;
    if (dtype == MB2_F32)
        fold_norm_kernel<float><<<grid, 256, 0, st>>>(
            static_cast<const float *>(w), static_cast<const float *>(norm_weight),
            static_cast<float *>(out), rows, cols);
    else
        fold_norm_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
            static_cast<const __nv_bfloat16 *>(w), static_cast<const __nv_bfloat16 *>(norm_weight),
            static_cast<__nv_bfloat16 *>(out), rows, cols);
    return check_launch("fold_norm_kernel");
}

static size_t stack_bytes(const mb2_block *layers, int64_t n_layers, int64_t batch,
                          int64_t seqlen, size_t *off_r) {
    size_t ws = 0;
    const int64_t rows = batch * seqlen;
    for (int64_t i = 0; i < n_layers; ++i) {
        const size_t t = make_layout(&layers[i], rows, false, batch, seqlen).total;
        ws = t > ws ? t : ws;
    }
    *off_r = ws;
    return ws + align256((size_t)rows * sizeof(float));
}

extern "C" size_t mb2_stack_workspace_bytes(const mb2_block *layers, int64_t n_layers,
                                            int64_t batch, int64_t seqlen) {
    if (!layers || n_layers <= 0 || batch < 0 || seqlen < 0) return 0;
    size_t off_r;
    return stack_bytes(layers, n_layers, batch, seqlen, &off_r);
}

static int check_stack(const mb2_block *layers, int64_t n_layers, float eps) {
    MB2_REQUIRE(layers && n_layers > 0, MB2_ERR_ARG, "stack: no layers");
    MB2_REQUIRE(eps >= 0.0f, MB2_ERR_ARG, "stack: negative eps");
    for (int64_t i = 0; i < n_layers; ++i) {
        MB2_TRY(check_block(&layers[i]));
        MB2_REQUIRE(layers[i].d_model == layers[0].d_model && layers[i].dtype == layers[0].dtype,
                    MB2_ERR_SHAPE, "stack: layer %lld differs in d_model or dtype",
                    (long long)i);
    }
    return MB2_OK;
}

extern "C" int mb2_stack_forward(const mb2_block *layers, int64_t n_layers, float eps, void *x,
                                 int64_t batch, int64_t seqlen, void *workspace,
                                 size_t workspace_bytes, mb2_stream_t stream) {
    return mb2_stack_forward_state(layers, n_layers, eps, x, batch, seqlen, nullptr, nullptr,
                                   workspace, workspace_bytes, stream);
}

extern "C" int mb2_stack_forward_state(const mb2_block *layers, int64_t n_layers, float eps,
                                       void *x, int64_t batch, int64_t seqlen,
                                       float *const *h_last, void *const *conv_tail,
                                       void *workspace, size_t workspace_bytes,
                                       mb2_stream_t stream) {
    MB2_TRY(check_stack(layers, n_layers, eps));
    MB2_REQUIRE(batch >= 0 && seqlen >= 0, MB2_ERR_SHAPE, "stack: negative size");
    const int64_t N = batch * seqlen;
    size_t off_r;
    const size_t need = stack_bytes(layers, n_layers, batch, seqlen, &off_r);
    MB2_REQUIRE(workspace_bytes >= need, MB2_ERR_WORKSPACE,
                "stack: workspace %zu < required %zu", workspace_bytes, need);
    if (N == 0) return MB2_OK;
    MB2_REQUIRE(x && workspace, MB2_ERR_ARG, "stack: null pointer");
    cudaStream_t st = (cudaStream_t)stream;
    char *ws = static_cast<char *>(workspace);
    float *r = reinterpret_cast<float *>(ws + off_r);
    for (int64_t i = 0; i < n_layers; ++i) {
        const mb2_block &b = layers[i];
        const Layout l = make_layout(&b, N, false, batch, seqlen);
        MB2_TRY(rms_scale(b.dtype, x, N, b.d_model, eps, r, st));
        MB2_TRY(block_pipeline(b, l, x, x, batch, seqlen, h_last ? h_last[i] : nullptr,
                               conv_tail ? conv_tail[i] : nullptr, ws, st, r, x));
    }
    return MB2_OK;
}

// One decode step of the stack: per layer the row-rms of the token rows, then
// the block's step with 1/rms in in_proj's epilogue (norm weight folded into
// in_proj) and the residual added in place by out_proj's epilogue.
static size_t stack_step_bytes(const mb2_block *layers, int64_t n_layers, int64_t batch,
                               size_t *off_r) {
    size_t ws = 0;
    for (int64_t i = 0; i < n_layers; ++i) {
        const size_t t = make_layout(&layers[i], batch, true).total;
        ws = t > ws ? t : ws;
    }
    *off_r = ws;
    return ws + align256((size_t)batch * sizeof(float));
}

extern "C" size_t mb2_stack_step_workspace_bytes(const mb2_block *layers, int64_t n_layers,
                                                 int64_t batch) {
    if (!layers || n_layers <= 0 || batch < 0) return 0;
    size_t off_r;
    return stack_step_bytes(layers, n_layers, batch, &off_r);
}

extern "C" int mb2_stack_step(const mb2_block *layers, int64_t n_layers, float eps, void *x,
                              float *const *h, void *const *conv_state, int64_t batch,
                              void *workspace, size_t workspace_bytes, mb2_stream_t stream) {
    MB2_TRY(check_stack(layers, n_layers, eps));
    MB2_REQUIRE(batch >= 0, MB2_ERR_SHAPE, "stack step: negative batch");
    size_t off_r;
    const size_t need = stack_step_bytes(layers, n_layers, batch, &off_r);
    MB2_REQUIRE(workspace_bytes >= need, MB2_ERR_WORKSPACE,
                "stack step: workspace %zu < required %zu", workspace_bytes, need);
    if (batch == 0) return MB2_OK;
    MB2_REQUIRE(x && h && conv_state && workspace, MB2_ERR_ARG, "stack step: null pointer");
    for (int64_t i = 0; i < n_layers; ++i)
        MB2_REQUIRE(h[i] && conv_state[i], MB2_ERR_ARG, "stack step: layer %lld state missing",
                    (long long)i);
    cudaStream_t st = (cudaStream_t)stream;
    char *ws = static_cast<char *>(workspace);
    float *r = reinterpret_cast<float *>(ws + off_r);
    for (int64_t i = 0; i < n_layers; ++i) {
        const mb2_block &b = layers[i];
        const Layout l = make_layout(&b, batch, true);
        MB2_TRY(rms_scale(b.dtype, x, batch, b.d_model, eps, r, st));
        MB2_TRY(step_head(b, l, x, conv_state[i], batch, ws, st, r));
        MB2_TRY(step_tail(b, l, x, h[i], batch, ws, st, x));
    }
    return MB2_OK;
}
