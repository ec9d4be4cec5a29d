// Selective scan kernels (Mamba S6 recurrence) for sm_100a.
//
// Reference semantics: src/cpu_mamba/selective_scan_cpu.cpp:56-85 -- for each
// (batch b, channel d): h[s] = 0; for t: dA = exp(dt*A[d,s]);
// dBx = (dt*B[b,t,s])*x; h = dA*h + dBx; y += h*C[b,t,s]; out = y + D[d]*x.
//
// Mapping: one CTA owns (batch b, 128/L consecutive channels) for the whole
// sequence.  Each channel is handled by L adjacent lanes, each holding SPL of
// the d_state states of h in registers (L*SPL >= d_state, padded states have
// A = B = C = 0 so they stay 0).  The per-lane partial y is reduced with
// shuffles.  Time is sequential; inputs for SCAN_TC timesteps are staged in
// shared memory by asynchronous copies one chunk ahead (double buffer).
//
// exp(dt*A) is evaluated as exp2(dt * (A*log2 e)) on the MUFU pipe, which is
// the bound of this kernel (d_state exponentials per token-channel).
//
// Two modes:
//   plain  -- drop-in for selective_scan_cpu: dt given, A given, no gate;
//   fused  -- dt = softplus(dt_low . W_dt[d] + b_dt) computed in registers
//             (dt_proj fused: _mamba.py:219-220), A = -exp(A_log) (:222),
//             output cast to the activation dtype and gated by SiLU(z)
//             (:263-264).
#include "common.cuh"

namespace mb2 {

constexpr int SCAN_THREADS = 128;  // threads per CTA; channels per CTA = 128 / L
constexpr int SCAN_TC = 16;        // timesteps per staged chunk

struct ScanParams {
    const void *x;    int64_t ld_x;   // (N, ld_x)   x (plain) / conv output (fused)
    const void *d2;   int64_t ld_d2;  // (N, ld_d2)  dt (plain) / z (fused)
    const void *bm;   int64_t ld_b;   // rows of B
    const void *cm;   int64_t ld_c;   // rows of C
    const void *dl;   int64_t ld_dl;  // rows of dt_low (fused)
    const void *w_dt; const void *b_dt;  // (di, R), (di)            (fused)
    const void *A;                    // A (fp32, plain) or A_log (dtype, fused)
    const void *D;                    // (di) fp32 (plain) / dtype (fused)
    const float *h0; float *h_last;   // (batch, di, S) or null
    void *y;          int64_t ld_y;
    int64_t batch, seqlen, d_inner;
    int d_state, dt_rank, lanes;      // lanes == L
};

// Words (4-byte units) of one staged row segment of `n` elements of T.
template <typename T> __host__ __device__ constexpr int epw() { return 4 / (int)sizeof(T); }

// Stage `rows` x `cols_padded` elements (cols valid, rest zero) of a row-major
// source into shared memory, as 4-byte async copies with zero fill.
template <typename T>
__device__ __forceinline__ void stage_rows(T *dst, int cols_padded, const T *src,
                                           int64_t ld, int64_t row0, int rows_valid,
                                           int rows, int cols, int tid, int nthr) {
    constexpr int E = epw<T>();
    const int wpr = cols_padded / E;  // words per row (cols_padded % E == 0)
    const int total = rows * wpr;
    for (int i = tid; i < total; i += nthr) {
        const int r = i / wpr;
        const int w = i - r * wpr;
        const int c = w * E;
        int bytes = 0;
        const T *g = src;
        if (r < rows_valid && c < cols) {
            g = src + (row0 + r) * ld + c;
            bytes = (cols - c >= E) ? 4 : 2;  // half word only for bf16 tails
        }
        uint32_t s = smem_u32(dst + r * cols_padded + c);
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(g),
                     "r"(bytes));
    }
}

template <typename T, int SPL, int RMAX, bool FUSED>
__global__ void __launch_bounds__(SCAN_THREADS, 4)
scan_kernel(const ScanParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    constexpr int E = epw<T>();
    const int L = p.lanes;
    const int CH = SCAN_THREADS / L;  // channels per CTA
    const int nthr = SCAN_THREADS;
    const int tid = threadIdx.x;
    const int c = tid / L;         // channel within CTA
    const int j = tid - c * L;     // lane within channel group
    const int b = blockIdx.y;
    const int64_t d0 = (int64_t)blockIdx.x * CH;
    const int64_t d = d0 + c;
    const bool active = d < p.d_inner;
    const int S = p.d_state;
    const int T_ = (int)p.seqlen;
    const int ch_valid = (int)((p.d_inner - d0 < CH) ? p.d_inner - d0 : CH);

    // staged layout (per stage), all row lengths multiples of E elements
    const int SP = L * SPL;                        // padded states per row
    const int SPp = ((SP + E - 1) / E) * E;
    const int RP = FUSED ? L * RMAX : 0;           // padded dt_low per row
    const int n_x = SCAN_TC * CH;
    const int n_bc = SCAN_TC * SPp;
    const int n_dl = SCAN_TC * RP;
    const int stage_elems = 2 * n_x + 2 * n_bc + n_dl;
    T *stage0 = reinterpret_cast<T *>(smem_raw);

    // per-thread constants
    float A2[SPL], h[SPL];
#pragma unroll
    for (int i = 0; i < SPL; ++i) {
        const int s = j * SPL + i;
        float a = 0.0f, h_init = 0.0f;
        if (active && s < S) {
            if (FUSED) {
                const float alog = io<T>::to_f(static_cast<const T *>(p.A)[d * S + s]);
                a = -expf(alog);
            } else {
                a = static_cast<const float *>(p.A)[d * S + s];
            }
            if (p.h0) h_init = p.h0[((int64_t)b * p.d_inner + d) * S + s];
        }
        A2[i] = a * kLog2e;
        h[i] = h_init;
    }
    float wdt[FUSED ? RMAX : 1];
    float bias_dt = 0.0f, Dv = 0.0f;
    if (FUSED) {
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
            const int rr = j * RMAX + r;
            wdt[r] = (active && rr < p.dt_rank)
                         ? io<T>::to_f(static_cast<const T *>(p.w_dt)[d * p.dt_rank + rr])
                         : 0.0f;
        }
        if (active) {
            bias_dt = p.b_dt ? io<T>::to_f(static_cast<const T *>(p.b_dt)[d]) : 0.0f;
            Dv = p.D ? io<T>::to_f(static_cast<const T *>(p.D)[d]) : 0.0f;
        }
    } else if (active) {
        Dv = p.D ? static_cast<const float *>(p.D)[d] : 0.0f;
    }

    const int64_t row_base = (int64_t)b * p.seqlen;
    const T *xg = static_cast<const T *>(p.x) + d0;
    const T *d2g = static_cast<const T *>(p.d2) + d0;
    const T *bg = static_cast<const T *>(p.bm);
    const T *cg = static_cast<const T *>(p.cm);
    const T *dlg = static_cast<const T *>(p.dl);

    auto issue = [&](int chunk) {
        T *st = stage0 + (chunk & 1) * stage_elems;
        const int t0 = chunk * SCAN_TC;
        const int rv = min(SCAN_TC, T_ - t0);
        const int64_t r0 = row_base + t0;
        stage_rows<T>(st, CH, xg, p.ld_x, r0, rv, SCAN_TC, ch_valid, tid, nthr);
        stage_rows<T>(st + n_x, CH, d2g, p.ld_d2, r0, rv, SCAN_TC, ch_valid, tid, nthr);
        stage_rows<T>(st + 2 * n_x, SPp, bg, p.ld_b, r0, rv, SCAN_TC, S, tid, nthr);
        stage_rows<T>(st + 2 * n_x + n_bc, SPp, cg, p.ld_c, r0, rv, SCAN_TC, S, tid, nthr);
        if (FUSED)
            stage_rows<T>(st + 2 * n_x + 2 * n_bc, RP, dlg, p.ld_dl, r0, rv, SCAN_TC,
                          p.dt_rank, tid, nthr);
    };

    const int nchunks = (T_ + SCAN_TC - 1) / SCAN_TC;
    if (nchunks > 0) issue(0);
    cp_async_commit();
    T *yg = static_cast<T *>(p.y);

    for (int ch = 0; ch < nchunks; ++ch) {
        if (ch + 1 < nchunks) issue(ch + 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const T *st = stage0 + (ch & 1) * stage_elems;
        const T *xs = st;
        const T *d2s = st + n_x;
        const T *bs = st + 2 * n_x + j * SPL;
        const T *cs = st + 2 * n_x + n_bc + j * SPL;
        const T *dls = st + 2 * n_x + 2 * n_bc + j * RMAX;
        const int t0 = ch * SCAN_TC;
        const int tn = min(SCAN_TC, T_ - t0);
        for (int tt = 0; tt < tn; ++tt) {
            const float xv = io<T>::to_f(xs[tt * CH + c]);
            float dtv;
            if (FUSED) {
                float part = 0.0f;
#pragma unroll
                for (int r = 0; r < RMAX; ++r)
                    part = fmaf(io<T>::to_f(dls[tt * RP + r]), wdt[r], part);
                for (int m = 1; m < L; m <<= 1) part += __shfl_xor_sync(0xffffffffu, part, m);
                const float v = io<T>::round(part + bias_dt);
                dtv = io<T>::round(softplus_f(v));
            } else {
                dtv = io<T>::to_f(d2s[tt * CH + c]);
            }
            float yp = 0.0f;
#pragma unroll
            for (int i = 0; i < SPL; ++i) {
                const float bv = io<T>::to_f(bs[tt * SPp + i]);
                const float cv = io<T>::to_f(cs[tt * SPp + i]);
                const float dA = exp2f(dtv * A2[i]);
                const float dBx = (dtv * bv) * xv;
                h[i] = fmaf(dA, h[i], dBx);
                yp = fmaf(h[i], cv, yp);
            }
            for (int m = 1; m < L; m <<= 1) yp += __shfl_xor_sync(0xffffffffu, yp, m);
            if (j == 0 && active) {
                float out = yp + Dv * xv;
                if (FUSED) {
                    const float zv = io<T>::to_f(d2s[tt * CH + c]);
                    out = io<T>::round(out) * io<T>::round(silu_f(zv));
                }
                yg[(row_base + t0 + tt) * p.ld_y + d] = io<T>::from_f(out);
            }
        }
        __syncthreads();
    }
    cp_async_wait<0>();
    if (p.h_last && active) {
#pragma unroll
        for (int i = 0; i < SPL; ++i) {
            const int s = j * SPL + i;
            if (s < S) p.h_last[((int64_t)b * p.d_inner + d) * S + s] = h[i];
        }
    }
}

// -------------------------------------------------------------- dispatch ---
struct ScanShape { int spl, lanes; };

static ScanShape pick_shape(int S) {
    if (S <= 8) return {8, 1};
    if (S <= 16) return {8, 2};
    if (S <= 24) return {12, 2};
    if (S <= 32) return {16, 2};
    if (S <= 64) return {16, 4};
    if (S <= 128) return {16, 8};
    return {16, 16};
}

static int pick_rmax(int R, int L) {
    const int per = (R + L - 1) / L;
    const int opts[] = {8, 16, 24, 32, 48, 64};
    for (int o : opts)
        if (per <= o) return o;
    return -1;
}

template <typename T, int SPL, int RMAX, bool FUSED>
static int launch_scan(const ScanParams &p, cudaStream_t st) {
    constexpr int E = epw<T>();
    const int L = p.lanes;
    const int SP = L * SPL;
    const int SPp = ((SP + E - 1) / E) * E;
    const int RP = FUSED ? L * RMAX : 0;
    const int CH = SCAN_THREADS / L;
    const size_t stage = (size_t)(2 * SCAN_TC * CH + 2 * SCAN_TC * SPp + SCAN_TC * RP) * sizeof(T);
    const size_t smem = 2 * stage;
    auto kern = scan_kernel<T, SPL, RMAX, FUSED>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return fail(MB2_ERR_CUDA, "scan: smem attribute: %s", cudaGetErrorString(e));
    }
    dim3 grid((unsigned)ceil_div(p.d_inner, CH), (unsigned)p.batch);
    kern<<<grid, SCAN_THREADS, smem, st>>>(p);
    return check_launch("scan_kernel");
}

template <typename T, bool FUSED, int SPL>
static int dispatch_rmax(const ScanParams &p, int rmax, cudaStream_t st) {
    if constexpr (!FUSED) {
        return launch_scan<T, SPL, 8, false>(p, st);
    } else {
    switch (rmax) {
        case 8: return launch_scan<T, SPL, 8, FUSED>(p, st);
        case 16: return launch_scan<T, SPL, 16, FUSED>(p, st);
        case 24: return launch_scan<T, SPL, 24, FUSED>(p, st);
        case 32: return launch_scan<T, SPL, 32, FUSED>(p, st);
        case 48: return launch_scan<T, SPL, 48, FUSED>(p, st);
        case 64: return launch_scan<T, SPL, 64, FUSED>(p, st);
    }
    return fail(MB2_ERR_UNSUPPORTED, "scan: dt_rank %d too large for %d lanes", p.dt_rank, p.lanes);
    }
}

template <typename T, bool FUSED>
static int dispatch_scan(ScanParams p, cudaStream_t st) {
    const ScanShape sh = pick_shape(p.d_state);
    p.lanes = sh.lanes;
    const int rmax = FUSED ? pick_rmax(p.dt_rank, sh.lanes) : 8;
    if (FUSED && rmax < 0)
        return fail(MB2_ERR_UNSUPPORTED, "scan: dt_rank %d too large (max %d for d_state %d)",
                    p.dt_rank, 64 * sh.lanes, p.d_state);
    switch (sh.spl) {
        case 8: return dispatch_rmax<T, FUSED, 8>(p, rmax, st);
        case 12: return dispatch_rmax<T, FUSED, 12>(p, rmax, st);
        default: return dispatch_rmax<T, FUSED, 16>(p, rmax, st);
    }
}

}  // namespace mb2

using namespace mb2;

extern "C" int mb2_selective_scan(const float *x, const float *dt, const float *A,
                                  const float *B, const float *C, const float *D,
                                  float *y, int64_t batch, int64_t seqlen,
                                  int64_t d_inner, int64_t d_state, const float *h0,
                                  float *h_last, mb2_stream_t stream) {
    MB2_REQUIRE(batch >= 0 && seqlen >= 0 && d_inner >= 0, MB2_ERR_SHAPE,
                "selective_scan: negative size");
    MB2_REQUIRE(d_state >= 1 && d_state <= 256, MB2_ERR_SHAPE,
                "d_state > 256 not supported (got %lld)", (long long)d_state);
    MB2_REQUIRE(batch < 65536, MB2_ERR_SHAPE, "selective_scan: batch %lld >= 65536",
                (long long)batch);
    if (batch == 0 || d_inner == 0) return MB2_OK;
    MB2_REQUIRE(A && D && (seqlen == 0 || (x && dt && B && C && y)), MB2_ERR_ARG,
                "selective_scan: null pointer");
    ScanParams p{};
    p.x = x; p.ld_x = d_inner;
    p.d2 = dt; p.ld_d2 = d_inner;
    p.bm = B; p.ld_b = d_state;
    p.cm = C; p.ld_c = d_state;
    p.A = A; p.D = D; p.h0 = h0; p.h_last = h_last;
    p.y = y; p.ld_y = d_inner;
    p.batch = batch; p.seqlen = seqlen; p.d_inner = d_inner;
    p.d_state = (int)d_state; p.dt_rank = 0;
    return dispatch_scan<float, false>(p, (cudaStream_t)stream);
}

extern "C" int mb2_scan_fused(int dtype, const void *xc, int64_t ld_xc, const void *xdbl,
                              int64_t ld_xdbl, const void *z, int64_t ld_z,
                              const void *w_dt, const void *b_dt, const void *A_log,
                              const void *D, const float *h0, float *h_last, void *y,
                              int64_t ld_y, int64_t batch, int64_t seqlen, int64_t d_inner,
                              int64_t d_state, int64_t dt_rank, mb2_stream_t stream) {
    MB2_REQUIRE(dtype == MB2_F32 || dtype == MB2_BF16, MB2_ERR_ARG, "scan_fused: bad dtype");
    MB2_REQUIRE(batch >= 0 && seqlen >= 0 && d_inner >= 0 && dt_rank >= 1, MB2_ERR_SHAPE,
                "scan_fused: bad sizes");
    MB2_REQUIRE(d_state >= 1 && d_state <= 256, MB2_ERR_SHAPE,
                "d_state > 256 not supported (got %lld)", (long long)d_state);
    MB2_REQUIRE(batch < 65536, MB2_ERR_SHAPE, "scan_fused: batch too large");
    if (batch == 0 || d_inner == 0) return MB2_OK;
    MB2_REQUIRE(w_dt && A_log && (seqlen == 0 || (xc && xdbl && z && y)), MB2_ERR_ARG,
                "scan_fused: null pointer");
    MB2_REQUIRE(ld_xc >= d_inner && ld_z >= d_inner && ld_y >= d_inner &&
                    ld_xdbl >= dt_rank + 2 * d_state,
                MB2_ERR_SHAPE, "scan_fused: leading dimension too small");
    const size_t es = dtype_size(dtype);
    if (dtype == MB2_BF16) {
        // 4-byte staging copies: every row segment must start on a 4-byte boundary
        MB2_REQUIRE(aligned(xc, 4) && aligned(z, 4) && aligned(xdbl, 4) && ld_xc % 2 == 0 &&
                        ld_z % 2 == 0 && ld_xdbl % 2 == 0 && dt_rank % 2 == 0 &&
                        d_state % 2 == 0 && d_inner % 2 == 0,
                    MB2_ERR_ALIGN,
                    "scan_fused(bf16): pointers, leading dims, d_inner, dt_rank and d_state "
                    "must be even / 4-byte aligned");
    }
    (void)es;
    ScanParams p{};
    const char *xd = static_cast<const char *>(xdbl);
    p.x = xc; p.ld_x = ld_xc;
    p.d2 = z; p.ld_d2 = ld_z;
    p.dl = xd; p.ld_dl = ld_xdbl;
    p.bm = xd + dt_rank * es; p.ld_b = ld_xdbl;
    p.cm = xd + (dt_rank + d_state) * es; p.ld_c = ld_xdbl;
    p.w_dt = w_dt; p.b_dt = b_dt; p.A = A_log; p.D = D;
    p.h0 = h0; p.h_last = h_last;
    p.y = y; p.ld_y = ld_y;
    p.batch = batch; p.seqlen = seqlen; p.d_inner = d_inner;
    p.d_state = (int)d_state; p.dt_rank = (int)dt_rank;
    if (dtype == MB2_F32) return dispatch_scan<float, true>(p, (cudaStream_t)stream);
    return dispatch_scan<__nv_bfloat16, true>(p, (cudaStream_t)stream);
}

// Internal entry for the block forward: x_dbl with separately aligned segments.
namespace mb2 {
int scan_fused_segments(int dtype, const void *xc, int64_t ld_xc, const void *dl,
                        const void *bm, const void *cm, int64_t ld_row, const void *z,
                        int64_t ld_z, const void *w_dt, const void *b_dt, const void *A_log,
                        const void *D, const float *h0, float *h_last, void *y, int64_t ld_y,
                        int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state,
                        int64_t dt_rank, cudaStream_t stream) {
    ScanParams p{};
    p.x = xc; p.ld_x = ld_xc;
    p.d2 = z; p.ld_d2 = ld_z;
    p.dl = dl; p.ld_dl = ld_row;
    p.bm = bm; p.ld_b = ld_row;
    p.cm = cm; p.ld_c = ld_row;
    p.w_dt = w_dt; p.b_dt = b_dt; p.A = A_log; p.D = D;
    p.h0 = h0; p.h_last = h_last;
    p.y = y; p.ld_y = ld_y;
    p.batch = batch; p.seqlen = seqlen; p.d_inner = d_inner;
    p.d_state = (int)d_state; p.dt_rank = (int)dt_rank;
    if (batch == 0 || d_inner == 0) return MB2_OK;
    if (dtype == MB2_F32) return dispatch_scan<float, true>(p, stream);
    return dispatch_scan<__nv_bfloat16, true>(p, stream);
}
}  // namespace mb2
