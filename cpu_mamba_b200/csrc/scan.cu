// Selective scan kernels (Mamba S6 recurrence) for sm_100a.
//
// Reference semantics: src/cpu_mamba/selective_scan_cpu.cpp:56-85 -- for each
// (batch b, channel d): h[s] = h0 or 0; for t: dA = exp(dt*A[d,s]);
// dBx = (dt*B[b,t,s])*x; h = dA*h + dBx; y += h*C[b,t,s]; out = y + D[d]*x.
//
// Mapping: one CTA owns (batch b, 128/L consecutive channels) for the whole
// sequence.  Each channel is handled by L adjacent lanes, each holding SPL of
// the d_state states of h in registers (L*SPL >= d_state; padded states have
// A = B = C = 0 and stay 0).  The per-step loop does only the state update and
// writes each lane's partial y to shared memory; after each chunk a read-out
// pass sums the lane partials, adds D x, applies the gate and stores the
// chunk's rows with coalesced writes.
// Time is sequential: the recurrence is cheap, the d_state exponentials per
// token-channel on the MUFU pipe are the bound, and every (b, channel) pair is
// independent, so the GPU is filled by batch x channels without splitting T.
// Inputs for SCAN_TC timesteps are staged in shared memory by asynchronous
// copies one chunk ahead (double buffer): the per-channel x / dt / z rows
// (coalesced across the CTA's channels) and the B / C rows, which every
// channel of the CTA reads with vector loads.
//
// exp(dt*A) is evaluated as 2^(dt * (A log2 e)) with ex2.approx.ftz.
//
// Two modes:
//   plain  -- drop-in for selective_scan_cpu: A given, output y + D x in fp32;
//   gated  -- A = -exp(A_log) from the module's parameter (_mamba.py:222),
//             output cast to the activation dtype and multiplied by SiLU(z)
//             (_mamba.py:263-264).
// dt always arrives precomputed (softplus(dt_proj(.)) is the epilogue of the
// dt_proj GEMM).
#include "common.cuh"

namespace mb2 {

constexpr int SCAN_THREADS = 128;  // threads per CTA; channels per CTA = 128 / L
constexpr int SCAN_TC = 16;        // timesteps per staged chunk

struct ScanParams {
    const void *x;  int64_t ld_x;    // (N, ld_x)  x / conv output
    const void *dt; int64_t ld_dt;   // (N, ld_dt) dt (softplus applied)
    const void *z;  int64_t ld_z;    // (N, ld_z)  gate input (gated mode)
    const void *bm; int64_t ld_b;    // rows of B
    const void *cm; int64_t ld_c;    // rows of C
    const void *A;                   // A fp32 (plain) or A_log in T (gated)
    const void *D;                   // (di) fp32 (plain) / T (gated), may be null
    const float *h0; float *h_last;  // (batch, di, S) or null
    void *y;        int64_t ld_y;
    int64_t batch, seqlen, d_inner;
    int d_state, lanes;              // lanes == L
    unsigned vec16;                  // bit i: array i rows are 16-byte aligned
};

enum { ARR_X = 1, ARR_DT = 2, ARR_Z = 4, ARR_B = 8, ARR_C = 16 };

template <typename T> __host__ __device__ constexpr int epw() { return 4 / (int)sizeof(T); }

__device__ __forceinline__ float ex2(float v) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}

// Stage rows x cols_padded elements of a row-major source into shared memory
// (valid cols copied, the rest zero-filled): 16-byte async copies when the
// rows are 16-byte aligned, else 4-byte copies with hardware zero fill.
template <typename T>
__device__ __forceinline__ void stage_rows(T *dst, int cols_padded, const T *src, int64_t ld,
                                           int64_t row0, int rows_valid, int rows, int cols,
                                           bool vec16, int tid, int nthr) {
    constexpr int E = epw<T>();
    if (vec16) {
        constexpr int V = 16 / (int)sizeof(T);        // elements per 16-byte chunk
        const int cpr = cols_padded / V;              // chunks per row
        const int total = rows * cpr;
        for (int i = tid; i < total; i += nthr) {
            const int r = i / cpr;
            const int c = (i - r * cpr) * V;
            const uint32_t s = smem_u32(dst + r * cols_padded + c);
            const bool rv = r < rows_valid;
            if (rv && c + V <= cols) {
                cp_async16(dst + r * cols_padded + c, src + (row0 + r) * ld + c);
            } else {
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const int cw = c + w * E;
                    int bytes = 0;
                    const T *g = src;
                    if (rv && cw < cols) {
                        g = src + (row0 + r) * ld + cw;
                        bytes = (cols - cw >= E) ? 4 : 2;
                    }
                    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n"
                                 ::"r"(s + 4 * w), "l"(g), "r"(bytes));
                }
            }
        }
        return;
    }
    const int wpr = cols_padded / E;  // words per row
    const int total = rows * wpr;
    for (int i = tid; i < total; i += nthr) {
        const int r = i / wpr;
        const int c = (i - r * wpr) * E;
        int bytes = 0;
        const T *g = src;
        if (r < rows_valid && c < cols) {
            g = src + (row0 + r) * ld + c;
            bytes = (cols - c >= E) ? 4 : 2;  // half word only for bf16 tails
        }
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n"
                     ::"r"(smem_u32(dst + r * cols_padded + c)), "l"(g), "r"(bytes));
    }
}

// N consecutive values from shared memory as floats, widest aligned loads.
template <typename T, int N> struct Vec;
template <int N> struct Vec<float, N> {
    static __device__ __forceinline__ void load(const float *p, float (&v)[N]) {
#pragma unroll
        for (int k = 0; k < N / 4; ++k) {
            const float4 q = reinterpret_cast<const float4 *>(p)[k];
            v[4 * k] = q.x; v[4 * k + 1] = q.y; v[4 * k + 2] = q.z; v[4 * k + 3] = q.w;
        }
    }
};
template <int N> struct Vec<__nv_bfloat16, N> {
    static __device__ __forceinline__ void load(const __nv_bfloat16 *p, float (&v)[N]) {
#pragma unroll
        for (int k = 0; k < N / 4; ++k) {
            const uint2 q = reinterpret_cast<const uint2 *>(p)[k];
            v[4 * k] = __uint_as_float(q.x << 16);
            v[4 * k + 1] = __uint_as_float(q.x & 0xFFFF0000u);
            v[4 * k + 2] = __uint_as_float(q.y << 16);
            v[4 * k + 3] = __uint_as_float(q.y & 0xFFFF0000u);
        }
    }
};

// Per-stage layout (elements of T): x | dt | z | B | C, each block a multiple
// of 16 bytes so every array starts 16-byte aligned.  After the two stages
// comes one float block of SCAN_TC x 128 per-lane partial sums of y.
struct StageLayout {
    int CH, SPp, n_x, n_bc, elems;
    __host__ __device__ StageLayout(int L, int spl, int esize, bool gated) {
        CH = SCAN_THREADS / L;
        const int v = 16 / esize;
        SPp = ((L * spl + v - 1) / v) * v;
        n_x = SCAN_TC * CH;
        n_bc = SCAN_TC * SPp;
        elems = (gated ? 3 : 2) * n_x + 2 * n_bc;
    }
    __host__ __device__ size_t bytes(int esize) const {
        return 2 * (size_t)elems * esize + (size_t)SCAN_TC * SCAN_THREADS * sizeof(float);
    }
};

template <typename T, int SPL, bool GATED>
__global__ void __launch_bounds__(SCAN_THREADS, 5)
scan_kernel(const ScanParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int L = p.lanes;
    const StageLayout lay(L, SPL, (int)sizeof(T), GATED);
    const int CH = lay.CH;
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
    T *stage0 = reinterpret_cast<T *>(smem_raw);
    // per-lane partial y of the current chunk: ys[tt][tid]
    float *ys = reinterpret_cast<float *>(smem_raw + 2 * (size_t)lay.elems * sizeof(T));

    float A2[SPL], h[SPL];
#pragma unroll
    for (int i = 0; i < SPL; ++i) {
        const int s = j * SPL + i;
        float a = 0.0f, h_init = 0.0f;
        if (active && s < S) {
            if (GATED)
                a = -expf(io<T>::to_f(static_cast<const T *>(p.A)[d * S + s]));
            else
                a = static_cast<const float *>(p.A)[d * S + s];
            if (p.h0) h_init = p.h0[((int64_t)b * p.d_inner + d) * S + s];
        }
        A2[i] = a * kLog2e;
        h[i] = h_init;
    }

    const int64_t row_base = (int64_t)b * p.seqlen;
    const T *xg = static_cast<const T *>(p.x) + d0;
    const T *dtg = static_cast<const T *>(p.dt) + d0;
    const T *zg = GATED ? static_cast<const T *>(p.z) + d0 : nullptr;
    const T *bg = static_cast<const T *>(p.bm);
    const T *cg = static_cast<const T *>(p.cm);
    const int nz = GATED ? 1 : 0;

    auto issue = [&](int chunk) {
        T *st = stage0 + (chunk & 1) * lay.elems;
        const int t0 = chunk * SCAN_TC;
        const int rv = min(SCAN_TC, T_ - t0);
        const int64_t r0 = row_base + t0;
        stage_rows<T>(st, CH, xg, p.ld_x, r0, rv, SCAN_TC, ch_valid, p.vec16 & ARR_X,
                      tid, SCAN_THREADS);
        stage_rows<T>(st + lay.n_x, CH, dtg, p.ld_dt, r0, rv, SCAN_TC, ch_valid,
                      p.vec16 & ARR_DT, tid, SCAN_THREADS);
        if (GATED)
            stage_rows<T>(st + 2 * lay.n_x, CH, zg, p.ld_z, r0, rv, SCAN_TC, ch_valid,
                          p.vec16 & ARR_Z, tid, SCAN_THREADS);
        stage_rows<T>(st + (2 + nz) * lay.n_x, lay.SPp, bg, p.ld_b, r0, rv, SCAN_TC, S,
                      p.vec16 & ARR_B, tid, SCAN_THREADS);
        stage_rows<T>(st + (2 + nz) * lay.n_x + lay.n_bc, lay.SPp, cg, p.ld_c, r0, rv, SCAN_TC,
                      S, p.vec16 & ARR_C, tid, SCAN_THREADS);
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
        const T *st = stage0 + (ch & 1) * lay.elems;
        const T *xs = st + c;
        const T *dts = st + lay.n_x + c;
        const T *bs = st + (2 + nz) * lay.n_x + j * SPL;
        const T *cs = bs + lay.n_bc;
        const int t0 = ch * SCAN_TC;
        const int tn = min(SCAN_TC, T_ - t0);
        // recurrence: per step only the state update and this lane's partial y
#pragma unroll 2
        for (int tt = 0; tt < tn; ++tt) {
            const float xv = io<T>::to_f(xs[tt * CH]);
            const float dtv = io<T>::to_f(dts[tt * CH]);
            const float dtx = dtv * xv;
            float bv[SPL], cv[SPL];
            Vec<T, SPL>::load(bs + tt * lay.SPp, bv);
            Vec<T, SPL>::load(cs + tt * lay.SPp, cv);
            float y0 = 0.0f, y1 = 0.0f, y2 = 0.0f;
#pragma unroll
            for (int i = 0; i < SPL; ++i) {
                const float dA = ex2(dtv * A2[i]);
                h[i] = fmaf(dA, h[i], dtx * bv[i]);
                if (i % 3 == 0) y0 = fmaf(h[i], cv[i], y0);
                else if (i % 3 == 1) y1 = fmaf(h[i], cv[i], y1);
                else y2 = fmaf(h[i], cv[i], y2);
            }
            ys[tt * SCAN_THREADS + tid] = (y0 + y1) + y2;
        }
        __syncthreads();
        // read-out: y = sum of lane partials + D x, then (gated) cast and
        // SiLU(z) gate; coalesced row segments of CH channels
        const T *xrow = st;
        const T *zrow = st + 2 * lay.n_x;
        for (int e = tid; e < tn * CH; e += SCAN_THREADS) {
            const int tt = e / CH, cc = e - tt * CH;
            const int64_t dd = d0 + cc;
            if (dd >= p.d_inner) continue;
            float yv = 0.0f;
            for (int l = 0; l < L; ++l) yv += ys[tt * SCAN_THREADS + cc * L + l];
            const float xv = io<T>::to_f(xrow[tt * CH + cc]);
            const float dd_v = GATED ? io<T>::to_f(static_cast<const T *>(p.D)[dd])
                                     : static_cast<const float *>(p.D)[dd];
            float out = yv + (p.D ? dd_v : 0.0f) * xv;
            if (GATED) {
                const float zv = io<T>::to_f(zrow[tt * CH + cc]);
                out = io<T>::round(out) * io<T>::round(silu_f(zv));
            }
            yg[(row_base + t0 + tt) * p.ld_y + dd] = io<T>::from_f(out);
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

static bool rows16(const void *p, int64_t ld, size_t es) {
    return aligned(p, 16) && (ld * (int64_t)es) % 16 == 0;
}

template <typename T, int SPL, bool GATED>
static int launch_scan(ScanParams p, cudaStream_t st) {
    const StageLayout lay(p.lanes, SPL, (int)sizeof(T), GATED);
    const size_t smem = lay.bytes((int)sizeof(T));
    auto kern = scan_kernel<T, SPL, GATED>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return fail(MB2_ERR_CUDA, "scan: smem attribute: %s", cudaGetErrorString(e));
    }
    const size_t es = sizeof(T);
    // the x / dt / z tiles start at channel d0 = blockIdx.x * CH
    const bool ch16 = (lay.CH * es) % 16 == 0;
    p.vec16 = 0;
    if (ch16 && rows16(p.x, p.ld_x, es)) p.vec16 |= ARR_X;
    if (ch16 && rows16(p.dt, p.ld_dt, es)) p.vec16 |= ARR_DT;
    if (GATED && ch16 && rows16(p.z, p.ld_z, es)) p.vec16 |= ARR_Z;
    if (rows16(p.bm, p.ld_b, es)) p.vec16 |= ARR_B;
    if (rows16(p.cm, p.ld_c, es)) p.vec16 |= ARR_C;
    dim3 grid((unsigned)ceil_div(p.d_inner, lay.CH), (unsigned)p.batch);
    kern<<<grid, SCAN_THREADS, smem, st>>>(p);
    return check_launch("scan_kernel");
}

template <typename T, bool GATED>
static int dispatch_scan(ScanParams p, cudaStream_t st) {
    const ScanShape sh = pick_shape(p.d_state);
    p.lanes = sh.lanes;
    switch (sh.spl) {
        case 8: return launch_scan<T, 8, GATED>(p, st);
        case 12: return launch_scan<T, 12, GATED>(p, st);
        default: return launch_scan<T, 16, GATED>(p, st);
    }
}

// Shared argument checks; 4-byte staging copies need 4-byte aligned bf16 rows.
static int check_rows(int dtype, const void *ptr, int64_t ld, int64_t cols, const char *name) {
    MB2_REQUIRE(ld >= cols, MB2_ERR_SHAPE, "scan: leading dimension of %s too small", name);
    if (dtype == MB2_BF16)
        MB2_REQUIRE(aligned(ptr, 4) && ld % 2 == 0, MB2_ERR_ALIGN,
                    "scan(bf16): %s rows must start on 4-byte boundaries (even offsets and "
                    "leading dimension)", name);
    return MB2_OK;
}

int scan_gated(int dtype, const void *xc, int64_t ld_xc, const void *dt, int64_t ld_dt,
               const void *bm, int64_t ld_b, const void *cm, int64_t ld_c, const void *z,
               int64_t ld_z, const void *A_log, const void *D, const float *h0, float *h_last,
               void *y, int64_t ld_y, int64_t batch, int64_t seqlen, int64_t d_inner,
               int64_t d_state, cudaStream_t stream) {
    MB2_REQUIRE(dtype == MB2_F32 || dtype == MB2_BF16, MB2_ERR_ARG, "scan: bad dtype");
    MB2_REQUIRE(batch >= 0 && seqlen >= 0 && d_inner >= 0, MB2_ERR_SHAPE, "scan: bad sizes");
    MB2_REQUIRE(d_state >= 1 && d_state <= 256, MB2_ERR_SHAPE,
                "d_state > 256 not supported (got %lld)", (long long)d_state);
    MB2_REQUIRE(batch < 65536, MB2_ERR_SHAPE, "scan: batch too large");
    if (batch == 0 || d_inner == 0) return MB2_OK;
    MB2_REQUIRE(A_log && (seqlen == 0 || (xc && dt && bm && cm && z && y)), MB2_ERR_ARG,
                "scan: null pointer");
    if (dtype == MB2_BF16)
        MB2_REQUIRE(d_inner % 2 == 0 && d_state % 2 == 0, MB2_ERR_ALIGN,
                    "scan(bf16): d_inner and d_state must be even");
    MB2_TRY(check_rows(dtype, xc, ld_xc, d_inner, "x"));
    MB2_TRY(check_rows(dtype, dt, ld_dt, d_inner, "dt"));
    MB2_TRY(check_rows(dtype, z, ld_z, d_inner, "z"));
    MB2_TRY(check_rows(dtype, bm, ld_b, d_state, "B"));
    MB2_TRY(check_rows(dtype, cm, ld_c, d_state, "C"));
    MB2_REQUIRE(ld_y >= d_inner, MB2_ERR_SHAPE, "scan: leading dimension of y too small");
    ScanParams p{};
    p.x = xc; p.ld_x = ld_xc;
    p.dt = dt; p.ld_dt = ld_dt;
    p.z = z; p.ld_z = ld_z;
    p.bm = bm; p.ld_b = ld_b;
    p.cm = cm; p.ld_c = ld_c;
    p.A = A_log; p.D = D; p.h0 = h0; p.h_last = h_last;
    p.y = y; p.ld_y = ld_y;
    p.batch = batch; p.seqlen = seqlen; p.d_inner = d_inner;
    p.d_state = (int)d_state;
    if (dtype == MB2_F32) return dispatch_scan<float, true>(p, stream);
    return dispatch_scan<__nv_bfloat16, true>(p, stream);
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
    p.dt = dt; p.ld_dt = d_inner;
    p.bm = B; p.ld_b = d_state;
    p.cm = C; p.ld_c = d_state;
    p.A = A; p.D = D; p.h0 = h0; p.h_last = h_last;
    p.y = y; p.ld_y = d_inner;
    p.batch = batch; p.seqlen = seqlen; p.d_inner = d_inner;
    p.d_state = (int)d_state;
    return dispatch_scan<float, false>(p, (cudaStream_t)stream);
}

extern "C" int mb2_scan_fused(int dtype, const void *xc, int64_t ld_xc, const void *dt,
                              int64_t ld_dt, const void *B, int64_t ld_b, const void *C,
                              int64_t ld_c, const void *z, int64_t ld_z, const void *A_log,
                              const void *D, const float *h0, float *h_last, void *y,
                              int64_t ld_y, int64_t batch, int64_t seqlen, int64_t d_inner,
                              int64_t d_state, mb2_stream_t stream) {
    return scan_gated(dtype, xc, ld_xc, dt, ld_dt, B, ld_b, C, ld_c, z, ld_z, A_log, D, h0,
                      h_last, y, ld_y, batch, seqlen, d_inner, d_state, (cudaStream_t)stream);
}
