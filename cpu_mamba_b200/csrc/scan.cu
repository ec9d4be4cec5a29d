// Selective scan kernels (Mamba S6 recurrence) for sm_100a.
//
// Reference semantics: src/cpu_mamba/selective_scan_cpu.cpp:56-85 -- for each
// (batch b, channel d): h[s] = h0 or 0; for t: dA = exp(dt*A[d,s]);
// dBx = (dt*B[b,t,s])*x; h = dA*h + dBx; y += h*C[b,t,s]; out = y + D[d]*x.
//
// Mapping: one CTA owns (batch b, CH = 128/L consecutive channels) for the
// whole sequence.  Each channel is handled by L adjacent lanes, each holding
// SPL of the d_state states of h in registers (L*SPL >= d_state; padded
// states have A = B = C = 0 and stay 0).  Time is sequential: the recurrence
// is cheap, the d_state exponentials per token-channel on the MUFU pipe are
// the bound, and (batch x channel) pairs fill the GPU without splitting T.
//
// Per chunk of SCAN_TC timesteps, inputs are staged in shared memory by
// asynchronous copies one chunk ahead (double buffer): the per-channel x and
// z rows and the per-token rows of B, C (and dt_low) that all channels read.
// The per-step loop only updates the states and writes each lane's partial y
// to shared memory; a read-out pass per chunk sums the L partials, adds D x,
// applies the gate and writes the chunk's rows with coalesced stores.
//
// Modes:
//   PLAIN -- drop-in for selective_scan_cpu: dt, A given; out = y + D x (fp32)
//   FUSED -- the block's stage: dt = softplus(dt_low . W_dt[d] + b_dt) with
//            W_dt's row in registers (dt_proj + softplus, _mamba.py:219-220;
//            exact fp32 FMA dot products for a whole chunk at a time, the
//            softplus of each token-channel computed once, by one of the
//            channel's lanes, into a shared-memory dt tile),
//            A = -exp(A_log) (:222), output cast to the activation dtype and
//            multiplied by SiLU(z) (:263-264).
//   GATED -- FUSED with dt_proj's output given: the block's forward runs the
//            dt_proj GEMM on the tensor cores (bias in its epilogue); the scan
//            stages its rows like x and z and applies the softplus once per
//            token-channel per chunk into the shared-memory dt tile.
// exp(dt*A) is evaluated as 2^(dt * (A log2 e)) with ex2.approx.ftz.
#include "internal.cuh"

namespace mb2 {

constexpr int SCAN_THREADS = 128;  // threads per CTA
constexpr int SCAN_TC = 16;        // timesteps per staged chunk

// SUMMARY: the first pass of a T-segmented GATED scan -- from h = 0, no y;
// writes the segment's final state and the sum of its dt.
enum ScanMode { PLAIN = 0, FUSED = 1, GATED = 2, SUMMARY = 3 };

struct ScanParams {
    const void *x;  int64_t ld_x;    // (N, ld_x)  x / conv output
    const void *dt; int64_t ld_dt;   // PLAIN, GATED: (N, ld_dt) dt
    const void *z;  int64_t ld_z;    // FUSED, GATED: (N, ld_z) gate input
    const void *bm; int64_t ld_b;    // rows of B
    const void *cm; int64_t ld_c;    // rows of C
    const void *dl; int64_t ld_dl;   // FUSED: rows of dt_low (R values)
    const void *w_dt; const void *b_dt;  // FUSED: (di, R), (di)
    const void *A;                   // PLAIN: A fp32; FUSED, GATED: A_log in T
    const void *D;                   // (di) fp32 (PLAIN) / T (FUSED, GATED), may be null
    const float *h0; float *h_last;  // (batch, di, S) or null
    void *y;        int64_t ld_y;
    int64_t batch, seqlen, d_inner;
    int d_state, dt_rank;
    unsigned vec16;                  // bit i: array i rows are 16-byte aligned
    // T segments (few independent chains, long sequences): blockIdx.y =
    // b * nseg + g runs steps [g * seg_len, (g + 1) * seg_len) of sequence b
    int nseg;                        // <= 1: no segments
    int64_t seg_len;
    float *seg_hend;                 // (batch, nseg, d_inner, S)
    float *seg_sdt;                  // (batch, nseg, d_inner)
    const float *seg_hstart;         // pass 3: (batch, nseg, d_inner, S) starting states
    unsigned *amax;                  // or null: fused maxima of |y| (AMAX_SLOTS slots)
    // the block forward's producers apply the activations where they write:
    int dt_act;                      // GATED, SUMMARY: dt rows are softplus(dt_proj) already
    int z_act;                       // FUSED, GATED: z rows are SiLU(z) already
    // T segments with dt rows that are scratch: the summary pass overwrites
    // them with softplus(dt), so the output pass does not evaluate it again
    // (the last segment, which has no summary pass, still does)
    int dt_wb;
};

enum { ARR_X = 1, ARR_D2 = 2, ARR_B = 4, ARR_C = 8, ARR_DL = 16, ARR_Z = 32 };

template <typename T> __host__ __device__ constexpr int epw() { return 4 / (int)sizeof(T); }

// Packed fp32 pairs (sm_100 f32x2 arithmetic: two IEEE fp32 round-to-nearest
// lanes per instruction, halving the FMA-pipe instruction count of the state
// update).  A pair lives in a 64-bit register.
using f2 = unsigned long long;
__device__ __forceinline__ f2 pk(float a, float b) {
    f2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk(f2 v, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
    f2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
    f2 d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// Stage ROWS x COLS_P elements of a row-major source into shared memory
// (`cols` valid, the rest zero-filled).  16-byte async copies when the rows
// are 16-byte aligned, else 4-byte copies with hardware zero fill.
template <typename T, int ROWS, int COLS_P>
__device__ __forceinline__ void stage_rows(T *dst, const T *src, int64_t ld, int rows_valid,
                                           int cols, bool vec16, int tid) {
    constexpr int E = epw<T>();
    if (vec16) {
        constexpr int V = 16 / (int)sizeof(T);       // elements per 16-byte chunk
        constexpr int CPR = COLS_P / V;              // chunks per row
        static_assert(COLS_P % V == 0, "row not a multiple of 16 bytes");
#pragma unroll 1
        for (int i = tid; i < ROWS * CPR; i += SCAN_THREADS) {
            const int r = i / CPR;
            const int c = (i - r * CPR) * V;
            T *d = dst + r * COLS_P + c;
            const bool rv = r < rows_valid;
            if (rv && c + V <= cols) {
                cp_async16(d, src + r * ld + c);
            } else {
                const uint32_t s = smem_u32(d);
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const int cw = c + w * E;
                    const bool ok = rv && cw < cols;
                    const T *g = ok ? src + r * ld + cw : src;
                    const int bytes = ok ? ((cols - cw >= E) ? 4 : 2) : 0;
                    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n"
                                 ::"r"(s + 4 * w), "l"(g), "r"(bytes));
                }
            }
        }
        return;
    }
    constexpr int WPR = COLS_P / E;
    static_assert(COLS_P % E == 0, "row not a multiple of 4 bytes");
#pragma unroll 1
    for (int i = tid; i < ROWS * WPR; i += SCAN_THREADS) {
        const int r = i / WPR;
        const int c = (i - r * WPR) * E;
        const bool ok = r < rows_valid && c < cols;
        const T *g = ok ? src + r * ld + c : src;
        const int bytes = ok ? ((cols - c >= E) ? 4 : 2) : 0;
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n"
                     ::"r"(smem_u32(dst + r * COLS_P + c)), "l"(g), "r"(bytes));
    }
}

// N consecutive values from shared memory as floats, widest aligned loads.
// N consecutive elements of a staged row.  N % 4 == 0: 16-byte (fp32) or
// 8-byte (bf16) loads; otherwise pairs (8 / 4 bytes).  Callers keep the start
// a multiple of 4 elements (of 2 when N % 4 != 0), so every load is aligned.
template <typename T, int N> struct Vec;
template <int N> struct Vec<float, N> {
    static __device__ __forceinline__ void load(const float *p, float (&v)[N]) {
        static_assert(N % 2 == 0, "pairs");
        if constexpr (N % 4 == 0) {
#pragma unroll
            for (int k = 0; k < N / 4; ++k) {
                const float4 q = reinterpret_cast<const float4 *>(p)[k];
                v[4 * k] = q.x; v[4 * k + 1] = q.y; v[4 * k + 2] = q.z; v[4 * k + 3] = q.w;
            }
        } else {
#pragma unroll
            for (int k = 0; k < N / 2; ++k) {
                const float2 q = reinterpret_cast<const float2 *>(p)[k];
                v[2 * k] = q.x; v[2 * k + 1] = q.y;
            }
        }
    }
};
template <int N> struct Vec<__nv_bfloat16, N> {
    static __device__ __forceinline__ void load(const __nv_bfloat16 *p, float (&v)[N]) {
        static_assert(N % 2 == 0, "pairs");
        if constexpr (N % 4 == 0) {
#pragma unroll
            for (int k = 0; k < N / 4; ++k) {
                const uint2 q = reinterpret_cast<const uint2 *>(p)[k];
                v[4 * k] = __uint_as_float(q.x << 16);
                v[4 * k + 1] = __uint_as_float(q.x & 0xFFFF0000u);
                v[4 * k + 2] = __uint_as_float(q.y << 16);
                v[4 * k + 3] = __uint_as_float(q.y & 0xFFFF0000u);
            }
        } else {
#pragma unroll
            for (int k = 0; k < N / 2; ++k) {
                const uint32_t q = reinterpret_cast<const uint32_t *>(p)[k];
                v[2 * k] = __uint_as_float(q << 16);
                v[2 * k + 1] = __uint_as_float(q & 0xFFFF0000u);
            }
        }
    }
};

// Compile-time geometry of one instantiation.
template <typename T, int SPL, int L, int MODE, int RL>
struct Geo {
    static constexpr int CH = SCAN_THREADS / L;              // channels per CTA
    static constexpr int V = 16 / (int)sizeof(T);            // elements per 16 B
    static constexpr int SPP = ((L * SPL + V - 1) / V) * V;  // padded B/C row
    static constexpr int RP = ((L * RL + V - 1) / V) * V;    // padded dt_low row
    static constexpr int NX = SCAN_TC * CH;
    static constexpr int NBC = SCAN_TC * SPP;
    static constexpr int NDL = MODE == FUSED ? SCAN_TC * RP : 0;
    static constexpr int NZ = MODE == GATED ? NX : 0;
    // x | dt (PLAIN, GATED) or z (FUSED) | B | C | dt_low (FUSED) or z (GATED)
    static constexpr int ELEMS = 2 * NX + 2 * NBC + NDL + NZ;
    // after the two stages: per-lane partial y (SCAN_TC x 128 floats) and, in
    // FUSED mode, the chunk's dt tile (SCAN_TC x CH floats)
    static constexpr size_t BYTES = 2 * (size_t)ELEMS * sizeof(T) +
                                    (size_t)SCAN_TC * SCAN_THREADS * sizeof(float) +
                                    (MODE != PLAIN ? (size_t)SCAN_TC * CH * sizeof(float) : 0);
};

// 6 CTAs per SM (registers <= 80) where dt is given; the fused kernel keeps
// W_dt's row slice in registers and needs the 128 of 4 CTAs per SM
template <typename T, int SPL, int L, int MODE, int RL>
__global__ void __launch_bounds__(SCAN_THREADS, MODE == FUSED ? 4 : 6)
scan_kernel(const ScanParams p) {
    using Gm = Geo<T, SPL, L, MODE, RL>;
    constexpr int CH = Gm::CH;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T *stage0 = reinterpret_cast<T *>(smem_raw);
    float *ys = reinterpret_cast<float *>(smem_raw + 2 * (size_t)Gm::ELEMS * sizeof(T));
    float *dts = ys + SCAN_TC * SCAN_THREADS;   // FUSED, GATED: dt of the chunk, [tt][channel]

    const int tid = threadIdx.x;
    const int c = tid / L;          // channel within CTA
    const int j = tid % L;          // lane within the channel's group
    const int nseg = p.nseg > 1 ? p.nseg : 1;
    // the summary pass skips each sequence's last segment (nothing needs its
    // summary: the output pass runs it from its start state to the final state)
    const int gsegs = (MODE == SUMMARY && nseg > 1) ? nseg - 1 : nseg;
    const int b = blockIdx.y / gsegs;
    const int g = blockIdx.y - b * gsegs;             // T segment
    const int64_t tb = (int64_t)g * p.seg_len;        // first step of the segment
    int64_t tl = nseg > 1 ? p.seqlen - tb : p.seqlen;
    if (nseg > 1 && tl > p.seg_len) tl = p.seg_len;
    if (tl < 0) tl = 0;
    const int64_t segidx = (int64_t)b * nseg + g;
    const int64_t d0 = (int64_t)blockIdx.x * CH;
    const int64_t d = d0 + c;
    const bool active = d < p.d_inner;
    const int S = p.d_state;
    const int T_ = (int)tl;
    const int ch_valid = (int)((p.d_inner - d0 < CH) ? p.d_inner - d0 : CH);

    static_assert(SPL % 2 == 0 && (RL % 2 == 0 || RL == 1), "states / dt_rank slices come in pairs");
    constexpr int NP = SPL / 2;
    f2 A2[NP], h[NP];
#pragma unroll
    for (int q = 0; q < NP; ++q) {
        float a[2] = {0.0f, 0.0f}, hi[2] = {0.0f, 0.0f};
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int s = j * SPL + 2 * q + e;
            if (active && s < S) {
                if (MODE != PLAIN)
                    a[e] = -expf(io<T>::to_f(static_cast<const T *>(p.A)[d * S + s]));
                else
                    a[e] = static_cast<const float *>(p.A)[d * S + s];
                if (p.seg_hstart)
                    hi[e] = p.seg_hstart[(segidx * p.d_inner + d) * S + s];
                else if (p.h0 && MODE != SUMMARY)
                    hi[e] = p.h0[((int64_t)b * p.d_inner + d) * S + s];
            }
        }
        A2[q] = pk(a[0] * kLog2e, a[1] * kLog2e);
        h[q] = pk(hi[0], hi[1]);
    }
    // FUSED: this lane's slice of W_dt[d, :] (as pairs) and the bias
    constexpr int RP2 = MODE == FUSED ? RL / 2 : 1;
    f2 wdt[RP2];
    float bias_dt = 0.0f;
    if (MODE == FUSED) {
#pragma unroll
        for (int q = 0; q < RP2; ++q) {
            float w[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int rr = j * RL + 2 * q + e;
                w[e] = (active && rr < p.dt_rank)
                           ? io<T>::to_f(static_cast<const T *>(p.w_dt)[d * p.dt_rank + rr]) : 0.0f;
            }
            wdt[q] = pk(w[0], w[1]);
        }
        if (active && p.b_dt) bias_dt = io<T>::to_f(static_cast<const T *>(p.b_dt)[d]);
    }

    const int64_t row_base = (int64_t)b * p.seqlen + tb;
    const T *xg = static_cast<const T *>(p.x) + row_base * p.ld_x + d0;
    const T *d2g = MODE == FUSED ? static_cast<const T *>(p.z) + row_base * p.ld_z + d0
                                 : static_cast<const T *>(p.dt) + row_base * p.ld_dt + d0;
    const int64_t ld_d2 = MODE == FUSED ? p.ld_z : p.ld_dt;
    const T *bg = static_cast<const T *>(p.bm) + row_base * p.ld_b;
    const T *cg = static_cast<const T *>(p.cm) + row_base * p.ld_c;
    const T *dlg = MODE == FUSED ? static_cast<const T *>(p.dl) + row_base * p.ld_dl : nullptr;
    const T *zg = MODE == GATED ? static_cast<const T *>(p.z) + row_base * p.ld_z + d0 : nullptr;

    auto issue = [&](int chunk) {
        T *st = stage0 + (chunk & 1) * Gm::ELEMS;
        const int64_t t0 = (int64_t)chunk * SCAN_TC;
        const int rv = min(SCAN_TC, T_ - (int)t0);
        stage_rows<T, SCAN_TC, CH>(st, xg + t0 * p.ld_x, p.ld_x, rv, ch_valid,
                                   p.vec16 & ARR_X, tid);
        stage_rows<T, SCAN_TC, CH>(st + Gm::NX, d2g + t0 * ld_d2, ld_d2, rv, ch_valid,
                                   p.vec16 & ARR_D2, tid);
        stage_rows<T, SCAN_TC, Gm::SPP>(st + 2 * Gm::NX, bg + t0 * p.ld_b, p.ld_b, rv, S,
                                        p.vec16 & ARR_B, tid);
        if (MODE != SUMMARY)   // C only enters y
            stage_rows<T, SCAN_TC, Gm::SPP>(st + 2 * Gm::NX + Gm::NBC, cg + t0 * p.ld_c, p.ld_c,
                                            rv, S, p.vec16 & ARR_C, tid);
        if (MODE == FUSED)
            stage_rows<T, SCAN_TC, Gm::RP>(st + 2 * Gm::NX + 2 * Gm::NBC, dlg + t0 * p.ld_dl,
                                           p.ld_dl, rv, p.dt_rank, p.vec16 & ARR_DL, tid);
        if (MODE == GATED)
            stage_rows<T, SCAN_TC, CH>(st + 2 * Gm::NX + 2 * Gm::NBC, zg + t0 * p.ld_z, p.ld_z,
                                       rv, ch_valid, p.vec16 & ARR_Z, tid);
    };

    // read-out geometry: thread owns column cc of rows rr0, rr0 + 128/CH, ...
    constexpr int RSTEP = SCAN_THREADS / CH;
    const int cc = tid % CH, rr0 = tid / CH;
    const bool col_ok = cc < ch_valid;
    float d_skip = 0.0f;
    if (col_ok && p.D)
        d_skip = MODE != PLAIN ? io<T>::to_f(static_cast<const T *>(p.D)[d0 + cc])
                               : static_cast<const float *>(p.D)[d0 + cc];
    T *yg = static_cast<T *>(p.y) + row_base * p.ld_y + d0 + cc;

    const int nchunks = (T_ + SCAN_TC - 1) / SCAN_TC;
    // dt rows that hold softplus(dt) already: given so, or written back by
    // this segment's summary pass
    const bool dt_ready = p.dt_act || (MODE == GATED && p.dt_wb && nseg > 1 && g < nseg - 1);
    T *dt_back = (MODE == SUMMARY && p.dt_wb && !p.dt_act)
                     ? const_cast<T *>(static_cast<const T *>(p.dt)) + row_base * p.ld_dt + d
                     : nullptr;
    float sdt = 0.0f;                                  // sum of this channel's dt (pass 1)
    float ymax = 0.0f;                                 // max |y| written by this thread
    if (nchunks > 0) issue(0);
    cp_async_commit();

    for (int ch = 0; ch < nchunks; ++ch) {
        if (ch + 1 < nchunks) issue(ch + 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const T *st = stage0 + (ch & 1) * Gm::ELEMS;
        const T *xs = st + c;
        const T *d2s = st + Gm::NX + c;
        const T *bs = st + 2 * Gm::NX + j * SPL;
        const T *cs = bs + Gm::NBC;
        const T *dls = st + 2 * Gm::NX + 2 * Gm::NBC + j * RL;
        const int tn = min(SCAN_TC, T_ - ch * SCAN_TC);

        if (MODE == FUSED) {
            // ---- dt of the whole chunk: 16 independent dot products per lane
            // (rows >= tn are zero-filled and never used), shuffle-reduced over
            // the channel's L lanes; lane j finishes steps j, j + L, ... with
            // bias + softplus, so each token-channel's softplus runs once.
            constexpr int HALF = SCAN_TC / 2;     // two passes of 8 independent chains
#pragma unroll 1
            for (int t0 = 0; t0 < SCAN_TC; t0 += HALF) {
                float part[HALF];
#pragma unroll
                for (int u = 0; u < HALF; ++u) {
                    float dlv[RL > 1 ? RL : 4];
                    Vec<T, (RL > 1 ? RL : 4)>::load(dls + (t0 + u) * Gm::RP, dlv);
                    f2 acc = pk(0.0f, 0.0f);
#pragma unroll
                    for (int q = 0; q < RP2; ++q)
                        acc = fma2(pk(dlv[2 * q], dlv[2 * q + 1]), wdt[q], acc);
                    float pa, pb;
                    upk(acc, pa, pb);
                    part[u] = pa + pb;
                }
#pragma unroll
                for (int u = 0; u < HALF; ++u)
#pragma unroll
                    for (int m = 1; m < L; m <<= 1)
                        part[u] += __shfl_xor_sync(0xffffffffu, part[u], m);
#pragma unroll
                for (int k = 0; k < HALF; k += (L < HALF ? L : HALF)) {
                    float v = part[k];
#pragma unroll
                    for (int l = 1; l < L && k + l < HALF; ++l) v = (j == l) ? part[k + l] : v;
                    if (L <= HALF || j < HALF)
                        dts[(t0 + k + j) * CH + c] = io<T>::round(softplus_f(io<T>::round(v + bias_dt)));
                }
            }
            __syncwarp();   // a channel's L lanes share one warp
        }
        if (MODE == GATED || MODE == SUMMARY) {
            // ---- dt = softplus(dt_proj output) once per token-channel: lane j
            // takes steps j, j + L, ... (rows >= tn are zero-filled, unused)
#pragma unroll
            for (int tt = j; tt < SCAN_TC; tt += L) {
                const float v = io<T>::to_f(d2s[tt * CH]);
                const float dv = dt_ready ? v : io<T>::round(softplus_f(v));
                dts[tt * CH + c] = dv;
                if (dt_back && active && tt < tn)
                    dt_back[((int64_t)ch * SCAN_TC + tt) * p.ld_dt] = io<T>::from_f(dv);
            }
            __syncwarp();   // a channel's L lanes share one warp
        }
        // ---- recurrence (tn is CTA-uniform)
#pragma unroll 8
        for (int tt = 0; tt < tn; ++tt) {
            const float dtv = MODE != PLAIN ? dts[tt * CH + c] : io<T>::to_f(d2s[tt * CH]);
            if (MODE == SUMMARY) sdt += dtv;
            const float dtx = dtv * io<T>::to_f(xs[tt * CH]);
            const f2 dt2 = pk(dtv, dtv), dtx2 = pk(dtx, dtx);
            float bv[SPL], cv[SPL];
            Vec<T, SPL>::load(bs + tt * Gm::SPP, bv);
            Vec<T, SPL>::load(cs + tt * Gm::SPP, cv);
            f2 ya = pk(0.0f, 0.0f), yb = ya;
#pragma unroll
            for (int q = 0; q < NP; ++q) {
                float e0, e1;
                upk(mul2(dt2, A2[q]), e0, e1);
                const f2 dA = pk(ex2(e0), ex2(e1));
                h[q] = fma2(dA, h[q], mul2(dtx2, pk(bv[2 * q], bv[2 * q + 1])));
                if (MODE != SUMMARY) {
                    if (q & 1) yb = fma2(h[q], pk(cv[2 * q], cv[2 * q + 1]), yb);
                    else ya = fma2(h[q], pk(cv[2 * q], cv[2 * q + 1]), ya);
                }
            }
            if (MODE != SUMMARY) {
                float y0, y1, y2, y3;
                upk(ya, y0, y1);
                upk(yb, y2, y3);
                ys[tt * SCAN_THREADS + tid] = (y0 + y1) + (y2 + y3);
            }
        }
        __syncthreads();
        // ---- read-out: sum lane partials, D skip, (FUSED) cast + SiLU(z) gate
        const T *xrow = st + cc;
        const T *zrow = st + (MODE == FUSED ? Gm::NX : 2 * Gm::NX + 2 * Gm::NBC) + cc;
        if (MODE != SUMMARY && col_ok) {
#pragma unroll 4
            for (int tt = rr0; tt < tn; tt += RSTEP) {
                float yv = 0.0f;
#pragma unroll
                for (int l = 0; l < L; ++l) yv += ys[tt * SCAN_THREADS + cc * L + l];
                float out = yv + d_skip * io<T>::to_f(xrow[tt * CH]);
                if (MODE != PLAIN) {
                    const float zv = io<T>::to_f(zrow[tt * CH]);
                    out = io<T>::round(out) * (p.z_act ? zv : io<T>::round(silu_f(zv)));
                }
                ymax = fmaxf(ymax, fabsf(out));
                yg[((int64_t)ch * SCAN_TC + tt) * p.ld_y] = io<T>::from_f(out);
            }
        }
        __syncthreads();
    }
    cp_async_wait<0>();
    // final state: of the segment (pass 1), or of the sequence, which the
    // sequence's last segment (the whole sequence without segments) ends in
    float *hout = MODE == SUMMARY ? p.seg_hend + segidx * p.d_inner * S
                            : ((g == nseg - 1 && p.h_last) ? p.h_last + (int64_t)b * p.d_inner * S
                                                           : nullptr);
    if (hout && active) {
#pragma unroll
        for (int q = 0; q < NP; ++q) {
            float hv[2];
            upk(h[q], hv[0], hv[1]);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int s = j * SPL + 2 * q + e;
                if (s < S) hout[d * S + s] = hv[e];
            }
        }
        if (MODE == SUMMARY && j == 0) p.seg_sdt[segidx * p.d_inner + d] = sdt;
    }
    if (MODE != SUMMARY && p.amax) amax_publish(p.amax, ymax);   // launch-uniform branch
}

// Segments' carry (between pass 1 and pass 3): per (b, d, s), in segment
// order, start(g) = h, then h = exp(A sum(dt_g)) h + h_end(g) -- the product of
// the segment's per-step decays exp(dt_t A) is the exponential of A times the
// sum of its dt.  Only the start states are needed: the last segment has no
// summary, and pass 3 runs it from its start state to the sequence's final
// state.  A: fp32 (PLAIN) or A_log in T (A = -exp(A_log)).
template <typename T, bool A_F32>
__global__ void seg_carry_kernel(const void *A, const float *__restrict__ h0,
                                 const float *__restrict__ hend, const float *__restrict__ sdt,
                                 float *__restrict__ hstart, int64_t batch, int64_t di, int S,
                                 int nseg) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= batch * di * S) return;
    const int64_t s = i % S, bd = i / S;
    const int64_t d = bd % di, b = bd / di;
    const float a = A_F32 ? static_cast<const float *>(A)[d * S + s]
                          : -expf(io<T>::to_f(static_cast<const T *>(A)[d * S + s]));
    const float a2 = a * kLog2e;
    float hv = h0 ? h0[i] : 0.0f;
    for (int g = 0; g < nseg; ++g) {
        const int64_t idx = (b * nseg + g) * di + d;
        hstart[idx * S + s] = hv;
        if (g + 1 < nseg) hv = fmaf(ex2(a2 * sdt[idx]), hv, hend[idx * S + s]);
    }
}

// -------------------------------------------------------------- dispatch ---
static bool rows16(const void *p, int64_t ld, size_t es) {
    return aligned(p, 16) && (ld * (int64_t)es) % 16 == 0;
}

template <typename T, int SPL, int L, int MODE, int RL>
static int launch_scan(ScanParams p, cudaStream_t st) {
    using Gm = Geo<T, SPL, L, MODE, RL>;
    auto kern = scan_kernel<T, SPL, L, MODE, RL>;
    if (Gm::BYTES > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)Gm::BYTES);
        if (e != cudaSuccess) return fail(MB2_ERR_CUDA, "scan: smem attribute: %s", cudaGetErrorString(e));
    }
    const size_t es = sizeof(T);
    const bool ch16 = (Gm::CH * es) % 16 == 0;     // x / z tiles start at d0 = k * CH
    p.vec16 = 0;
    if (ch16 && rows16(p.x, p.ld_x, es)) p.vec16 |= ARR_X;
    if (MODE == FUSED ? (ch16 && rows16(p.z, p.ld_z, es)) : (ch16 && rows16(p.dt, p.ld_dt, es)))
        p.vec16 |= ARR_D2;
    if (MODE == GATED && ch16 && rows16(p.z, p.ld_z, es)) p.vec16 |= ARR_Z;
    if (rows16(p.bm, p.ld_b, es)) p.vec16 |= ARR_B;
    if (rows16(p.cm, p.ld_c, es)) p.vec16 |= ARR_C;
    if (MODE == FUSED && rows16(p.dl, p.ld_dl, es)) p.vec16 |= ARR_DL;
    const int gsegs = p.nseg > 1 ? (MODE == SUMMARY ? p.nseg - 1 : p.nseg) : 1;
    dim3 grid((unsigned)ceil_div(p.d_inner, Gm::CH), (unsigned)(p.batch * gsegs));
    kern<<<grid, SCAN_THREADS, Gm::BYTES, st>>>(p);
    return check_launch("scan_kernel");
}

// (SPL, L) by d_state; RL (dt_rank slice per lane, FUSED only) by dt_rank.
template <typename T, int MODE, int SPL, int L>
static int dispatch_rl(const ScanParams &p, cudaStream_t st) {
    if constexpr (MODE != FUSED) {
        return launch_scan<T, SPL, L, MODE, 1>(p, st);
    } else {
        const int per = (p.dt_rank + L - 1) / L;
        if (per <= 8) return launch_scan<T, SPL, L, FUSED, 8>(p, st);
        if (per <= 16) return launch_scan<T, SPL, L, FUSED, 16>(p, st);
        if (per <= 24) return launch_scan<T, SPL, L, FUSED, 24>(p, st);
        if (per <= 32) return launch_scan<T, SPL, L, FUSED, 32>(p, st);
        if (per <= 48) return launch_scan<T, SPL, L, FUSED, 48>(p, st);
        if (per <= 64) return launch_scan<T, SPL, L, FUSED, 64>(p, st);
        return fail(MB2_ERR_UNSUPPORTED, "scan: dt_rank %d too large for d_state %d (max %d)",
                    p.dt_rank, p.d_state, 64 * L);
    }
}

// Lanes per channel: each (batch, channel) chain -- per T segment when the
// sequence is cut -- is walked by L lanes holding SPL = S / L states each, 8
// to 16 states per lane, so that a lane's per-step overhead (its dt, x and y)
// is shared by many states.  (Shapes with few chains keep this split and run
// in T segments: measured on config 1's shapes, 4 or 8 lanes of 4 or 2
// states and no segments were 6-11 % slower than 2 lanes in 7 segments.)
static int scan_lanes(int S) { return S <= 8 ? 1 : S <= 32 ? 2 : S <= 64 ? 4 : S <= 128 ? 8 : 16; }

// (SPL, L) by d_state.
template <typename T, int MODE>
static int dispatch_scan(const ScanParams &p, cudaStream_t st) {
    const int S = p.d_state;
    if (S <= 8) return dispatch_rl<T, MODE, 8, 1>(p, st);
    if (S <= 16) return dispatch_rl<T, MODE, 8, 2>(p, st);
    if (S <= 24) return dispatch_rl<T, MODE, 12, 2>(p, st);
    if (S <= 32) return dispatch_rl<T, MODE, 16, 2>(p, st);
    if (S <= 64) return dispatch_rl<T, MODE, 16, 4>(p, st);
    if (S <= 128) return dispatch_rl<T, MODE, 16, 8>(p, st);
    return dispatch_rl<T, MODE, 16, 16>(p, st);
}

// bf16 staging copies 4-byte words: every row must start on a 4-byte boundary.
static int check_rows(int dtype, const void *ptr, int64_t ld, int64_t cols, const char *name) {
    MB2_REQUIRE(ld >= cols, MB2_ERR_SHAPE, "scan: leading dimension of %s too small", name);
    if (dtype == MB2_BF16)
        MB2_REQUIRE(aligned(ptr, 4) && ld % 2 == 0, MB2_ERR_ALIGN,
                    "scan(bf16): %s rows must start on 4-byte boundaries (even offsets and "
                    "leading dimension)", name);
    return MB2_OK;
}

int scan_fused(int dtype, const void *xc, int64_t ld_xc, const void *dl, int64_t ld_dl,
               const void *bm, int64_t ld_b, const void *cm, int64_t ld_c, const void *z,
               int64_t ld_z, const void *w_dt, const void *b_dt, const void *A_log,
               const void *D, const float *h0, float *h_last, void *y, int64_t ld_y,
               int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state, int64_t dt_rank,
               cudaStream_t stream, unsigned *amax, int act) {
    MB2_REQUIRE(dtype == MB2_F32 || dtype == MB2_BF16, MB2_ERR_ARG, "scan: bad dtype");
    MB2_REQUIRE(batch >= 0 && seqlen >= 0 && d_inner >= 0 && dt_rank >= 1, MB2_ERR_SHAPE,
                "scan: bad sizes");
    MB2_REQUIRE(d_state >= 1 && d_state <= 256, MB2_ERR_SHAPE,
                "d_state > 256 not supported (got %lld)", (long long)d_state);
    MB2_REQUIRE(batch < 65536, MB2_ERR_SHAPE, "scan: batch too large");
    if (batch == 0 || d_inner == 0) return MB2_OK;
    MB2_REQUIRE(A_log && w_dt && (seqlen == 0 || (xc && dl && bm && cm && z && y)), MB2_ERR_ARG,
                "scan: null pointer");
    if (dtype == MB2_BF16)
        MB2_REQUIRE(d_inner % 2 == 0, MB2_ERR_ALIGN, "scan(bf16): d_inner must be even");
    MB2_TRY(check_rows(dtype, xc, ld_xc, d_inner, "x"));
    MB2_TRY(check_rows(dtype, z, ld_z, d_inner, "z"));
    MB2_TRY(check_rows(dtype, bm, ld_b, d_state, "B"));
    MB2_TRY(check_rows(dtype, cm, ld_c, d_state, "C"));
    MB2_TRY(check_rows(dtype, dl, ld_dl, dt_rank, "dt_low"));
    MB2_REQUIRE(ld_y >= d_inner, MB2_ERR_SHAPE, "scan: leading dimension of y too small");
    ScanParams p{};
    p.x = xc; p.ld_x = ld_xc;
    p.z = z; p.ld_z = ld_z;
    p.bm = bm; p.ld_b = ld_b;
    p.cm = cm; p.ld_c = ld_c;
    p.dl = dl; p.ld_dl = ld_dl;
    p.w_dt = w_dt; p.b_dt = b_dt;
    p.A = A_log; p.D = D; p.h0 = h0; p.h_last = h_last;
    p.y = y; p.ld_y = ld_y;
    p.batch = batch; p.seqlen = seqlen; p.d_inner = d_inner;
    p.d_state = (int)d_state; p.dt_rank = (int)dt_rank;
    p.amax = amax;
    p.z_act = (act & SCAN_Z_ACT) != 0;
    if (dtype == MB2_F32) return dispatch_scan<float, FUSED>(p, stream);
    return dispatch_scan<__nv_bfloat16, FUSED>(p, stream);
}

// ------------------------------------------------------- T segments (host) --
int scan_segments(int64_t batch, int64_t d_inner, int64_t seqlen, int64_t d_state) {
    // few independent (batch, channel) chains leave most SMs idle while each
    // walks a long sequence: cut T into segments until about 148 x 1024
    // threads (8 CTAs per SM on a B200) are busy, segments >= 256 steps
    const int64_t threads = batch * d_inner * scan_lanes((int)d_state);
    const int64_t target = (int64_t)148 * 1024;
    if (threads <= 0 || threads * 2 > target) return 1;
    int64_t g = ceil_div(target, threads);
    const int64_t gmax = seqlen / 256;
    g = g < gmax ? g : gmax;
    g = g < 64 ? g : 64;
    return g >= 2 ? (int)g : 1;
}

size_t scan_segment_bytes(int64_t batch, int64_t d_inner, int64_t seqlen, int64_t d_state) {
    const int nseg = scan_segments(batch, d_inner, seqlen, d_state);
    if (nseg <= 1) return 0;
    return (size_t)batch * nseg * d_inner * (2 * d_state + 1) * sizeof(float);
}

// Pass 1 (segment summaries), carry, pass 3 (outputs).
template <typename T, int MODE>
static int run_segmented(ScanParams p, int nseg, float *ws, cudaStream_t st) {
    const int64_t S = p.d_state;
    p.seg_len = round_up(ceil_div(p.seqlen, (int64_t)nseg), (int64_t)SCAN_TC);
    p.nseg = (int)ceil_div(p.seqlen, p.seg_len);
    if (p.nseg < 2) {                    // rounding left one segment: run it whole
        p.nseg = 0;
        return dispatch_scan<T, MODE>(p, st);
    }
    const int64_t nstates = p.batch * p.nseg * p.d_inner * S;
    float *hend = ws, *hstart = ws + nstates, *sdt = ws + 2 * nstates;
    static_assert(MODE == GATED, "segments are run for the gated scan");
    p.seg_hend = hend; p.seg_sdt = sdt; p.seg_hstart = nullptr;
    MB2_TRY((dispatch_scan<T, SUMMARY>(p, st)));
    const int64_t n = p.batch * p.d_inner * S;
    seg_carry_kernel<T, MODE == PLAIN><<<(unsigned)ceil_div(n, (int64_t)256), 256, 0, st>>>(
        p.A, p.h0, hend, sdt, hstart, p.batch, p.d_inner, (int)S, p.nseg);
    MB2_TRY(check_launch("seg_carry_kernel"));
    p.seg_hstart = hstart;
    return dispatch_scan<T, MODE>(p, st);
}

// The block forward's scan stage given dt_proj's output (dt_low W_dt^T + b_dt,
// from the tensor-core GEMM): dt = softplus(.), A = -exp(A_log), recurrence,
// D skip, cast and SiLU(z) gate.
int scan_gated(int dtype, const void *xc, int64_t ld_xc, const void *dt, int64_t ld_dt,
               const void *bm, int64_t ld_b, const void *cm, int64_t ld_c, const void *z,
               int64_t ld_z, const void *A_log, const void *D, const float *h0, float *h_last,
               void *y, int64_t ld_y, int64_t batch, int64_t seqlen, int64_t d_inner,
               int64_t d_state, cudaStream_t stream, float *seg_ws, size_t seg_bytes,
               unsigned *amax, int act) {
    MB2_REQUIRE(dtype == MB2_F32 || dtype == MB2_BF16, MB2_ERR_ARG, "scan: bad dtype");
    MB2_REQUIRE(batch >= 0 && seqlen >= 0 && d_inner >= 0, MB2_ERR_SHAPE, "scan: bad sizes");
    MB2_REQUIRE(d_state >= 1 && d_state <= 256, MB2_ERR_SHAPE,
                "d_state > 256 not supported (got %lld)", (long long)d_state);
    MB2_REQUIRE(batch < 65536, MB2_ERR_SHAPE, "scan: batch too large");
    if (batch == 0 || d_inner == 0) return MB2_OK;
    MB2_REQUIRE(A_log && (seqlen == 0 || (xc && dt && bm && cm && z && y)), MB2_ERR_ARG,
                "scan: null pointer");
    if (dtype == MB2_BF16)
        MB2_REQUIRE(d_inner % 2 == 0, MB2_ERR_ALIGN, "scan(bf16): d_inner must be even");
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
    p.amax = amax;
    p.dt_act = (act & SCAN_DT_ACT) != 0;
    p.z_act = (act & SCAN_Z_ACT) != 0;
    p.dt_wb = (act & SCAN_DT_SCRATCH) != 0;
    const int nseg = scan_segments(batch, d_inner, seqlen, d_state);
    if (nseg > 1 && seg_ws && seg_bytes >= scan_segment_bytes(batch, d_inner, seqlen, d_state)) {
        if (dtype == MB2_F32) return run_segmented<float, GATED>(p, nseg, seg_ws, stream);
        return run_segmented<__nv_bfloat16, GATED>(p, nseg, seg_ws, stream);
    }
    if (dtype == MB2_F32) return dispatch_scan<float, GATED>(p, stream);
    return dispatch_scan<__nv_bfloat16, GATED>(p, stream);
}

// ------------------------------------------------------ single-token step ---
// The decode step's dt_proj, softplus and state update in one kernel
// (_mamba.py:146-163).  A CTA takes a tile of 8 sequences x 32 channels and
// stages the 8 dt_low rows, the 32 rows of W_dt and the 8 B and C rows in
// shared memory (each W_dt row is read once per 8 sequences).  Phase 1: each
// of its 256 threads forms one (sequence b, channel d)'s dt = softplus(dt_low[b]
// . W_dt[d] + b_dt[d]) as an fp32 dot product in a fixed order (rounded to T
// where the reference's bf16 linear output is).  Phase 2: QS = S / 4 threads
// per (b, d) advance h[b, d, :] in place, 4 states each in one 16-byte load
// and store (a warp moves 512 contiguous bytes of h), y = C.h summed by
// shuffles, + D x, cast, times SiLU(z).
constexpr int SDT_B = 8, SDT_D = 32, SDT_THREADS = 256;

template <typename T, int QS>
__global__ void __launch_bounds__(SDT_THREADS)
step_scan_dt_kernel(const T *__restrict__ xc, int64_t ld_x, const T *__restrict__ dl,
                    int64_t ld_dl, const T *__restrict__ w_dt, const T *__restrict__ b_dt,
                    const T *__restrict__ bm, const T *__restrict__ cm, int64_t ld_bc,
                    const T *__restrict__ z, int64_t ld_z, const T *__restrict__ A_log,
                    const T *__restrict__ D, float *__restrict__ h, T *__restrict__ y,
                    int64_t ld_y, int64_t batch, int64_t di, int R) {
    constexpr int S = 4 * QS;
    extern __shared__ float sdt_smem[];
    const int RP = R + 1;                       // odd row pitch: W_dt rows conflict-free
    float *dts = sdt_smem;                      // [SDT_B][SDT_D] dt of the tile
    float *bs = dts + SDT_B * SDT_D;            // [SDT_B][S]
    float *cs = bs + SDT_B * S;                 // [SDT_B][S]
    float *dls = cs + SDT_B * S;                // [SDT_B][R]
    float *ws = dls + SDT_B * R;                // [SDT_D][RP]
    const int64_t d0 = (int64_t)blockIdx.x * SDT_D, b0 = (int64_t)blockIdx.y * SDT_B;
    const int tid = threadIdx.x;
    // this thread's QS (b, d) pairs of phase 2 (pairs pi = tid / QS + k PAIRS,
    // channels fastest): their state, x and z are loaded first, so those
    // loads overlap the staging and the dt dot products
    constexpr int PAIRS = SDT_THREADS / QS;
    const int q = tid % QS;
    float4 hv[QS];
    float xv[QS], zv[QS];
#pragma unroll
    for (int k = 0; k < QS; ++k) {
        const int pi = tid / QS + k * PAIRS;
        const int bl = pi / SDT_D, dd = pi - bl * SDT_D;
        const int64_t b = b0 + bl, d = d0 + dd;
        const bool ok = b < batch && d < di;
        hv[k] = ok ? *reinterpret_cast<const float4 *>(h + (b * di + d) * S + 4 * q)
                   : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        xv[k] = ok ? io<T>::to_f(xc[b * ld_x + d]) : 0.0f;
        zv[k] = ok ? io<T>::to_f(z[b * ld_z + d]) : 0.0f;
    }
    for (int i = tid; i < SDT_D * R; i += SDT_THREADS) {
        const int dd = i / R, r = i - dd * R;
        ws[dd * RP + r] = d0 + dd < di ? io<T>::to_f(w_dt[(d0 + dd) * R + r]) : 0.0f;
    }
    // dt_low, B and C come from the kernel before this one in the decode
    // step's chain (x_proj's reduction); the state, x, z and W_dt above are
    // older (common.cuh, pdl_wait)
    pdl_wait();
    pdl_trigger();
    for (int i = tid; i < SDT_B * R; i += SDT_THREADS) {
        const int bl = i / R, r = i - bl * R;
        dls[i] = b0 + bl < batch ? io<T>::to_f(dl[(b0 + bl) * ld_dl + r]) : 0.0f;
    }
    for (int i = tid; i < SDT_B * S; i += SDT_THREADS) {
        const int bl = i / S, sidx = i - bl * S;
        const bool ok = b0 + bl < batch;
        bs[i] = ok ? io<T>::to_f(bm[(b0 + bl) * ld_bc + sidx]) : 0.0f;
        cs[i] = ok ? io<T>::to_f(cm[(b0 + bl) * ld_bc + sidx]) : 0.0f;
    }
    __syncthreads();
    {   // phase 1: one dt per thread, the dot product as four interleaved sums
        const int bl = tid / SDT_D, dd = tid - bl * SDT_D;
        const int64_t d = d0 + dd;
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        const float *dlr = dls + bl * R, *wr = ws + dd * RP;
        int r = 0;
        for (; r + 4 <= R; r += 4) {
            a0 = fmaf(dlr[r], wr[r], a0);
            a1 = fmaf(dlr[r + 1], wr[r + 1], a1);
            a2 = fmaf(dlr[r + 2], wr[r + 2], a2);
            a3 = fmaf(dlr[r + 3], wr[r + 3], a3);
        }
        for (; r < R; ++r) a0 = fmaf(dlr[r], wr[r], a0);
        const float acc = (a0 + a1) + (a2 + a3);
        const float pre = io<T>::round(acc + ((b_dt && d < di) ? io<T>::to_f(b_dt[d]) : 0.0f));
        dts[tid] = io<T>::round(softplus_f(pre));
    }
    __syncthreads();
    // phase 2: QS threads per (b, d), 4 states each
#pragma unroll
    for (int k = 0; k < QS; ++k) {
        const int pi = tid / QS + k * PAIRS;
        const int bl = pi / SDT_D, dd = pi - bl * SDT_D;
        const int64_t b = b0 + bl, d = d0 + dd;
        const bool ok = b < batch && d < di;          // every lane joins the shuffles below
        float yv = 0.0f;
        if (ok) {
            const float dt = dts[pi], x = xv[k];
            const int s0 = 4 * q;
            float hs[4] = {hv[k].x, hv[k].y, hv[k].z, hv[k].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float a = -expf(io<T>::to_f(A_log[d * S + s0 + e])) * kLog2e;
                hs[e] = fmaf(ex2(dt * a), hs[e], (dt * bs[bl * S + s0 + e]) * x);
                yv = fmaf(hs[e], cs[bl * S + s0 + e], yv);
            }
            *reinterpret_cast<float4 *>(h + (b * di + d) * S + s0) =
                make_float4(hs[0], hs[1], hs[2], hs[3]);
        }
#pragma unroll
        for (int o = QS / 2; o > 0; o >>= 1) yv += __shfl_xor_sync(0xffffffffu, yv, o);
        if (ok && q == 0) {
            float out = yv + (D ? io<T>::to_f(D[d]) : 0.0f) * xv[k];
            out = io<T>::round(out) * io<T>::round(silu_f(zv[k]));
            y[b * ld_y + d] = io<T>::from_f(out);
        }
    }
}

// One (b, d) per thread for d_state not of the form 4 x 2^k or without 16-byte
// aligned h rows: the same computation with the state row walked in place.
template <typename T>
__global__ void __launch_bounds__(SDT_THREADS)
step_scan_dt_any_kernel(const T *__restrict__ xc, int64_t ld_x, const T *__restrict__ dl,
                        int64_t ld_dl, const T *__restrict__ w_dt, const T *__restrict__ b_dt,
                        const T *__restrict__ bm, const T *__restrict__ cm, int64_t ld_bc,
                        const T *__restrict__ z, int64_t ld_z, const T *__restrict__ A_log,
                        const T *__restrict__ D, float *__restrict__ h, T *__restrict__ y,
                        int64_t ld_y, int64_t batch, int64_t di, int S, int R) {
    pdl_wait();
    pdl_trigger();
    const int64_t b = (int64_t)blockIdx.y * SDT_B + threadIdx.x / SDT_D;
    const int64_t d = (int64_t)blockIdx.x * SDT_D + threadIdx.x % SDT_D;
    if (b >= batch || d >= di) return;
    float acc = 0.0f;
    for (int r = 0; r < R; ++r)
        acc = fmaf(io<T>::to_f(dl[b * ld_dl + r]), io<T>::to_f(w_dt[d * R + r]), acc);
    const float pre = io<T>::round(acc + (b_dt ? io<T>::to_f(b_dt[d]) : 0.0f));
    const float dt = io<T>::round(softplus_f(pre));
    const float x = io<T>::to_f(xc[b * ld_x + d]);
    float *hr = h + (b * di + d) * S;
    float yv = 0.0f;
    for (int s = 0; s < S; ++s) {
        const float a = -expf(io<T>::to_f(A_log[d * S + s])) * kLog2e;
        const float hv = fmaf(ex2(dt * a), hr[s], (dt * io<T>::to_f(bm[b * ld_bc + s])) * x);
        hr[s] = hv;
        yv = fmaf(hv, io<T>::to_f(cm[b * ld_bc + s]), yv);
    }
    float out = yv + (D ? io<T>::to_f(D[d]) : 0.0f) * x;
    out = io<T>::round(out) * io<T>::round(silu_f(io<T>::to_f(z[b * ld_z + d])));
    y[b * ld_y + d] = io<T>::from_f(out);
}

int scan_step_dt(int dtype, const void *xc, int64_t ld_x, const void *dt_low, int64_t ld_dl,
                 const void *w_dt, const void *b_dt, const void *bm, const void *cm,
                 int64_t ld_bc, const void *z, int64_t ld_z, const void *A_log, const void *D,
                 float *h, void *y, int64_t ld_y, int64_t batch, int64_t d_inner, int64_t d_state,
                 int64_t dt_rank, cudaStream_t st, bool pdl) {
    MB2_REQUIRE(d_state >= 1 && d_state <= 256 && dt_rank >= 1 && dt_rank <= 1024, MB2_ERR_SHAPE,
                "step: d_state %lld or dt_rank %lld out of range", (long long)d_state,
                (long long)dt_rank);
    if (batch == 0 || d_inner == 0) return MB2_OK;
    const int S = (int)d_state, R = (int)dt_rank;
    dim3 grid((unsigned)ceil_div(d_inner, (int64_t)SDT_D), (unsigned)ceil_div(batch, (int64_t)SDT_B));
    const size_t smem = sizeof(float) * ((size_t)SDT_B * SDT_D + 2 * (size_t)SDT_B * S +
                                         (size_t)SDT_B * R + (size_t)SDT_D * (R + 1));
    auto run = [&](auto tag) -> int {
        using T = decltype(tag);
        const T *X = static_cast<const T *>(xc), *DL = static_cast<const T *>(dt_low);
        const T *W = static_cast<const T *>(w_dt), *BB = static_cast<const T *>(b_dt);
        const T *Bp = static_cast<const T *>(bm), *Cp = static_cast<const T *>(cm);
        const T *Z = static_cast<const T *>(z), *AL = static_cast<const T *>(A_log);
        const T *Dp = static_cast<const T *>(D);
        T *Y = static_cast<T *>(y);
        auto tiled = [&](auto kern) -> int {
            if (smem > 48 * 1024) {
                cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int)smem);
                if (e != cudaSuccess)
                    return fail(MB2_ERR_CUDA, "step: smem attribute: %s", cudaGetErrorString(e));
            }
            const cudaError_t le = launch_kernel(pdl, kern, grid, dim3(SDT_THREADS), smem, st, X,
                                                 ld_x, DL, ld_dl, W, BB, Bp, Cp, ld_bc, Z, ld_z,
                                                 AL, Dp, h, Y, ld_y, batch, d_inner, R);
            if (le != cudaSuccess)
                return fail(MB2_ERR_CUDA, "step_scan_dt_kernel launch: %s", cudaGetErrorString(le));
            return check_launch("step_scan_dt_kernel");
        };
        if (aligned(h, 16)) {
            if (S == 4) return tiled(step_scan_dt_kernel<T, 1>);
            if (S == 8) return tiled(step_scan_dt_kernel<T, 2>);
            if (S == 16) return tiled(step_scan_dt_kernel<T, 4>);
            if (S == 32) return tiled(step_scan_dt_kernel<T, 8>);
            if (S == 64) return tiled(step_scan_dt_kernel<T, 16>);
            if (S == 128) return tiled(step_scan_dt_kernel<T, 32>);
        }
        const cudaError_t le = launch_kernel(pdl, step_scan_dt_any_kernel<T>, grid,
                                             dim3(SDT_THREADS), 0, st, X, ld_x, DL, ld_dl, W, BB,
                                             Bp, Cp, ld_bc, Z, ld_z, AL, Dp, h, Y, ld_y, batch,
                                             d_inner, S, R);
        if (le != cudaSuccess)
            return fail(MB2_ERR_CUDA, "step_scan_dt_any_kernel launch: %s", cudaGetErrorString(le));
        return check_launch("step_scan_dt_any_kernel");
    };
    if (dtype == MB2_F32) return run(float{});
    return run(__nv_bfloat16{});
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
    return dispatch_scan<float, PLAIN>(p, (cudaStream_t)stream);
}

extern "C" int mb2_scan_fused(int dtype, const void *xc, int64_t ld_xc, const void *dt_low,
                              int64_t ld_dl, const void *B, int64_t ld_b, const void *C,
                              int64_t ld_c, const void *z, int64_t ld_z, const void *w_dt,
                              const void *b_dt, const void *A_log, const void *D,
                              const float *h0, float *h_last, void *y, int64_t ld_y,
                              int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state,
                              int64_t dt_rank, mb2_stream_t stream) {
    return scan_fused(dtype, xc, ld_xc, dt_low, ld_dl, B, ld_b, C, ld_c, z, ld_z, w_dt, b_dt,
                      A_log, D, h0, h_last, y, ld_y, batch, seqlen, d_inner, d_state, dt_rank,
                      (cudaStream_t)stream);
}

extern "C" int mb2_scan_gated(int dtype, const void *xc, int64_t ld_xc, const void *dt,
                              int64_t ld_dt, const void *B, int64_t ld_b, const void *C,
                              int64_t ld_c, const void *z, int64_t ld_z, const void *A_log,
                              const void *D, const float *h0, float *h_last, void *y,
                              int64_t ld_y, int64_t batch, int64_t seqlen, int64_t d_inner,
                              int64_t d_state, mb2_stream_t stream) {
    return scan_gated(dtype, xc, ld_xc, dt, ld_dt, B, ld_b, C, ld_c, z, ld_z, A_log, D, h0,
                      h_last, y, ld_y, batch, seqlen, d_inner, d_state, (cudaStream_t)stream,
                      nullptr, 0);
}

extern "C" size_t mb2_scan_workspace_bytes(int64_t batch, int64_t seqlen, int64_t d_inner,
                                           int64_t d_state) {
    if (batch < 0 || seqlen < 0 || d_inner < 0 || d_state < 1) return 0;
    return scan_segment_bytes(batch, d_inner, seqlen, d_state);
}

extern "C" int mb2_scan_gated_ws(int dtype, const void *xc, int64_t ld_xc, const void *dt,
                                 int64_t ld_dt, const void *B, int64_t ld_b, const void *C,
                                 int64_t ld_c, const void *z, int64_t ld_z, const void *A_log,
                                 const void *D, const float *h0, float *h_last, void *y,
                                 int64_t ld_y, int64_t batch, int64_t seqlen, int64_t d_inner,
                                 int64_t d_state, void *workspace, size_t workspace_bytes,
                                 mb2_stream_t stream) {
    return scan_gated(dtype, xc, ld_xc, dt, ld_dt, B, ld_b, C, ld_c, z, ld_z, A_log, D, h0,
                      h_last, y, ld_y, batch, seqlen, d_inner, d_state, (cudaStream_t)stream,
                      static_cast<float *>(workspace), workspace ? workspace_bytes : 0);
}
