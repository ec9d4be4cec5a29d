/*
 * ORACLE -- test infrastructure only.
 *
 * CPU restatement of cpu-mamba's selective scan, used solely as the checker
 * for the CUDA path (by tests/, __graft_entry__.smoke() and the cpu_baseline
 * leg of bench.py).  Nothing in the product links or calls this file.
 *
 * Follows src/cpu_mamba/selective_scan_cpu.cpp:19-87:
 *   for each (b, d):  h[s] = h0 or 0
 *     for t in [0, T):
 *       dA   = exp(dt[b,t,d] * A[d,s])                 (cpp:77)
 *       dBx  = (dt[b,t,d] * B[b,t,s]) * x[b,t,d]       (cpp:78, this association)
 *       h[s] = dA * h[s] + dBx                         (cpp:79)
 *       y   += h[s] * C[b,t,s]                         (cpp:80)
 *     out[b,t,d] = y + D[d] * x[b,t,d]                 (cpp:82)
 * The optional h0 / h_last arguments restate the time loop that
 * forward_with_final_state uses for the final state (src/cpu_mamba/_mamba.py:191-199),
 * which is the same recurrence without the C/D read-out.
 *
 * Parity is pinned against golden vectors produced by the reference's own
 * compiled C++ op (tests/golden/make_golden.py).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

int oracle_selective_scan_f32(const float *x, const float *dt, const float *A,
                              const float *B, const float *C, const float *D,
                              float *y, int64_t batch, int64_t seqlen,
                              int64_t d_inner, int64_t d_state,
                              const float *h0, float *h_last) {
    if (d_state <= 0 || d_state > 256) return 1;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < batch; ++b) {
        for (int64_t d = 0; d < d_inner; ++d) {
            float h[256];
            for (int64_t s = 0; s < d_state; ++s)
                h[s] = h0 ? h0[(b * d_inner + d) * d_state + s] : 0.0f;
            const float *a_row = A + d * d_state;
            const float d_skip = D ? D[d] : 0.0f;
            for (int64_t t = 0; t < seqlen; ++t) {
                const int64_t tok = b * seqlen + t;
                const float dtv = dt[tok * d_inner + d];
                const float xv = x[tok * d_inner + d];
                const float *b_row = B + tok * d_state;
                const float *c_row = C ? C + tok * d_state : NULL;
                float acc = 0.0f;
                for (int64_t s = 0; s < d_state; ++s) {
                    const float da = expf(dtv * a_row[s]);
                    const float dbx = (dtv * b_row[s]) * xv;
                    h[s] = da * h[s] + dbx;
                    if (c_row) acc += h[s] * c_row[s];
                }
                if (y) y[tok * d_inner + d] = acc + d_skip * xv;
            }
            if (h_last)
                for (int64_t s = 0; s < d_state; ++s)
                    h_last[(b * d_inner + d) * d_state + s] = h[s];
        }
    }
    return 0;
}
