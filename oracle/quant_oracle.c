/*
 * ORACLE -- test infrastructure only.
 *
 * CPU restatement of cpu-mamba's weight-only quantisation primitives
 * (src/cpu_mamba/quant.py:35-134).  Used by tests/ as the bit-exact checker for
 * the CUDA pack / unpack / dequant kernels; never linked into the product.
 *
 * Arithmetic follows torch's float32 semantics that quant.py relies on:
 *   - amax over |w| of a row, clamp(min=1e-8) with 1e-8 rounded to float32;
 *   - IEEE float32 division (w / scale);
 *   - round half to even (torch.round == nearbyint in the default mode);
 *   - argmin returns the FIRST minimal index (nf4 ties).
 * Pinned against golden vectors written by the reference itself
 * (tests/golden/make_golden.py).
 */
#include <math.h>
#include <stdint.h>

/* quant.py:35-40 -- the LUT is a tuple of Python floats turned into a float32
 * tensor, i.e. decimal -> double -> float.  Casting double literals reproduces
 * that exact rounding path. */
static const double NF4_LUT_D[16] = {
    -1.0, -0.6961928, -0.5250730, -0.39491748,
    -0.28444138, -0.18477343, -0.09105602, 0.0,
    0.07958029, 0.16093020, 0.24611230, 0.33791524,
    0.44070983, 0.56261897, 0.72295684, 1.0,
};

static float nf4_lut(int i) { return (float)NF4_LUT_D[i]; }

void oracle_nf4_lut(float *out16) {
    for (int i = 0; i < 16; ++i) out16[i] = nf4_lut(i);
}

static float row_amax(const float *w, int64_t cols) {
    float m = 0.0f;
    for (int64_t j = 0; j < cols; ++j) {
        float a = fabsf(w[j]);
        if (a > m || isnan(a)) m = a;
    }
    return m;
}

static float clamp_min_eps(float v) {
    const float eps = (float)1e-8;
    return v < eps ? eps : v;
}

/* quant.py:60-65 */
void oracle_quant_int8(const float *w, int64_t rows, int64_t cols, int8_t *q,
                       float *scale) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float *wr = w + r * cols;
        float s = clamp_min_eps(row_amax(wr, cols)) / 127.0f;
        scale[r] = s;
        for (int64_t j = 0; j < cols; ++j) {
            float v = nearbyintf(wr[j] / s);
            if (v < -127.0f) v = -127.0f;
            if (v > 127.0f) v = 127.0f;
            q[r * cols + j] = (int8_t)v;
        }
    }
}

/* quant.py:68-69 */
void oracle_dequant_int8(const int8_t *q, const float *scale, int64_t rows,
                         int64_t cols, float *out) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t j = 0; j < cols; ++j)
            out[r * cols + j] = (float)q[r * cols + j] * scale[r];
}

/* quant.py:72-87: codes in [-7, 7] stored as u = q + 7; even element in the
 * high nibble; an odd row length is padded with q = 0 (nibble 7). */
void oracle_quant_int4(const float *w, int64_t rows, int64_t cols,
                       uint8_t *packed, float *scale) {
    const int64_t pcols = (cols + 1) / 2;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float *wr = w + r * cols;
        float s = clamp_min_eps(row_amax(wr, cols)) / 7.0f;
        scale[r] = s;
        for (int64_t p = 0; p < pcols; ++p) {
            uint8_t nib[2];
            for (int k = 0; k < 2; ++k) {
                int64_t j = 2 * p + k;
                int qv = 0;
                if (j < cols) {
                    float v = nearbyintf(wr[j] / s);
                    if (v < -7.0f) v = -7.0f;
                    if (v > 7.0f) v = 7.0f;
                    qv = (int)v;
                }
                nib[k] = (uint8_t)(qv + 7);
            }
            packed[r * pcols + p] = (uint8_t)((nib[0] << 4) | nib[1]);
        }
    }
}

/* quant.py:90-101 */
void oracle_dequant_int4(const uint8_t *packed, const float *scale,
                         int64_t rows, int64_t in_dim, float *out) {
    const int64_t pcols = (in_dim + 1) / 2;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t j = 0; j < in_dim; ++j) {
            uint8_t byte = packed[r * pcols + j / 2];
            int u = (j & 1) ? (byte & 0x0F) : ((byte >> 4) & 0x0F);
            out[r * in_dim + j] = (float)(int8_t)(u - 7) * scale[r];
        }
}

/* quant.py:104-121: nearest LUT entry of clamp(w / amax, -1, 1). */
void oracle_quant_nf4(const float *w, int64_t rows, int64_t cols,
                      uint8_t *packed, float *scale) {
    const int64_t pcols = (cols + 1) / 2;
    float lut[16];
    oracle_nf4_lut(lut);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float *wr = w + r * cols;
        float s = clamp_min_eps(row_amax(wr, cols));
        scale[r] = s;
        for (int64_t p = 0; p < pcols; ++p) {
            uint8_t nib[2];
            for (int k = 0; k < 2; ++k) {
                int64_t j = 2 * p + k;
                int best = 0;
                if (j < cols) {
                    float wn = wr[j] / s;
                    if (wn < -1.0f) wn = -1.0f;
                    if (wn > 1.0f) wn = 1.0f;
                    float bd = fabsf(wn - lut[0]);
                    for (int i = 1; i < 16; ++i) {
                        float dd = fabsf(wn - lut[i]);
                        if (dd < bd) { bd = dd; best = i; }
                    }
                }
                nib[k] = (uint8_t)best;
            }
            packed[r * pcols + p] = (uint8_t)((nib[0] << 4) | nib[1]);
        }
    }
}

/* quant.py:124-134 */
void oracle_dequant_nf4(const uint8_t *packed, const float *scale,
                        int64_t rows, int64_t in_dim, float *out) {
    const int64_t pcols = (in_dim + 1) / 2;
    float lut[16];
    oracle_nf4_lut(lut);
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t j = 0; j < in_dim; ++j) {
            uint8_t byte = packed[r * pcols + j / 2];
            int idx = (j & 1) ? (byte & 0x0F) : ((byte >> 4) & 0x0F);
            out[r * in_dim + j] = lut[idx] * scale[r];
        }
}
