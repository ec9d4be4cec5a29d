// First-order linear recurrence over time, h[t] = a[t] * h[t-1] + b[t] with
// h[-1] = 0: the primitive of the reference's associative scans
// (src/cpu_mamba/scan_assoc.py:24-55, recursive doubling over dim 1 of
// (B, T, ...) tensors).  On the GPU every trailing element is an independent
// chain, so one thread walks each chain through time (the doubling tree's
// T log T work is not needed) and consecutive threads take consecutive
// elements of a row, so every time step reads and writes whole rows
// coalesced.  HBM-bound: 3 x B x T x inner elements move once.  The state is
// kept in fp32 (bf16 tensors are read and written in bf16).

#include "common.cuh"

namespace mb2 {

template <typename T>
__global__ void __launch_bounds__(256)
recurrence_kernel(const T *__restrict__ a, const T *__restrict__ b, T *__restrict__ h,
                  int64_t seqlen, int64_t inner) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= inner) return;
    const int64_t base = (int64_t)blockIdx.y * seqlen * inner + e;
    const T *ap = a + base;
    const T *bp = b + base;
    T *hp = h + base;
    float hv = 0.0f;
    int64_t t = 0;
    // four steps' loads issued together, then the dependent updates
    for (; t + 4 <= seqlen; t += 4) {
        float av[4], bv[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            av[k] = io<T>::to_f(ap[(t + k) * inner]);
            bv[k] = io<T>::to_f(bp[(t + k) * inner]);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            hv = fmaf(av[k], hv, bv[k]);
            hp[(t + k) * inner] = io<T>::from_f(hv);
        }
    }
    for (; t < seqlen; ++t) {
        hv = fmaf(io<T>::to_f(ap[t * inner]), hv, io<T>::to_f(bp[t * inner]));
        hp[t * inner] = io<T>::from_f(hv);
    }
}

}  // namespace mb2

using namespace mb2;

extern "C" int mb2_linear_recurrence(int dtype, const void *a, const void *b, void *h,
                                     int64_t batch, int64_t seqlen, int64_t inner,
                                     mb2_stream_t stream) {
    MB2_REQUIRE(dtype == MB2_F32 || dtype == MB2_BF16, MB2_ERR_ARG, "recurrence: bad dtype");
    MB2_REQUIRE(batch >= 0 && seqlen >= 0 && inner >= 0, MB2_ERR_SHAPE,
                "recurrence: negative size");
    MB2_REQUIRE(batch < 65536, MB2_ERR_SHAPE, "recurrence: batch %lld >= 65536",
                (long long)batch);
    if (batch == 0 || seqlen == 0 || inner == 0) return MB2_OK;
    MB2_REQUIRE(a && b && h, MB2_ERR_ARG, "recurrence: null pointer");
    const dim3 grid((unsigned)ceil_div(inner, (int64_t)256), (unsigned)batch);
    cudaStream_t st = (cudaStream_t)stream;
    if (dtype == MB2_F32)
        recurrence_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float *>(a),
                                                      static_cast<const float *>(b),
                                                      static_cast<float *>(h), seqlen, inner);
    else
        recurrence_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
            static_cast<const __nv_bfloat16 *>(a), static_cast<const __nv_bfloat16 *>(b),
            static_cast<__nv_bfloat16 *>(h), seqlen, inner);
    return check_launch("recurrence_kernel");
}
