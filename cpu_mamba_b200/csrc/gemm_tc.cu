// Tensor-core GEMM entry (tcgen05).  Placeholder until the sm_100a kernel
// lands: reports "not used" so callers take the CUDA-core kernel.
#include "common.cuh"

namespace mb2 {

int gemm_tc(int dtype, const void *x, int64_t ld_x, const void *w, const float *w_split,
            const void *bias, void *y, int64_t ld_y, int64_t M, int64_t N, int64_t K,
            int64_t n1, int64_t off1, int64_t n2, int64_t off2, cudaStream_t st, bool *used) {
    (void)dtype; (void)x; (void)ld_x; (void)w; (void)w_split; (void)bias; (void)y; (void)ld_y;
    (void)M; (void)N; (void)K; (void)n1; (void)off1; (void)n2; (void)off2; (void)st;
    *used = false;
    return MB2_OK;
}

}  // namespace mb2

// ------------------------------------------------------------- TF32 split ---
// hi = tf32_rn(w), lo = tf32_rn(w - hi): w == hi + lo up to 2^-22 |w|.  Used
// as a derived cache of fp32 weights for the 3-term TF32 tensor-core GEMM.
namespace mb2 {
__device__ __forceinline__ float tf32_rn(float v) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return __uint_as_float(r);
}

__global__ void split_tf32_kernel(const float *__restrict__ w, float *__restrict__ out,
                                  int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = w[i];
    const float h = tf32_rn(v);
    out[i] = h;
    out[n + i] = tf32_rn(v - h);
}
}  // namespace mb2

extern "C" int mb2_split_tf32(const float *w, float *out, int64_t numel,
                              mb2_stream_t stream) {
    MB2_REQUIRE(numel >= 0, MB2_ERR_SHAPE, "split_tf32: negative size");
    if (numel == 0) return MB2_OK;
    MB2_REQUIRE(w && out, MB2_ERR_ARG, "split_tf32: null pointer");
    mb2::split_tf32_kernel<<<(unsigned)mb2::ceil_div(numel, 256), 256, 0, (cudaStream_t)stream>>>(
        w, out, numel);
    return mb2::check_launch("split_tf32_kernel");
}
