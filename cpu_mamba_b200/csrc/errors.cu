// Status reporting for the C ABI: a thread-local message for the last failing
// call, returned by mb2_last_error().
#include "common.cuh"

namespace mb2 {

static thread_local std::string g_last_error;

void set_error(const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(MB2_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return MB2_OK;
}

}  // namespace mb2

extern "C" const char *mb2_last_error(void) { return mb2::g_last_error.c_str(); }

extern "C" int mb2_version(void) { return 2; }
