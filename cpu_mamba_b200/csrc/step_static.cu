// mb2_block_step_static: the one-token decode step (mb2_block_step) for
// callers that cannot allocate device memory.
//
// Who needs it: a host program whose device memory is owned and budgeted by
// another runtime (a plugin inside a larger application), or a serving loop
// that must not allocate once it is running, because an allocation there can
// stall the device or fail under memory pressure in the middle of a request.
// Such a caller can hand over its inputs, outputs and state buffers but has no
// way to supply the step's workspace.  This entry point takes the workspace
// from a fixed array that lives inside this library instead.
//
// The array (MB2_STEP_STATIC_SCRATCH_BYTES, 8 MiB) is a file-scope __device__
// variable: every GPU that loads the library holds it until the process exits.
// Its host-side name is only a stand-in, so its device address is looked up
// with cudaGetSymbolAddress, once per device, the first time this entry point
// runs on that device (with that device current).  That lookup can load the
// module onto the device, so the first call on each device should come before
// any stream capture.
//
// All calls on a device share the one array, and it keeps whatever the last
// call left in it.  The step writes every scratch byte it reads before reading
// it (the x_proj padding columns it skips are zero-filled on the way into
// shared memory, never read from the array), so nothing has to be cleared
// between calls.  Calls whose work overlaps on the GPU (on different streams,
// or from different host threads without ordering) race on the array; callers
// must order them.
#include "common.cuh"

#include <mutex>

static __device__ __align__(256) unsigned char g_step_scratch[MB2_STEP_STATIC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void *g_scratch_ptr[kMaxDevices];   // device address of g_step_scratch, per device

// device address of the scratch array on the current device (looked up once)
int scratch_for_current_device(void **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    MB2_REQUIRE(e == cudaSuccess, MB2_ERR_CUDA, "step_static: cudaGetDevice: %s",
                cudaGetErrorString(e));
    MB2_REQUIRE(dev >= 0 && dev < kMaxDevices, MB2_ERR_UNSUPPORTED,
                "step_static: device ordinal %d above %d", dev, kMaxDevices - 1);
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_step_scratch);
        MB2_REQUIRE(e == cudaSuccess && p, MB2_ERR_CUDA,
                    "step_static: cudaGetSymbolAddress on device %d: %s", dev,
                    cudaGetErrorString(e));
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return MB2_OK;
}

}  // namespace

extern "C" int mb2_block_step_static(const mb2_block *blk, const void *x, void *out, float *h,
                                     void *conv_state, int64_t batch, mb2_stream_t stream) {
    MB2_REQUIRE(blk, MB2_ERR_ARG, "step_static: null descriptor");
    MB2_REQUIRE(batch >= 0, MB2_ERR_SHAPE, "step_static: negative batch");
    const size_t need = mb2_step_workspace_bytes(blk, batch);
    MB2_REQUIRE(need <= (size_t)MB2_STEP_STATIC_SCRATCH_BYTES, MB2_ERR_WORKSPACE,
                "step_static: batch %lld needs %zu bytes of scratch, more than the fixed "
                "%zu-byte array; use mb2_block_step with a caller workspace",
                (long long)batch, need, (size_t)MB2_STEP_STATIC_SCRATCH_BYTES);
    if (batch == 0) return mb2_block_step(blk, x, out, h, conv_state, 0, nullptr, 0, stream);
    void *scratch = nullptr;
    MB2_TRY(scratch_for_current_device(&scratch));
    return mb2_block_step(blk, x, out, h, conv_state, batch, scratch,
                          (size_t)MB2_STEP_STATIC_SCRATCH_BYTES, stream);
}
