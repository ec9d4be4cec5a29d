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
// with cudaGetSymbolAddress, with the device current, the first time this
// entry point runs on a device.  That lookup can load the module onto the
// device, so the first call on each device should come before any stream
// capture.  The address is kept per device together with the id of the CUDA
// context it was found in: after cudaDeviceReset (which unloads the module and
// frees the array) the device has a new context, the ids differ, and the next
// call looks the address up again instead of handing a freed one to the kernels.
//
// All calls on a device share the one array, and it keeps whatever the last
// call left in it.  The step writes every scratch byte it reads before reading
// it (the x_proj padding columns it skips are zero-filled on the way into
// shared memory, never read from the array), so nothing has to be cleared
// between calls.  Calls whose work overlaps on the GPU (on different streams,
// or from different host threads without ordering) race on the array; callers
// must order them.
#include <cuda.h>

#include "common.cuh"

#include <mutex>

static __device__ __align__(256) unsigned char g_step_scratch[MB2_STEP_STATIC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
struct ScratchAddr {
    void *ptr;              // device address of g_step_scratch
    unsigned long long ctx; // id of the context it belongs to
};
ScratchAddr g_scratch[kMaxDevices];

using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);

// id of the current CUDA context (unique for the process's lifetime), or 0
// when the driver cannot tell; 0 makes the caller look the address up again
unsigned long long current_context_id() {
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static bool tried = false;
    if (!tried) {    // called under g_setup_mu
        tried = true;
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
        fn = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(fn);
    }
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx ||
        get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

// device address of the scratch array in the current device's context
int scratch_for_current_device(void **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    MB2_REQUIRE(e == cudaSuccess, MB2_ERR_CUDA, "step_static: cudaGetDevice: %s",
                cudaGetErrorString(e));
    MB2_REQUIRE(dev >= 0 && dev < kMaxDevices, MB2_ERR_UNSUPPORTED,
                "step_static: device ordinal %d above %d", dev, kMaxDevices - 1);
    std::lock_guard<std::mutex> lock(g_setup_mu);
    const unsigned long long ctx = current_context_id();
    ScratchAddr &a = g_scratch[dev];
    if (!a.ptr || ctx == 0 || a.ctx != ctx) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_step_scratch);
        MB2_REQUIRE(e == cudaSuccess && p, MB2_ERR_CUDA,
                    "step_static: cudaGetSymbolAddress on device %d: %s", dev,
                    cudaGetErrorString(e));
        a.ptr = p;
        // read again: the lookup makes the device's primary context current
        // when nothing had used the device yet
        a.ctx = current_context_id();
    }
    *out = a.ptr;
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
