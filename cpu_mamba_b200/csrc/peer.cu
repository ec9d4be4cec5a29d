// All-reduce (sum) over the GPUs of one node through peer memory: the
// reduction a channel-sharded block needs after x_proj and after out_proj.
//
// Every rank owns one buffer (cudaMalloc, shared with the other ranks'
// processes by CUDA IPC):
//   [0, 256)          status word (first expired wait) + call counter + done count
//   flags             uint32 [MAX_RANKS][MAX_CTAS]: flags[src][c] = the last
//                     call in which rank src delivered chunk c here
//   slots             float [2][world][slot_elems]: slots[call & 1][src] =
//                     rank src's contribution (fp32, whatever the data type)
// One kernel per call, one chunk of the data per CTA.  Each CTA pushes its
// chunk, converted to fp32, into slot [call & 1][rank] of every rank's buffer
// (NVLink stores; its own buffer included), raises its flag in every buffer
// (release, system scope), waits (bounded) for every rank's flag of the same
// chunk in its own buffer (acquire), and sums the world slots in rank order,
// so every rank computes the same bits.  The call number lives in device
// memory (incremented by the last CTA to finish), so the kernel can be
// replayed from a CUDA graph.  Two slot parities keep a fast rank's next call
// from overwriting a slot a slow rank is still summing: a rank reaches call
// k+1 only after every rank raised its call-k flags, i.e. finished call k-1.
// Waits give up after the group's timeout: the status word records it and the
// kernel returns (the data is then not the sum).

#include "common.cuh"

namespace mb2 {

constexpr int PEER_MAX_CTAS = 256;
constexpr int PEER_THREADS = 256;
constexpr size_t PEER_FLAGS_OFF = 256;
constexpr size_t PEER_SLOTS_OFF =
    (PEER_FLAGS_OFF + sizeof(uint32_t) * MB2_PEER_MAX_RANKS * PEER_MAX_CTAS + 255) & ~size_t(255);

struct PeerHeader {
    int status;          // 0, or MB2_PEER_TIMEOUT once a wait expired
    uint32_t calls;      // calls completed on this rank
    uint32_t done;       // CTAs of the running call that have finished
};

struct PeerArgs {
    char *bufs[MB2_PEER_MAX_RANKS];
    int world, rank;
    int64_t slot_elems, count, chunk;
    int64_t timeout_ns;
};

__device__ __forceinline__ uint64_t peer_clock() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// four consecutive elements as fp32 (16-byte fp32 / 8-byte bf16 accesses)
__device__ __forceinline__ float4 ld4f(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ float4 ld4f(const __nv_bfloat16 *p) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void st4f(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }
__device__ __forceinline__ void st4f(__nv_bfloat16 *p, float4 v) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t *>(&a);
    u.y = *reinterpret_cast<const uint32_t *>(&b);
    *reinterpret_cast<uint2 *>(p) = u;
}

// VEC 4: every chunk boundary and the count are multiples of 4 and the data
// and slots 4-element aligned (checked on the host), so each thread moves four
// elements per access; VEC 1: one element per access.
template <typename T, int VEC>
__global__ void __launch_bounds__(PEER_THREADS)
peer_allreduce_kernel(T *__restrict__ data, const __grid_constant__ PeerArgs a) {
    __shared__ uint32_t s_call;
    char *own = a.bufs[a.rank];
    PeerHeader *hdr = reinterpret_cast<PeerHeader *>(own);
    if (threadIdx.x == 0) s_call = *reinterpret_cast<volatile uint32_t *>(&hdr->calls) + 1;
    __syncthreads();
    const uint32_t call = s_call;
    const int c = blockIdx.x;
    const int64_t lo = (int64_t)c * a.chunk;
    const int64_t hi = lo + a.chunk < a.count ? lo + a.chunk : a.count;
    const int64_t par_off = (int64_t)(call & 1) * a.world * a.slot_elems;

    // push this rank's chunk into every rank's slot [call & 1][rank]
    const int64_t own_slot = par_off + (int64_t)a.rank * a.slot_elems;
    if (VEC == 4) {
        for (int64_t i = lo + 4 * threadIdx.x; i < hi; i += 4 * PEER_THREADS) {
            const float4 v = ld4f(data + i);
            for (int p = 0; p < a.world; ++p)
                st4f(reinterpret_cast<float *>(a.bufs[p] + PEER_SLOTS_OFF) + own_slot + i, v);
        }
    } else {
        for (int p = 0; p < a.world; ++p) {
            float *dst = reinterpret_cast<float *>(a.bufs[p] + PEER_SLOTS_OFF) + own_slot;
            for (int64_t i = lo + threadIdx.x; i < hi; i += PEER_THREADS)
                dst[i] = io<T>::to_f(data[i]);
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < a.world) {
        uint32_t *flags = reinterpret_cast<uint32_t *>(a.bufs[threadIdx.x] + PEER_FLAGS_OFF);
        st_release_sys(&flags[a.rank * PEER_MAX_CTAS + c], call);
        // wait for rank threadIdx.x's delivery of this chunk into our buffer
        const uint32_t *mine = reinterpret_cast<const uint32_t *>(own + PEER_FLAGS_OFF) +
                               threadIdx.x * PEER_MAX_CTAS + c;
        if ((int32_t)(ld_acquire_sys(mine) - call) < 0) {
            const uint64_t t0 = peer_clock();
            while ((int32_t)(ld_acquire_sys(mine) - call) < 0) {
                if (peer_clock() - t0 > (uint64_t)a.timeout_ns) {
                    atomicCAS(&hdr->status, 0, MB2_PEER_TIMEOUT);
                    break;
                }
            }
        }
    }
    __syncthreads();

    // sum the world contributions in rank order (the same bits on every rank)
    const float *slots = reinterpret_cast<const float *>(own + PEER_SLOTS_OFF) + par_off;
    if (VEC == 4) {
        for (int64_t i = lo + 4 * threadIdx.x; i < hi; i += 4 * PEER_THREADS) {
            float4 s = __ldcg(reinterpret_cast<const float4 *>(slots + i));
            for (int p = 1; p < a.world; ++p) {
                const float4 v =
                    __ldcg(reinterpret_cast<const float4 *>(slots + (int64_t)p * a.slot_elems + i));
                s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
            }
            st4f(data + i, s);
        }
    } else {
        for (int64_t i = lo + threadIdx.x; i < hi; i += PEER_THREADS) {
            float s = __ldcg(slots + i);
            for (int p = 1; p < a.world; ++p) s += __ldcg(slots + (int64_t)p * a.slot_elems + i);
            data[i] = io<T>::from_f(s);
        }
    }

    // the last CTA to finish advances the call counter
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&hdr->done, 1u) == gridDim.x - 1) {
            hdr->done = 0;
            __threadfence();
            *reinterpret_cast<volatile uint32_t *>(&hdr->calls) = call;
        }
    }
}

}  // namespace mb2

using namespace mb2;

extern "C" size_t mb2_peer_buffer_bytes(int world, int64_t slot_elems) {
    if (world < 1 || world > MB2_PEER_MAX_RANKS || slot_elems < 0) return 0;
    return PEER_SLOTS_OFF + sizeof(float) * 2 * (size_t)world * (size_t)slot_elems;
}

extern "C" int mb2_peer_alloc(size_t bytes, void **ptr, void *ipc_handle) {
    MB2_REQUIRE(ptr && ipc_handle && bytes >= PEER_SLOTS_OFF, MB2_ERR_ARG,
                "peer_alloc: bad argument");
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return fail(MB2_ERR_CUDA, "peer_alloc: %s", cudaGetErrorString(e));
    e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(MB2_ERR_CUDA, "peer_alloc: %s", cudaGetErrorString(e));
    }
    memcpy(ipc_handle, &h, sizeof(h));
    *ptr = p;
    return MB2_OK;
}

extern "C" int mb2_peer_open(const void *ipc_handle, void **ptr) {
    MB2_REQUIRE(ptr && ipc_handle, MB2_ERR_ARG, "peer_open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return fail(MB2_ERR_CUDA, "peer_open: %s", cudaGetErrorString(e));
    return MB2_OK;
}

extern "C" int mb2_peer_close(void *ptr) {
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) return fail(MB2_ERR_CUDA, "peer_close: %s", cudaGetErrorString(e));
    return MB2_OK;
}

extern "C" int mb2_peer_free(void *ptr) {
    cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) return fail(MB2_ERR_CUDA, "peer_free: %s", cudaGetErrorString(e));
    return MB2_OK;
}

extern "C" int mb2_peer_allreduce(int dtype, void *data, int64_t count, const mb2_peer_group *g,
                                  mb2_stream_t stream) {
    MB2_REQUIRE(g, MB2_ERR_ARG, "peer_allreduce: null group");
    MB2_REQUIRE(g->world >= 1 && g->world <= MB2_PEER_MAX_RANKS && g->rank >= 0 &&
                    g->rank < g->world,
                MB2_ERR_ARG, "peer_allreduce: rank %d of world %d", g->rank, g->world);
    MB2_REQUIRE(dtype == MB2_F32 || dtype == MB2_BF16, MB2_ERR_ARG, "peer_allreduce: bad dtype");
    MB2_REQUIRE(count >= 0 && count <= g->slot_elems, MB2_ERR_SHAPE,
                "peer_allreduce: %lld elements > slot of %lld", (long long)count,
                (long long)g->slot_elems);
    MB2_REQUIRE(g->timeout_ns > 0, MB2_ERR_ARG, "peer_allreduce: timeout must be positive");
    if (count == 0) return MB2_OK;
    MB2_REQUIRE(data, MB2_ERR_ARG, "peer_allreduce: null data");
    PeerArgs a{};
    for (int p = 0; p < g->world; ++p) {
        MB2_REQUIRE(g->bufs[p] && aligned(g->bufs[p], 256), MB2_ERR_ALIGN,
                    "peer_allreduce: buffer of rank %d missing or misaligned", p);
        a.bufs[p] = static_cast<char *>(g->bufs[p]);
    }
    a.world = g->world;
    a.rank = g->rank;
    a.slot_elems = g->slot_elems;
    a.count = count;
    a.timeout_ns = g->timeout_ns;
    const size_t es = dtype == MB2_F32 ? 4 : 2;
    const bool vec = count % 4 == 0 && g->slot_elems % 4 == 0 && aligned(data, 4 * es);
    // about 2048 elements per CTA (more CTAs push more bytes over NVLink at once)
    int64_t ctas = ceil_div(count, (int64_t)2048);
    if (ctas > PEER_MAX_CTAS) ctas = PEER_MAX_CTAS;
    a.chunk = ceil_div(count, ctas);
    if (vec) a.chunk = round_up(a.chunk, 4);
    ctas = ceil_div(count, a.chunk);
    cudaStream_t st = (cudaStream_t)stream;
    if (dtype == MB2_F32) {
        float *d = static_cast<float *>(data);
        if (vec) peer_allreduce_kernel<float, 4><<<(unsigned)ctas, PEER_THREADS, 0, st>>>(d, a);
        else peer_allreduce_kernel<float, 1><<<(unsigned)ctas, PEER_THREADS, 0, st>>>(d, a);
    } else {
        __nv_bfloat16 *d = static_cast<__nv_bfloat16 *>(data);
        if (vec)
            peer_allreduce_kernel<__nv_bfloat16, 4><<<(unsigned)ctas, PEER_THREADS, 0, st>>>(d, a);
        else
            peer_allreduce_kernel<__nv_bfloat16, 1><<<(unsigned)ctas, PEER_THREADS, 0, st>>>(d, a);
    }
    return check_launch("peer_allreduce_kernel");
}

extern "C" int mb2_peer_status(const mb2_peer_group *g, int *code, int clear) {
    MB2_REQUIRE(g && code && g->rank >= 0 && g->rank < g->world && g->bufs[g->rank], MB2_ERR_ARG,
                "peer_status: bad argument");
    cudaError_t e = cudaMemcpy(code, g->bufs[g->rank], sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) {
        const int zero = 0;
        e = cudaMemcpy(g->bufs[g->rank], &zero, sizeof(int), cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) return fail(MB2_ERR_CUDA, "peer_status: %s", cudaGetErrorString(e));
    return MB2_OK;
}
