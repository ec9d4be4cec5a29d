// Tensor-core GEMM for sm_100a (tcgen05 + TMA + TMEM): y = x W^T (+ bias).
//
// Used for the block's large-M projections (in_proj, x_proj, out_proj;
// nn.Linear at src/cpu_mamba/_mamba.py:67,74,84).
//
//   BF16 mode : A, B bf16 (K-major), kind::f16 MMA, fp32 accumulation in TMEM,
//               bf16 output -- the reference's bf16 F.linear.
//   F32 mode  : fp32-faithful 3-term TF32 split.  W arrives pre-split as TF32
//               hi / lo planes (mb2_split_tf32).  Each A tile is loaded as fp32
//               by TMA; four transform warps read it row by row, split it into
//               hi = tf32_rn(a) and lo = tf32_rn(a - hi) and write both into
//               tensor memory (tcgen05.st), so the MMAs take A from TMEM and
//               only W from shared memory.  The MMA warp issues
//               A_hi*W_hi + A_hi*W_lo + A_lo*W_hi.  The dropped A_lo*W_lo term
//               and the rounding of lo are <= 2^-21 |a||w|.  The tensor core
//               truncates when it adds into an fp32 accumulator, so the error
//               grows with the number of MMAs per accumulator: the big hi*hi
//               products alternate between two TMEM accumulators by K slice,
//               the small cross terms go to a third, and the epilogue sums the
//               three in fp32 round-to-nearest.
//
// Persistent, warp-specialised: one CTA per SM walks the 128 x 128 output
// tiles (n fastest, so co-resident CTAs share A rows in L2):
//   warp 0      TMA producer (one lane), STAGES-deep shared-memory ring that
//               runs ahead across tile boundaries
//   warp 1      TMEM allocator + MMA issuer (one lane)
//   warps 2-5   F32 mode: A split into TMEM (two k-block slots)
//   last 4      epilogue: drain the accumulator(s) from TMEM, hand TMEM back
//               to the MMA warp, then bias / softplus / dtype conversion into
//               a 128B-swizzled staging tile in shared memory and TMA bulk
//               tensor stores to global memory, overlapping the next tile's
//               main loop.  (A column remap or an unaligned output falls back
//               to plain stores.)
// Operand tiles are 128 rows x 128 bytes, 128-byte swizzled (TMA and UMMA
// descriptors agree).  Every mbarrier wait is bounded (~2 s): on expiry the
// thread records an error in g_mb2_device_error and stops, and the allocating
// warp still frees its TMEM.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "internal.cuh"

namespace mb2 {

__device__ int g_mb2_device_error = 0;  // 0 = ok; else a code of where a wait expired

namespace tc {

constexpr int BM = 128;
constexpr int TILE_BYTES = 128 * 128;   // 128 operand rows x 128 B
constexpr uint64_t WAIT_NS = 2000000000ull;  // 2 s bound on any wait

enum Mode { F32X3 = 0, BF16 = 1 };

template <int MODE> struct Cfg;
// F32X3: 3-deep TMA ring of (A raw, W_hi, W_lo) tiles; the split A (hi, lo)
// lives in two TMEM slots of 64 columns next to the three accumulators.
template <> struct Cfg<F32X3> {
    static constexpr int BN = 128;            // tile columns (MMA N)
    static constexpr int STAGES = 3;
    static constexpr int LO = 2;              // TMEM slots for the split A
    static constexpr int BK = 32;             // fp32 elements per 128 B row
    static constexpr int KSTEP = 8;           // K per tf32 MMA
    static constexpr uint32_t STAGE_BYTES = (BM + 2 * BN) * 128;  // A raw | W_hi | W_lo
    static constexpr uint32_t TX = STAGE_BYTES;  // bytes by TMA per stage
    static constexpr int NACC = 1;            // accumulator sets (3 x BN columns)
    static constexpr int ACC_COLS = 3 * BN;
    static constexpr int TMEM_COLS = 512;
    static constexpr int A_COL = 3 * BN;      // split-A slot l at 384 + 64 l (hi), +32 (lo)
    static constexpr int WARPS = 10;
    static constexpr int EPI0 = 6;            // first epilogue warp
    static constexpr int EPG = 1;             // epilogue warps per TMEM lane quarter (two:
                                              // decode step 49.4 -> 50.6 us, not kept)
    static constexpr int SPLIT = 1;           // output staged in one piece
};
// BF16: 128 x 256 tiles (N = 256 MMAs: the 128-wide ones ran the tensor pipe
// at about half its rate), 4-deep ring of (A, W) tiles, two 256-column
// accumulators (all 512 TMEM columns) so the MMAs of the next tile overlap the
// epilogue of the previous one.  Eight epilogue warps, two per TMEM lane
// quarter (one per 128-column half), each staging its output 64 columns at a
// time: with few k-blocks (dt_proj, K = 48) the tile's drain is the bound.
template <> struct Cfg<BF16> {
    static constexpr int BN = 256;
    static constexpr int STAGES = 4;
    static constexpr int LO = 1;              // (no split A; one unused barrier)
    static constexpr int BK = 64;
    static constexpr int KSTEP = 16;
    static constexpr uint32_t STAGE_BYTES = (BM + BN) * 128;       // A | W
    static constexpr uint32_t TX = STAGE_BYTES;
    static constexpr int NACC = 2;
    static constexpr int ACC_COLS = BN;
    static constexpr int TMEM_COLS = 512;
    static constexpr int A_COL = 0;
    static constexpr int WARPS = 10;
    static constexpr int EPI0 = 2;
    static constexpr int EPG = 2;
    static constexpr int SPLIT = 2;           // parts of a warp's columns staged at a time
};

// shared memory: ring | output staging (BM x BN/SPLIT of TO: 4 EPG warps of
// 32 rows x BN/(EPG SPLIT) columns) | barriers
template <int MODE, typename TO>
__host__ __device__ constexpr size_t staging_bytes() {
    return (size_t)BM * (Cfg<MODE>::BN / Cfg<MODE>::SPLIT) * sizeof(TO);
}
template <int MODE, typename TO>
constexpr size_t smem_bytes() {
    return 1024 /*align slack*/ + (size_t)Cfg<MODE>::STAGES * Cfg<MODE>::STAGE_BYTES +
           staging_bytes<MODE, TO>() + 256;
}

struct Params {
    void *y; int64_t ld_y;
    const void *bias;
    int64_t M, N, K;
    int64_t n1, n2, off1, off2;   // output column remap
    int epi;                      // MB2_EPI_NONE / MB2_EPI_SOFTPLUS
    int tma_store;                // 1: store through map_y
    const float *row_scale;       // EpiExtra terms (internal.cuh)
    const void *resid; int64_t ld_r;
    // split-K (few rows): tiles = (m, n, split), each split a range of kbs
    // k-blocks, raw fp32 partial sums stored through a 3D map (N, M, split)
    int ksplit, kbs;
    int64_t silu_from = -1;       // EpiExtra's SiLU columns (< 0: none)
    // launched as part of a programmatic chain whose previous kernel writes
    // nothing the weights' loads read: the first stages' weight tiles are
    // loaded before waiting for that kernel (common.cuh, pdl_wait)
    int w_early = 0;
};

// ------------------------------------------------------------- primitives
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}

// Bounded wait with cluster-scope acquire: for barriers that the other CTA
// of an SM pair arrives on remotely.
__device__ __forceinline__ bool mbar_try_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, int where) {
    if (mbar_try_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_cluster(bar, parity)) return true;
        if ((i & 255) == 0 && globaltimer() - t0 > WAIT_NS) {
            atomicCAS(&g_mb2_device_error, 0, where);
            return false;
        }
    }
}

// Bounded wait; false (and the device error flag set) when it expired.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int where) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try(bar, parity)) return true;
        if ((i & 255) == 0 && globaltimer() - t0 > WAIT_NS) {
            atomicCAS(&g_mb2_device_error, 0, where);
            return false;
        }
    }
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                            int32_t c0, int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups of
// 1024 B (SBO), sm100 descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}

template <int MODE>
__host__ __device__ constexpr uint32_t instr_desc() {
    // D fmt F32 (bits 4-5 = 1); A/B fmt (bits 7-9, 10-12): TF32 = 2, BF16 = 1;
    // K-major A and B; N >> 3 at bits 17-22; M >> 4 at bits 24-28.
    constexpr uint32_t fmt = MODE == F32X3 ? 2u : 1u;
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(Cfg<MODE>::BN >> 3) << 17) |
           ((uint32_t)(BM >> 4) << 24);
}

template <int MODE>
__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accum) {
    const uint32_t idesc = instr_desc<MODE>();
    if (MODE == F32X3) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accum));
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accum));
    }
}

// tf32 MMA with A (128 x 8) read from tensor memory, B from shared memory.
__device__ __forceinline__ void mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db,
                                       uint32_t accum) {
    const uint32_t idesc = instr_desc<F32X3>();
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(accum));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
          "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]),
          "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
          "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
          "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]),
          "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(bar) : "memory");
}

__device__ __forceinline__ float tf32_rn(float v) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return __uint_as_float(r);
}

// 32 lanes x 32 columns from TMEM; the load is asynchronous until tmem_wait_ld()
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}
// 32 lanes x 16 columns from TMEM; asynchronous until tmem_wait_ld()
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t src, int32_t c0,
                                             int32_t c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(c0), "r"(c1) : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, uint32_t src, int32_t c0,
                                             int32_t c1, int32_t c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;"); }
__device__ __forceinline__ void bulk_wait_read0() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ----------------------------------------------------------------- kernel
// EXTRA: the epilogue applies EpiExtra's row scale / residual and the softplus
// epilogue (a separate instantiation, so the plain projections carry none of
// its code: the kernel is sensitive to instruction-cache misses)
template <int MODE, typename TO, bool EXTRA>
__global__ void __launch_bounds__(Cfg<MODE>::WARPS * 32, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b0,
               const __grid_constant__ CUtensorMap map_b1, const __grid_constant__ CUtensorMap map_y,
               const Params p) {
    using C = Cfg<MODE>;
    constexpr int BN = C::BN;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *gbase = smem_raw + (base - raw);
    const uint32_t out_base = base + C::STAGES * C::STAGE_BYTES;   // 1024-aligned
    const uint32_t bars = out_base + (uint32_t)staging_bytes<MODE, TO>();
    // barriers: full[S] empty[S] xform[S] a_empty[LO] acc_full[NACC] acc_empty[NACC]; tmem slot
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (C::STAGES + s); };
    auto xform = [&](int s) { return bars + 8u * (2 * C::STAGES + s); };
    auto a_empty = [&](int l) { return bars + 8u * (3 * C::STAGES + l); };
    auto acc_full = [&](int b) { return bars + 8u * (3 * C::STAGES + C::LO + b); };
    auto acc_empty = [&](int b) { return bars + 8u * (3 * C::STAGES + C::LO + C::NACC + b); };
    const uint32_t tmem_slot = bars + 8u * (3 * C::STAGES + C::LO + 2 * C::NACC);
    uint32_t *tmem_slot_ptr = reinterpret_cast<uint32_t *>(gbase + (tmem_slot - base));
    // stage s: A (BM rows) | W (BN rows) [| W_lo (BN rows)], each 128 B per row
    auto tile = [&](int s, int t) {
        return base + (uint32_t)(s * C::STAGE_BYTES) +
               (t == 0 ? 0u : (uint32_t)(TILE_BYTES + (t - 1) * BN * 128));
    };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_n = (int)ceil_div(p.N, BN);
    const int num_mn = (int)ceil_div(p.M, BM) * num_n;
    const int nsplit = p.ksplit > 1 ? p.ksplit : 1;
    const int num_tiles = num_mn * nsplit;
    const int nk = (int)ceil_div(p.K, C::BK);
    const int kbs = nsplit > 1 ? p.kbs : nk;         // k-blocks per split
    // tile t -> output tile origin and its k-block range [kb0, kb1)
    auto coords = [&](int t, int64_t &m0, int64_t &n0, int &z, int &kb0, int &kb1) {
        z = t / num_mn;
        const int r = t - z * num_mn;
        m0 = (int64_t)(r / num_n) * BM;
        n0 = (int64_t)(r % num_n) * BN;
        kb0 = z * kbs;
        kb1 = kb0 + kbs < nk ? kb0 + kbs : nk;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
            mbar_init(xform(s), 128);
        }
        for (int l = 0; l < C::LO; ++l) mbar_init(a_empty(l), 1);
        for (int b = 0; b < C::NACC; ++b) {
            mbar_init(acc_full(b), 1);
            mbar_init(acc_empty(b), 128 * C::EPG);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(tmem_slot), "r"(C::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot_ptr;

    // weight tiles of the first stages while the previous kernel of a
    // programmatic chain finishes (the stages are free at the start)
    int pre = 0;
    if (p.w_early && warp == 0 && lane == 0 && (int)blockIdx.x < num_tiles) {
        int64_t m0, n0;
        int z, kb0, kb1;
        coords((int)blockIdx.x, m0, n0, z, kb0, kb1);
        for (int kb = kb0; kb < kb1 && pre < C::STAGES; ++kb, ++pre) {
            mbar_expect_tx(full(pre), C::TX);
            tma_load_2d(tile(pre, 1), &map_b0, full(pre), kb * C::BK, (int32_t)n0);
            if (MODE == F32X3) tma_load_2d(tile(pre, 2), &map_b1, full(pre), kb * C::BK, (int32_t)n0);
        }
    }
    pdl_wait();        // inputs (and outputs' previous readers) of a chained launch
    pdl_trigger();

    if (warp == 0) {
        // ---------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t g = 0;  // k-blocks issued by this CTA
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                int64_t m0, n0;
                int z, kb0, kb1;
                coords(t, m0, n0, z, kb0, kb1);
                for (int kb = kb0; kb < kb1; ++kb, ++g) {
                    const int s = g % C::STAGES;
                    const uint32_t ph = (g / C::STAGES) & 1;
                    const int32_t kc = kb * C::BK;
                    if ((int)g >= pre) {     // else: stage s was armed and its W loaded above
                        if (!mbar_wait(empty(s), ph ^ 1, 1)) { ok = false; break; }
                        mbar_expect_tx(full(s), C::TX);
                        tma_load_2d(tile(s, 1), &map_b0, full(s), kc, (int32_t)n0);
                        if (MODE == F32X3) tma_load_2d(tile(s, 2), &map_b1, full(s), kc, (int32_t)n0);
                    }
                    tma_load_2d(tile(s, 0), &map_a, full(s), kc, (int32_t)m0);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        uint32_t g = 0;
        int it = 0;
        bool ok = true;
        if (lane == 0) {
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
                const int b = it % C::NACC;
                ok = mbar_wait(acc_empty(b), ((it / C::NACC) & 1) ^ 1, 8);
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t acc = tmem + (uint32_t)(b * C::ACC_COLS);
                int64_t m0, n0;
                int z, kb0, kb1;
                coords(t, m0, n0, z, kb0, kb1);
                for (int kb = kb0; kb < kb1; ++kb, ++g) {
                    const int s = g % C::STAGES;
                    const uint32_t ph = (g / C::STAGES) & 1;
                    ok = mbar_wait(full(s), ph, 2);
                    if (ok && MODE == F32X3) ok = mbar_wait(xform(s), ph, 3);
                    if (!ok) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                    for (int kk = 0; kk < C::BK / C::KSTEP; ++kk) {
                        const uint32_t koff = kk * 32;  // 32 bytes of K per MMA
                        const uint32_t acc0 = (kb > kb0 || kk > 0) ? 1u : 0u;
                        if (MODE == F32X3) {
                            const uint32_t ah = tmem + C::A_COL + (uint32_t)((g % C::LO) * 64 + kk * C::KSTEP);
                            const uint32_t al = ah + 32;
                            const uint64_t bh = smem_desc(tile(s, 1) + koff);
                            const uint64_t bl = smem_desc(tile(s, 2) + koff);
                            // big: accumulator (kk & 1) (4 K slices per k-block,
                            // so both are initialised in k-block 0)
                            mma_ts(acc + (uint32_t)((kk & 1) * BN), ah, bh, (kb > kb0 || kk > 1) ? 1u : 0u);
                            mma_ts(acc + 2 * BN, ah, bl, acc0);
                            mma_ts(acc + 2 * BN, al, bh, 1u);
                        } else {
                            mma<MODE>(acc, smem_desc(tile(s, 0) + koff), smem_desc(tile(s, 1) + koff),
                                      acc0);
                        }
                    }
                    mma_commit(empty(s));   // frees the stage once these MMAs have read it
                    if (MODE == F32X3) mma_commit(a_empty(g % C::LO));
                }
                if (ok) mma_commit(acc_full(b));  // this tile's accumulator is complete
            }
        }
        __syncwarp();
        // free TMEM after the epilogue drained the last tile (bounded)
        const int it_all = __shfl_sync(0xffffffffu, it, 0);
        if (it_all > 0) {
            const int last = it_all - 1;
            mbar_wait(acc_empty(last % C::NACC), (last / C::NACC) & 1, 4);
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     ::"r"(tmem), "r"(C::TMEM_COLS));
    } else if (MODE == F32X3 && warp < C::EPI0) {
        // ------------------------------------------- A split into TMEM, F32
        const int q = warp & 3;                // TMEM lane quarter of this warp
        const int row = q * 32 + lane;
        uint32_t g = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            int64_t m0, n0;
            int z, kb0, kb1;
            coords(t, m0, n0, z, kb0, kb1);
            for (int kb = kb0; kb < kb1; ++kb, ++g) {
                const int s = g % C::STAGES;
                const uint32_t ph = (g / C::STAGES) & 1;
                const int l = g % C::LO;
                // split as soon as the tile has landed; wait for the TMEM slot
                // (freed when the MMAs of k-block g - LO complete) only before
                // storing into it
                bool w = mbar_wait(full(s), ph, 5);
                if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
                // this thread's row of the 128B-swizzled A tile: logical 16-byte
                // chunk c sits at physical chunk c ^ (row & 7)
                const uint8_t *arow = gbase + (tile(s, 0) - base) + row * 128;
                uint32_t hi[32], lo[32];
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const float4 v = *reinterpret_cast<const float4 *>(arow + ((c ^ (row & 7)) << 4));
                    const float a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float h = tf32_rn(a[e]);
                        hi[4 * c + e] = __float_as_uint(h);
                        lo[4 * c + e] = __float_as_uint(tf32_rn(a[e] - h));
                    }
                }
                w = mbar_wait(a_empty(l), ((g / C::LO) & 1) ^ 1, 7);
                if (!__all_sync(0xffffffffu, w)) { ok = false; break; }  // tcgen05.st is warp-wide
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + C::A_COL + l * 64;
                tmem_st32(ta, hi);
                tmem_st32(ta + 32, lo);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                mbar_arrive(xform(s));
            }
        }
    } else if (warp >= C::EPI0) {
        // ---------------------------------------------------------- epilogue
        const int q = warp & 3;                 // TMEM lane quarter this warp may read
        constexpr int VEC = 16 / (int)sizeof(TO);     // outputs per 16-byte chunk
        constexpr int BOXC = 128 / (int)sizeof(TO);   // columns per 128-byte staging row
        constexpr int WCOLS = BN / C::EPG;            // accumulator columns of this warp
        constexpr int HCOLS = WCOLS / C::SPLIT;       // columns staged at a time
        constexpr int CBH = HCOLS / 32;               // 32-column blocks per staged part
        static_assert(HCOLS % BOXC == 0 || HCOLS < BOXC, "staging boxes");
        // this warp's column group: columns cg0 .. cg0 + WCOLS of the tile
        const int cg0 = ((warp - C::EPI0) >> 2) * WCOLS;
        // this warp's staging: HCOLS / BOXC boxes of 32 rows x 128 B, 128B-swizzled
        const uint32_t wst = out_base + (uint32_t)((warp - C::EPI0) * 32 * HCOLS * sizeof(TO));
        uint8_t *wst_g = gbase + (wst - base);
        TO *Y = static_cast<TO *>(p.y);
        const TO *bias = static_cast<const TO *>(p.bias);
        // write staged part `part` (columns part * HCOLS ...) of this warp's 32 rows
        auto flush = [&](int part, int64_t m0, int64_t n0, int z) {
            const int64_t c0 = cg0 + (int64_t)part * HCOLS;
            if (p.tma_store) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
#pragma unroll
                    for (int bx = 0; bx < HCOLS / BOXC; ++bx) {
                        if (nsplit > 1)   // split-K partials: (N, M, split), rows >= M clipped
                            tma_store_3d(&map_y, wst + bx * 32 * 128, (int32_t)(n0 + c0 + bx * BOXC),
                                         (int32_t)(m0 + q * 32), z);
                        else
                            tma_store_2d(&map_y, wst + bx * 32 * 128, (int32_t)(n0 + c0 + bx * BOXC),
                                         (int32_t)(m0 + q * 32));
                    }
                    bulk_commit();
                }
            } else {
                // plain stores with the column remap: row rr of this warp's slab
                __syncwarp();
                for (int rr = 0; rr < 32; ++rr) {
                    const int64_t m = m0 + q * 32 + rr;
                    if (m >= p.M) break;
#pragma unroll
                    for (int c4 = 0; c4 < CBH; ++c4) {
                        const int col = c4 * 32 + lane;
                        const int64_t n = n0 + c0 + col;
                        if (n >= p.N) continue;
                        const int box = col / BOXC, ce = col % BOXC;
                        const uint8_t *src = wst_g + box * (32 * 128) + rr * 128 +
                                             (((ce / VEC) ^ (rr & 7)) << 4) + (ce % VEC) * sizeof(TO);
                        const int64_t dst = n + (n >= p.n1 ? p.off1 : 0) + (n >= p.n2 ? p.off2 : 0);
                        Y[m * p.ld_y + dst] = *reinterpret_cast<const TO *>(src);
                    }
                }
                __syncwarp();
            }
        };
        int it = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
            int64_t m0, n0;
            int z, kb0, kb1;
            coords(t, m0, n0, z, kb0, kb1);
            const int b = it % C::NACC;
            bool w = mbar_wait(acc_full(b), (it / C::NACC) & 1, 6);
            if (!__all_sync(0xffffffffu, w)) break;   // tcgen05.ld is warp-collective
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            // the previous tile's stores must have read the staging tile
            if (lane == 0) bulk_wait_read0();
            __syncwarp();
            const uint32_t acc = tmem + (uint32_t)(b * C::ACC_COLS) + ((uint32_t)(q * 32) << 16);
            const int64_t m_row = m0 + q * 32 + lane;     // the output row this thread drains
            const bool row_ok = m_row < p.M;
            const float rscale = (p.row_scale && row_ok) ? p.row_scale[m_row] : 1.0f;
            const TO *rrow = static_cast<const TO *>(p.resid) + (row_ok ? m_row : 0) * p.ld_r;
            uint32_t ra[32], rb[32], rc[32];
#pragma unroll 1
            for (int cb = 0; cb < WCOLS / 32; ++cb) {
                const int cbase = cg0 + cb * 32;     // tile column of this 32-column block
                if (C::SPLIT > 1 && cb > 0 && cb % CBH == 0) {
                    // staging full: store the finished part, then reuse the buffer
                    flush(cb / CBH - 1, m0, n0, z);
                    if (p.tma_store && lane == 0) bulk_wait_read0();
                    __syncwarp();
                }
                float v[32];
                if (MODE == F32X3) {
                    // the three accumulators of this 32-column block in one round trip
                    tmem_ld32_async(acc + cbase, ra);
                    tmem_ld32_async(acc + BN + cbase, rb);
                    tmem_ld32_async(acc + 2 * BN + cbase, rc);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        v[j] = (__uint_as_float(ra[j]) + __uint_as_float(rb[j])) + __uint_as_float(rc[j]);
                } else {
                    tmem_ld32_async(acc + cbase, ra);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(ra[j]);
                }
                // each optional term behind ONE branch per column block: a
                // per-element test would make every not-taken softplus body a
                // jump into a new instruction-cache line (measured: 6.7 us of
                // drain per tile instead of 0.8)
                if (EXTRA && p.row_scale) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] *= rscale;
                }
                if (bias) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int64_t n = n0 + cbase + j;
                        v[j] += (n < p.N) ? io<TO>::to_f(bias[n]) : 0.0f;
                    }
                }
                if (EXTRA && p.epi == MB2_EPI_SOFTPLUS) {
                    // dt_proj's softplus (_mamba.py:219-220) on the value the
                    // reference would have stored in its dtype
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = softplus_f(io<TO>::round(v[j]));
                }
                if (EXTRA && p.silu_from >= 0 && n0 + cbase + 31 >= p.silu_from) {
                    // in_proj's z half: SiLU(z) on the value stored in TO
                    const int64_t nb = n0 + cbase;
                    if (nb >= p.silu_from) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = silu_f(io<TO>::round(v[j]));
                    } else {
                        for (int j = 0; j < 32; ++j)
                            if (nb + j >= p.silu_from) v[j] = silu_f(io<TO>::round(v[j]));
                    }
                }
                if (EXTRA && p.resid && row_ok) {
                    // residual add: this row's 32 columns, 16 bytes at a time
                    // (the host guarantees 16-byte rows and N % VEC == 0)
#pragma unroll
                    for (int c = 0; c < 32 / VEC; ++c) {
                        const int64_t nb = n0 + cbase + c * VEC;
                        if (nb < p.N) {
                            const uint4 u = *reinterpret_cast<const uint4 *>(rrow + nb);
                            const TO *e = reinterpret_cast<const TO *>(&u);
#pragma unroll
                            for (int k = 0; k < VEC; ++k) v[c * VEC + k] += io<TO>::to_f(e[k]);
                        }
                    }
                }
                // row `lane` of box cbl*32/BOXC: its 16-byte chunks at c ^ (row & 7)
                const int cbl = cb % CBH;
                const int box = (cbl * 32) / BOXC;
                const int col0 = (cbl * 32) % BOXC;         // element offset in the box row
                uint8_t *rowp = wst_g + box * (32 * 128) + lane * 128;
#pragma unroll
                for (int c = 0; c < 32 / VEC; ++c) {
                    const int chunk = (col0 / VEC) + c;
                    uint4 pk4;
                    uint32_t *pw = reinterpret_cast<uint32_t *>(&pk4);
                    if (sizeof(TO) == 4) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) pw[e] = __float_as_uint(v[c * VEC + e]);
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[c * VEC + 2 * e],
                                                                            v[c * VEC + 2 * e + 1]);
                            pw[e] = *reinterpret_cast<const uint32_t *>(&h2);
                        }
                    }
                    *reinterpret_cast<uint4 *>(rowp + ((chunk ^ (lane & 7)) << 4)) = pk4;
                }
            }
            // TMEM drained: the MMA warp may start the next tile in this buffer
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            mbar_arrive(acc_empty(b));
            flush(C::SPLIT - 1, m0, n0, z);
        }
        if (lane == 0) bulk_wait0();   // stores complete before the CTA exits
    }
}

#include "gemm_f16x3.cuh"
#include "gemm_f16w.cuh"

}  // namespace tc

// ------------------------------------------------------------------- host
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static int g_num_sms = 0;

static int get_encode() {
    if (g_encode) return MB2_OK;
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return fail(MB2_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return MB2_OK;
}

// 2D row-major map: rows x cols elements, box (box_rows x 128 bytes), 128B swizzle.
static int make_map_t(CUtensorMap *map, const void *ptr, int64_t rows, int64_t cols, int64_t ld,
                      CUtensorMapDataType type, size_t es, int box_rows) {
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
    cuuint32_t box[2] = {(cuuint32_t)(128 / es), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, type, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MB2_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return MB2_OK;
}
// The same with 64-byte boxes and 64B swizzle (fp16 operands of the wide F16X3 kernel).
static int make_map_sw64(CUtensorMap *map, const void *ptr, int64_t rows, int64_t cols,
                         int64_t ld, CUtensorMapDataType type, size_t es, int box_rows) {
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
    cuuint32_t box[2] = {(cuuint32_t)(64 / es), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, type, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MB2_ERR_CUDA, "cuTensorMapEncodeTiled (64B) failed (%d)", (int)r);
    return MB2_OK;
}
static int make_map(CUtensorMap *map, const void *ptr, int64_t rows, int64_t cols, int64_t ld,
                    bool bf16, int box_rows) {
    return make_map_t(map, ptr, rows, cols, ld,
                      bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                      bf16 ? 2 : 4, box_rows);
}

template <int MODE, typename TO, bool EXTRA>
static int launch_tc(const CUtensorMap &a, const CUtensorMap &b0, const CUtensorMap &b1,
                     const CUtensorMap &ym, const tc::Params &p, cudaStream_t st, bool pdl = false) {
    auto kern = tc::gemm_tc_kernel<MODE, TO, EXTRA>;
    constexpr size_t smem = tc::smem_bytes<MODE, TO>();
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(MB2_ERR_CUDA, "gemm_tc smem attribute: %s", cudaGetErrorString(e));
    if (g_num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    const int64_t tiles = ceil_div(p.M, (int64_t)tc::BM) * ceil_div(p.N, (int64_t)tc::Cfg<MODE>::BN) *
                          (p.ksplit > 1 ? p.ksplit : 1);
    const unsigned grid = (unsigned)(tiles < g_num_sms ? tiles : g_num_sms);
    const cudaError_t le = launch_kernel(pdl, kern, dim3(grid), dim3(tc::Cfg<MODE>::WARPS * 32),
                                         smem, st, a, b0, b1, ym, p);
    if (le != cudaSuccess) return fail(MB2_ERR_CUDA, "gemm_tc_kernel launch: %s", cudaGetErrorString(le));
    return check_launch("gemm_tc_kernel");
}

// Partial sums of a split-K launch: (split, M, N) fp32 in scratch, written
// through a 3D map whose box clips at M (a 128-row tile of a few-row GEMM
// must not spill into the next split's rows).
static int make_map_partials(CUtensorMap *map, float *ptr, int64_t M, int64_t N, int64_t ks) {
    cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)ks};
    cuuint64_t strides[2] = {(cuuint64_t)(N * 4), (cuuint64_t)(M * N * 4)};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, ptr, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MB2_ERR_CUDA, "cuTensorMapEncodeTiled (3D) failed (%d)", (int)r);
    return MB2_OK;
}

// The splits added in a fixed order (deterministic), then the epilogue terms
// in the order of the single-pass epilogue; one output element per thread.
__global__ void tc_splitk_reduce_kernel(const float *__restrict__ P, int ks, int64_t M, int64_t N,
                                        const float *__restrict__ bias,
                                        const float *__restrict__ row_scale, int epi,
                                        const float *__restrict__ resid, int64_t ld_r,
                                        float *__restrict__ y, int64_t ld_y, int64_t n1,
                                        int64_t off1, int64_t n2, int64_t off2,
                                        int64_t silu_from) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= M * N) return;
    const int64_t m = i / N, n = i - m * N;
    // four independent partial sums keep four loads in flight; combined in a
    // fixed order, so the result does not depend on timing
    const int64_t mn = M * N;
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    int z = 0;
    // unrolled so that up to 32 partial loads are in flight at once
#pragma unroll 8
    for (; z + 4 <= ks; z += 4) {
        a0 += P[(z + 0) * mn + i];
        a1 += P[(z + 1) * mn + i];
        a2 += P[(z + 2) * mn + i];
        a3 += P[(z + 3) * mn + i];
    }
    for (; z < ks; ++z) a0 += P[z * mn + i];
    float v = (a0 + a1) + (a2 + a3);
    if (row_scale) v *= row_scale[m];
    if (bias) v += bias[n];
    if (epi == MB2_EPI_SOFTPLUS) v = softplus_f(v);
    if (silu_from >= 0 && n >= silu_from) v = silu_f(v);
    if (resid) v += resid[m * ld_r + n];
    y[m * ld_y + n + (n >= n1 ? off1 : 0) + (n >= n2 ? off2 : 0)] = v;
}

// fp32 GEMM of few rows (the decode step) on the tensor cores: K split over
// about one CTA per SM, partial sums in scratch, then the reduction.
static int gemm_tc_splitk(const void *x, int64_t ld_x, const float *w_split, const void *bias,
                          void *y, int64_t ld_y, int64_t M, int64_t N, int64_t K, int64_t n1,
                          int64_t off1, int64_t n2, int64_t off2, int epi, cudaStream_t st,
                          bool *used, const EpiExtra &ex) {
    using CF = tc::Cfg<tc::F32X3>;
    if (!aligned(x, 16) || (ld_x * 4) % 16 != 0 || (K * 4) % 16 != 0 || (N * 4) % 16 != 0)
        return MB2_OK;
    const float *b0 = w_split, *b1 = w_split + N * K;
    if (!aligned(b0, 16) || !aligned(b1, 16) || !aligned(ex.scratch, 16)) return MB2_OK;
    if (g_num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    const int64_t nk = ceil_div(K, (int64_t)CF::BK);
    const int64_t mn = ceil_div(M, (int64_t)tc::BM) * ceil_div(N, (int64_t)CF::BN);
    int64_t ks = ceil_div((int64_t)g_num_sms, mn);
    ks = ks < nk / 2 ? ks : nk / 2;                      // >= 2 k-blocks per split
    const int64_t cap = (int64_t)(ex.scratch_bytes / ((size_t)M * N * sizeof(float)));
    ks = ks < cap ? ks : cap;
    if (ks < 2) return MB2_OK;
    const int64_t kbs = ceil_div(nk, ks);
    ks = ceil_div(nk, kbs);
    MB2_TRY(get_encode());
    CUtensorMap ma, mb0, mb1, my;
    MB2_TRY(make_map(&ma, x, M, K, ld_x, false, 128));
    MB2_TRY(make_map(&mb0, b0, N, K, K, false, CF::BN));
    MB2_TRY(make_map(&mb1, b1, N, K, K, false, CF::BN));
    MB2_TRY(make_map_partials(&my, ex.scratch, M, N, ks));
    tc::Params p{ex.scratch, N, nullptr, M, N, K, N, N, 0, 0, MB2_EPI_NONE, 1, nullptr, nullptr, 0,
                 (int)ks, (int)kbs};
    p.w_early = ex.pdl == PDL_WEIGHTS_EARLY ? 1 : 0;
    MB2_TRY((launch_tc<tc::F32X3, float, false>(ma, mb0, mb1, my, p, st, ex.pdl != PDL_NONE)));
    *used = true;
    if (ex.defer_splits) {            // the consumer sums the partials itself
        *ex.defer_splits = (int)ks;
        return MB2_OK;
    }
    const cudaError_t le = launch_kernel(
        ex.pdl != PDL_NONE, tc_splitk_reduce_kernel, dim3((unsigned)ceil_div(M * N, (int64_t)256)),
        dim3(256), 0, st, ex.scratch, (int)ks, M, N, static_cast<const float *>(bias),
        ex.row_scale, epi, static_cast<const float *>(ex.resid), ex.ld_r, static_cast<float *>(y),
        ld_y, n1, off1, n2, off2, ex.silu_from);
    if (le != cudaSuccess)
        return fail(MB2_ERR_CUDA, "tc_splitk_reduce_kernel launch: %s", cudaGetErrorString(le));
    MB2_TRY(check_launch("tc_splitk_reduce_kernel"));
    *used = true;
    return MB2_OK;
}

// Tensor-core path when it applies (large M, aligned operands); *used reports it.
int gemm_tc(int dtype, const void *x, int64_t ld_x, const void *w, const float *w_split,
            const void *bias, void *y, int64_t ld_y, int64_t M, int64_t N, int64_t K,
            int64_t n1, int64_t off1, int64_t n2, int64_t off2, int epi, cudaStream_t st,
            bool *used, const EpiExtra &ex) {
    *used = false;
    const bool bf16 = dtype == MB2_BF16;
    const size_t es = bf16 ? 2 : 4;
    if (N < 16 || K < 16 || M < 1) return MB2_OK;
    if (!bf16 && !w_split) return MB2_OK;                   // exact-fp32 path requested
    if (M < 256) {
        // few rows: fp32 with scratch splits K on the tensor cores; else the
        // CUDA-core kernel
        if (bf16 || !ex.scratch) return MB2_OK;
        return gemm_tc_splitk(x, ld_x, w_split, bias, y, ld_y, M, N, K, n1, off1, n2, off2, epi, st,
                              used, ex);
    }
    // TMA: 16-byte aligned bases and row strides
    if (!aligned(x, 16) || (ld_x * es) % 16 != 0 || (K * es) % 16 != 0) return MB2_OK;
    // the residual is read in 16-byte pieces
    if (ex.resid && (!aligned(ex.resid, 16) || (ex.ld_r * es) % 16 != 0 || (N * es) % 16 != 0))
        return MB2_OK;
    const void *b0 = bf16 ? w : (const void *)w_split;
    const void *b1 = bf16 ? w : (const void *)(w_split + N * K);
    if (!aligned(b0, 16) || !aligned(b1, 16)) return MB2_OK;
    MB2_TRY(get_encode());
    CUtensorMap ma, mb0, mb1, my;
    MB2_TRY(make_map(&ma, x, M, K, ld_x, bf16, 128));
    const int bn = bf16 ? tc::Cfg<tc::BF16>::BN : tc::Cfg<tc::F32X3>::BN;
    MB2_TRY(make_map(&mb0, b0, N, K, K, bf16, bn));
    MB2_TRY(make_map(&mb1, b1, N, K, K, bf16, bn));
    const bool remap = (n1 < N && off1 != 0) || (n2 < N && off2 != 0);
    const bool tma_store = !remap && aligned(y, 16) && (ld_y * es) % 16 == 0;
    if (tma_store) MB2_TRY(make_map(&my, y, M, N, ld_y, bf16, 32));
    else my = mb0;  // unused
    tc::Params p{y, ld_y, bias, M, N, K, n1, n2, off1, off2, epi, tma_store ? 1 : 0,
                 ex.row_scale, ex.resid, ex.ld_r, 1, 0, ex.silu_from};
    *used = true;
    const bool extra = ex.row_scale || ex.resid || epi == MB2_EPI_SOFTPLUS || ex.silu_from >= 0;
    if (bf16)
        return extra ? launch_tc<tc::BF16, __nv_bfloat16, true>(ma, mb0, mb1, my, p, st)
                     : launch_tc<tc::BF16, __nv_bfloat16, false>(ma, mb0, mb1, my, p, st);
    return extra ? launch_tc<tc::F32X3, float, true>(ma, mb0, mb1, my, p, st)
                 : launch_tc<tc::F32X3, float, false>(ma, mb0, mb1, my, p, st);
}

// ------------------------------------------------------- F16X3 (fp32 GEMM) --
// Partial maxima of |x| over row ranges: CTA b writes the maximum of its rows
// to parts[b] (gridDim.x <= AMAX_PARTS).  Max is order-independent, so the
// result does not depend on timing; nothing needs clearing beforehand.  Each
// warp walks rows two at a time, its lanes over the row's 16-byte pieces,
// so every lane keeps several independent loads in flight (HBM-bound).
__global__ void amax_rows_kernel(const float *__restrict__ x, int64_t ld, int64_t M, int64_t K,
                                 float *__restrict__ parts, int vec) {
    const int64_t per = ceil_div(M, (int64_t)gridDim.x);
    const int64_t r0 = (int64_t)blockIdx.x * per;
    const int64_t r1 = r0 + per < M ? r0 + per : M;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float m = 0.0f;
    for (int64_t r = r0 + warp; r < r1; r += 2 * nw) {
        const float *ra = x + r * ld;
        const float *rb = r + nw < r1 ? x + (r + nw) * ld : ra;   // second row, or the first again
        if (vec) {
            const int w = (int)(K >> 2);
#pragma unroll 4
            for (int c = lane; c < w; c += 32) {
                const float4 u = reinterpret_cast<const float4 *>(ra)[c];
                const float4 v = reinterpret_cast<const float4 *>(rb)[c];
                m = fmaxf(m, fmaxf(fmaxf(fabsf(u.x), fabsf(u.y)), fmaxf(fabsf(u.z), fabsf(u.w))));
                m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            }
        } else {
#pragma unroll 4
            for (int64_t c = lane; c < K; c += 32) m = fmaxf(m, fmaxf(fabsf(ra[c]), fabsf(rb[c])));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __shared__ float wm[32];
    if (lane == 0) wm[warp] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < nw; ++k) m = fmaxf(m, wm[k]);
        parts[blockIdx.x] = m;
    }
}

static int amax_parts(const float *x, int64_t ld, int64_t M, int64_t K, float *parts, int *n,
                      cudaStream_t st) {
    // about 32 KB of x per CTA, and no more than 16 rows per CTA (two per warp)
    int64_t g = ceil_div(M * K, (int64_t)8192);
    const int64_t by_rows = ceil_div(M, (int64_t)16);
    g = g > by_rows ? g : by_rows;
    g = g < tc::F16Cfg::AMAX_PARTS ? g : tc::F16Cfg::AMAX_PARTS;
    g = g < M ? g : M;
    g = g > 1 ? g : 1;
    const int vec = aligned(x, 16) && ld % 4 == 0 && K % 4 == 0;
    amax_rows_kernel<<<(unsigned)g, 256, 0, st>>>(x, ld, M, K, parts, vec);
    *n = (int)g;
    return check_launch("amax_rows_kernel");
}

// W (rows, cols) -> header | hi plane | lo plane (layout of mb2_split_f16).
__global__ void split_f16_kernel(const float *__restrict__ w, int64_t n,
                                 const float *__restrict__ parts, int nparts,
                                 __half *__restrict__ hi, __half *__restrict__ lo,
                                 float *__restrict__ inv_out) {
    __shared__ float sm[32];
    float m = 0.0f;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) m = fmaxf(m, parts[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); ++k) m = fmaxf(m, sm[k]);
        sm[0] = m;
    }
    __syncthreads();
    const int e = tc::f16_scale_exp(sm[0]);
    const float sc = tc::pow2f(e);
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i == 0) *inv_out = tc::pow2f(-e);
    if (i >= n) return;
    const float v = w[i] * sc;
    const __half h = __float2half_rn(v);
    hi[i] = h;
    lo[i] = __float2half_rn(v - __half2float(h));
}

constexpr size_t kF16Header = 4096;      // inv scale at 0, partial maxima from 2048

size_t split_f16_bytes(int64_t rows, int64_t cols) {
    return kF16Header + (size_t)rows * cols * 2 * sizeof(__half);
}

// Launch one F16X3 instantiation: persistent, one CTA per SM; pairs of CTAs
// (2-SM clusters) when PAIR, as many pairs as can be resident at once.
template <bool EXTRA, bool PAIR, bool CODES = false>
static int launch_f16(const CUtensorMap &ma, const CUtensorMap &mwh, const CUtensorMap &mwl,
                      const CUtensorMap &my, const tc::F16Params &fp, int64_t M, int64_t N,
                      cudaStream_t st) {
    auto kern = tc::gemm_f16x3_kernel<EXTRA, PAIR, CODES>;
    constexpr size_t smem = tc::f16_smem_bytes<PAIR, CODES>();
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(MB2_ERR_CUDA, "gemm_f16x3 smem attribute: %s", cudaGetErrorString(e));
    if (g_num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    const int64_t tiles = ceil_div(M, (int64_t)(PAIR ? 2 * tc::BM : tc::BM)) *
                          ceil_div(N, (int64_t)tc::F16Cfg::BN);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.blockDim = dim3(tc::F16Cfg::WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    int64_t units = g_num_sms;
    if (PAIR) {
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        static int max_pairs = 0;          // resident pairs of this kernel on this GPU
        if (max_pairs == 0) {
            cfg.gridDim = dim3((unsigned)(2 * (g_num_sms / 2)));
            int n = 0;
            e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
            if (e != cudaSuccess || n <= 0)
                return fail(MB2_ERR_CUDA, "gemm_f16x3: no resident SM pairs (%s)", cudaGetErrorString(e));
            max_pairs = n;
        }
        units = max_pairs;
    }
    units = tiles < units ? tiles : units;
    cfg.gridDim = dim3((unsigned)(PAIR ? 2 * units : units));
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, kern) == cudaSuccess &&
        fa.maxThreadsPerBlock < tc::F16Cfg::WARPS * 32)
        return fail(MB2_ERR_CUDA, "gemm_f16x3_kernel: %d registers per thread allow only %d threads",
                    fa.numRegs, fa.maxThreadsPerBlock);
    e = cudaLaunchKernelEx(&cfg, kern, ma, mwh, mwl, my, fp);
    if (e != cudaSuccess) return fail(MB2_ERR_CUDA, "gemm_f16x3_kernel launch: %s", cudaGetErrorString(e));
    return check_launch("gemm_f16x3_kernel");
}

// The wide F16X3 kernel (128 x 256 tiles): persistent, one CTA per SM.
template <bool EXTRA, int XFW, bool CODES = false>
static int launch_f16w(const CUtensorMap &ma, const CUtensorMap &mwh, const CUtensorMap &mwl,
                       const CUtensorMap &my, const tc::F16Params &fp, int64_t M, int64_t N,
                       cudaStream_t st, const CUtensorMap *mal = nullptr) {
    auto kern = tc::gemm_f16w_kernel<EXTRA, XFW, CODES>;
    using CW = tc::F16WCfg<XFW, CODES>;
    constexpr size_t smem = tc::f16w_smem_bytes<CODES>();
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(MB2_ERR_CUDA, "gemm_f16w smem attribute: %s", cudaGetErrorString(e));
    if (g_num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    const int64_t tiles = ceil_div(M, (int64_t)tc::BM) * ceil_div(N, (int64_t)CW::BN);
    const unsigned grid = (unsigned)(tiles < g_num_sms ? tiles : g_num_sms);
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, kern) == cudaSuccess && fa.maxThreadsPerBlock < CW::WARPS * 32)
        return fail(MB2_ERR_CUDA, "gemm_f16w_kernel: %d registers per thread allow only %d threads",
                    fa.numRegs, fa.maxThreadsPerBlock);
    kern<<<grid, CW::WARPS * 32, smem, st>>>(ma, mwh, mwl, my, mal ? *mal : ma, fp);
    return check_launch("gemm_f16w_kernel");
}

// x (M, K) fp32 -> x_hi, x_lo (M, K) fp16 and inv[m] = 2^-e_m, one warp per
// row: e_m puts the row's largest |x| in [2^14, 2^15) (the F16X3 scale, per
// row instead of per tensor), hi = fp16_rn(x 2^e_m), lo = fp16_rn(x 2^e_m - hi).
// Rows are 16-byte aligned and K % 4 == 0 (the wide kernel's conditions).
__global__ void split_rows_kernel(const float *__restrict__ x, int64_t ld, int64_t M, int64_t K,
                                  __half *__restrict__ hi, __half *__restrict__ lo,
                                  float *__restrict__ inv) {
    const int lane = threadIdx.x & 31;
    const int64_t wpb = blockDim.x >> 5;
    for (int64_t m = (int64_t)blockIdx.x * wpb + (threadIdx.x >> 5); m < M; m += gridDim.x * wpb) {
        const float4 *row = reinterpret_cast<const float4 *>(x + m * ld);
        const int64_t k4 = K >> 2;
        float mx = 0.0f;
        for (int64_t i = lane; i < k4; i += 32) {
            const float4 v = row[i];
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const int e = tc::f16_scale_exp(mx);
        const float sc = tc::pow2f(e);
        if (lane == 0) inv[m] = tc::pow2f(-e);
        uint2 *hrow = reinterpret_cast<uint2 *>(hi + m * K);
        uint2 *lrow = reinterpret_cast<uint2 *>(lo + m * K);
        for (int64_t i = lane; i < k4; i += 32) {
            const float4 v = row[i];
            const float a0 = v.x * sc, a1 = v.y * sc, a2 = v.z * sc, a3 = v.w * sc;
            const uint32_t h01 = tc::pack_h2(a0, a1), h23 = tc::pack_h2(a2, a3);
            const float2 f01 = tc::unpack_h2(h01), f23 = tc::unpack_h2(h23);
            hrow[i] = make_uint2(h01, h23);
            lrow[i] = make_uint2(tc::pack_h2(a0 - f01.x, a1 - f01.y), tc::pack_h2(a2 - f23.x, a3 - f23.y));
        }
    }
}

// fp32 GEMM through the F16X3 kernel; *used reports whether it ran.  parts:
// scratch of AMAX_PARTS floats for x's partial maxima.  pair: 1 = 256-row
// tiles on pairs of SMs, 0 or -1 = 128-row tiles on single SMs (the default:
// measured on the block's projections, the pairs took 8-13 % longer -- each
// SM loads 25 % fewer bytes per multiply-add, but every k-block waits for the
// second CTA's ready signal, and the kernel is bound by that pipeline latency
// rather than by L2 bandwidth).
int gemm_f16x3(const float *x, int64_t ld_x, const void *w16, const void *bias, float *y,
               int64_t ld_y, int64_t M, int64_t N, int64_t K, int64_t n1, int64_t off1,
               int64_t n2, int64_t off2, int epi, cudaStream_t st, bool *used,
               const EpiExtra &ex, float *parts, int pair) {
    *used = false;
    if (!w16 || !parts || M < 1 || N < 16 || K < 16) return MB2_OK;
    if (!aligned(x, 16) || (ld_x * 4) % 16 != 0 || K % 8 != 0 || !aligned(w16, 256)) return MB2_OK;
    if (ex.resid && (!aligned(ex.resid, 16) || ex.ld_r % 4 != 0 || N % 4 != 0)) return MB2_OK;
    const bool two = pair > 0;
    // 256-wide tiles for N >= 256 unless single-SM 128-wide tiles were asked
    // for (pair == 0) or SM pairs (pair == 1)
    const bool wide = pair < 0 && N >= 256;
    const char *wb = static_cast<const char *>(w16);
    const __half *whi = reinterpret_cast<const __half *>(wb + kF16Header);
    const __half *wlo = whi + N * K;
    MB2_TRY(get_encode());
    // many 256-wide column tiles: split x once, by rows, into the caller's scratch
    const size_t split_need = (size_t)M * K * 2 * sizeof(__half) + (size_t)M * sizeof(float) + 256;
    const bool presplit = wide && ceil_div(N, (int64_t)256) >= 4 && ex.xsplit &&
                          ex.xsplit_bytes >= split_need && aligned(ex.xsplit, 256);
    int nparts = ex.amax_n;        // > 0: the kernel that wrote x left its maxima in parts
    if (nparts <= 0 && !presplit) MB2_TRY(amax_parts(x, ld_x, M, K, parts, &nparts, st));
    if (presplit) {
        __half *xh = static_cast<__half *>(ex.xsplit);
        __half *xl = xh + M * K;
        float *inv = reinterpret_cast<float *>(reinterpret_cast<char *>(xl + M * K));
        const int64_t blocks = ceil_div(M, (int64_t)8);
        split_rows_kernel<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, st>>>(
            x, ld_x, M, K, xh, xl, inv);
        MB2_TRY(check_launch("split_rows_kernel"));
        CUtensorMap mah, mal, mwh, mwl, my;
        MB2_TRY(make_map_sw64(&mah, xh, M, K, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 128));
        MB2_TRY(make_map_sw64(&mal, xl, M, K, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 128));
        MB2_TRY(make_map_sw64(&mwh, whi, N, K, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 256));
        MB2_TRY(make_map_sw64(&mwl, wlo, N, K, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 256));
        const bool remap = (n1 < N && off1 != 0) || (n2 < N && off2 != 0);
        const bool tma_store = !remap && aligned(y, 16) && (ld_y * 4) % 16 == 0;
        if (tma_store)
            MB2_TRY(make_map_sw64(&my, y, M, N, ld_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 32));
        else my = mah;  // unused
        tc::F16Params fp{};
        fp.g = tc::Params{y, ld_y, bias, M, N, K, n1, n2, off1, off2, epi, tma_store ? 1 : 0,
                          ex.row_scale, ex.resid, ex.ld_r, 1, 0, ex.silu_from};
        fp.w_inv = reinterpret_cast<const float *>(w16);
        fp.x_row_inv = inv;
        const bool extra = ex.row_scale || ex.resid || epi == MB2_EPI_SOFTPLUS || ex.silu_from >= 0;
        const int rc = extra ? launch_f16w<true, 0>(mah, mwh, mwl, my, fp, M, N, st, &mal)
                             : launch_f16w<false, 0>(mah, mwh, mwl, my, fp, M, N, st, &mal);
        MB2_TRY(rc);
        *used = true;
        return MB2_OK;
    }
    if (wide) {
        CUtensorMap ma, mwh, mwl, my;
        MB2_TRY(make_map(&ma, x, M, K, ld_x, false, 128));
        MB2_TRY(make_map_sw64(&mwh, whi, N, K, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 256));
        MB2_TRY(make_map_sw64(&mwl, wlo, N, K, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 256));
        const bool remap = (n1 < N && off1 != 0) || (n2 < N && off2 != 0);
        const bool tma_store = !remap && aligned(y, 16) && (ld_y * 4) % 16 == 0;
        if (tma_store)
            MB2_TRY(make_map_sw64(&my, y, M, N, ld_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 32));
        else my = ma;  // unused
        tc::F16Params fp{};
        fp.g = tc::Params{y, ld_y, bias, M, N, K, n1, n2, off1, off2, epi, tma_store ? 1 : 0,
                          ex.row_scale, ex.resid, ex.ld_r, 1, 0, ex.silu_from};
        fp.x_parts = parts;
        fp.n_parts = nparts;
        fp.w_inv = reinterpret_cast<const float *>(w16);
        const bool extra = ex.row_scale || ex.resid || epi == MB2_EPI_SOFTPLUS || ex.silu_from >= 0;
        // four transform warps for long K (out_proj: measured 0.190 -> 0.171 ms),
        // two otherwise (in_proj and dt_proj were slower with four)
        const bool xf4 = K >= 1024;
        const int rc = extra ? (xf4 ? launch_f16w<true, 4>(ma, mwh, mwl, my, fp, M, N, st)
                                    : launch_f16w<true, 2>(ma, mwh, mwl, my, fp, M, N, st))
                             : (xf4 ? launch_f16w<false, 4>(ma, mwh, mwl, my, fp, M, N, st)
                                    : launch_f16w<false, 2>(ma, mwh, mwl, my, fp, M, N, st));
        MB2_TRY(rc);
        *used = true;
        return MB2_OK;
    }
    CUtensorMap ma, mwh, mwl, my;
    const int wrows = two ? tc::F16Stage<true>::WROWS : tc::F16Stage<false>::WROWS;
    MB2_TRY(make_map(&ma, x, M, K, ld_x, false, 128));
    MB2_TRY(make_map_t(&mwh, whi, N, K, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, wrows));
    MB2_TRY(make_map_t(&mwl, wlo, N, K, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, wrows));
    const bool remap = (n1 < N && off1 != 0) || (n2 < N && off2 != 0);
    const bool tma_store = !remap && aligned(y, 16) && (ld_y * 4) % 16 == 0;
    if (tma_store) MB2_TRY(make_map(&my, y, M, N, ld_y, false, 32));
    else my = ma;  // unused
    tc::F16Params fp{};
    fp.g = tc::Params{y, ld_y, bias, M, N, K, n1, n2, off1, off2, epi, tma_store ? 1 : 0,
                      ex.row_scale, ex.resid, ex.ld_r, 1, 0, ex.silu_from};
    fp.x_parts = parts;
    fp.n_parts = nparts;
    fp.w_inv = reinterpret_cast<const float *>(w16);
    const bool extra = ex.row_scale || ex.resid || epi == MB2_EPI_SOFTPLUS || ex.silu_from >= 0;
    int rc;
    if (two)
        rc = extra ? launch_f16<true, true>(ma, mwh, mwl, my, fp, M, N, st)
                   : launch_f16<false, true>(ma, mwh, mwl, my, fp, M, N, st);
    else
        rc = extra ? launch_f16<true, false>(ma, mwh, mwl, my, fp, M, N, st)
                   : launch_f16<false, false>(ma, mwh, mwl, my, fp, M, N, st);
    MB2_TRY(rc);
    *used = true;
    return MB2_OK;
}

// y = x (q s)^T for a quantised weight with one scale per row (int8 / int4
// codes q given as fp16 in `codes16`, N x K, 256-byte aligned): the F16X3
// kernel in its CODES form, the scale applied per output column in the
// epilogue.  *used reports whether it ran.
int gemm_f16x3_codes(const float *x, int64_t ld_x, const void *codes16, const float *col_scale,
                     const void *bias, float *y, int64_t ld_y, int64_t M, int64_t N, int64_t K,
                     int64_t n1, int64_t off1, int64_t n2, int64_t off2, int epi, cudaStream_t st,
                     bool *used, const EpiExtra &ex, float *parts) {
    *used = false;
    if (!codes16 || !col_scale || !parts || M < 1 || N < 16 || K < 16) return MB2_OK;
    if (!aligned(x, 16) || (ld_x * 4) % 16 != 0 || K % 8 != 0 || !aligned(codes16, 256)) return MB2_OK;
    if (ex.resid && (!aligned(ex.resid, 16) || ex.ld_r % 4 != 0 || N % 4 != 0)) return MB2_OK;
    MB2_TRY(get_encode());
    if (N >= 256) {
        // 128 x 256 tiles; x split once by rows when there are many column tiles
        const size_t split_need = (size_t)M * K * 2 * sizeof(__half) + (size_t)M * sizeof(float) + 256;
        const bool presplit = ceil_div(N, (int64_t)256) >= 4 && ex.xsplit &&
                              ex.xsplit_bytes >= split_need && aligned(ex.xsplit, 256);
        int nparts = ex.amax_n;
        if (nparts <= 0 && !presplit) MB2_TRY(amax_parts(x, ld_x, M, K, parts, &nparts, st));
        CUtensorMap ma, mal, mw, my;
        tc::F16Params fp{};
        if (presplit) {
            __half *xh = static_cast<__half *>(ex.xsplit);
            __half *xl = xh + M * K;
            float *inv = reinterpret_cast<float *>(xl + M * K);
            const int64_t blocks = ceil_div(M, (int64_t)8);
            split_rows_kernel<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, st>>>(
                x, ld_x, M, K, xh, xl, inv);
            MB2_TRY(check_launch("split_rows_kernel"));
            MB2_TRY(make_map_sw64(&ma, xh, M, K, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 128));
            MB2_TRY(make_map_sw64(&mal, xl, M, K, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 128));
            fp.x_row_inv = inv;
        } else {
            MB2_TRY(make_map(&ma, x, M, K, ld_x, false, 128));
            mal = ma;
            fp.x_parts = parts;
            fp.n_parts = nparts;
        }
        MB2_TRY(make_map_sw64(&mw, codes16, N, K, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 256));
        const bool remap = (n1 < N && off1 != 0) || (n2 < N && off2 != 0);
        const bool tma_store = !remap && aligned(y, 16) && (ld_y * 4) % 16 == 0;
        if (tma_store)
            MB2_TRY(make_map_sw64(&my, y, M, N, ld_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 32));
        else my = ma;  // unused
        fp.g = tc::Params{y, ld_y, bias, M, N, K, n1, n2, off1, off2, epi, tma_store ? 1 : 0,
                          ex.row_scale, ex.resid, ex.ld_r, 1, 0, ex.silu_from};
        fp.col_scale = col_scale;
        const bool extra = ex.row_scale || ex.resid || epi == MB2_EPI_SOFTPLUS || ex.silu_from >= 0;
        int rc;
        if (presplit)
            rc = extra ? launch_f16w<true, 0, true>(ma, mw, mw, my, fp, M, N, st, &mal)
                       : launch_f16w<false, 0, true>(ma, mw, mw, my, fp, M, N, st, &mal);
        else
            rc = extra ? launch_f16w<true, 2, true>(ma, mw, mw, my, fp, M, N, st)
                       : launch_f16w<false, 2, true>(ma, mw, mw, my, fp, M, N, st);
        MB2_TRY(rc);
        *used = true;
        return MB2_OK;
    }
    int nparts = ex.amax_n;
    if (nparts <= 0) MB2_TRY(amax_parts(x, ld_x, M, K, parts, &nparts, st));
    CUtensorMap ma, mw, my;
    MB2_TRY(make_map(&ma, x, M, K, ld_x, false, 128));
    MB2_TRY(make_map_t(&mw, codes16, N, K, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                       tc::F16Stage<false, true>::WROWS));
    const bool remap = (n1 < N && off1 != 0) || (n2 < N && off2 != 0);
    const bool tma_store = !remap && aligned(y, 16) && (ld_y * 4) % 16 == 0;
    if (tma_store) MB2_TRY(make_map(&my, y, M, N, ld_y, false, 32));
    else my = ma;  // unused
    tc::F16Params fp{};
    fp.g = tc::Params{y, ld_y, bias, M, N, K, n1, n2, off1, off2, epi, tma_store ? 1 : 0,
                      ex.row_scale, ex.resid, ex.ld_r, 1, 0, ex.silu_from};
    fp.x_parts = parts;
    fp.n_parts = nparts;
    fp.w_inv = nullptr;
    fp.col_scale = col_scale;
    const bool extra = ex.row_scale || ex.resid || epi == MB2_EPI_SOFTPLUS || ex.silu_from >= 0;
    const int rc = extra ? launch_f16<true, false, true>(ma, mw, mw, my, fp, M, N, st)
                         : launch_f16<false, false, true>(ma, mw, mw, my, fp, M, N, st);
    MB2_TRY(rc);
    *used = true;
    return MB2_OK;
}

}  // namespace mb2

extern "C" size_t mb2_split_f16_bytes(int64_t rows, int64_t cols) {
    if (rows < 0 || cols < 0) return 0;
    return mb2::split_f16_bytes(rows, cols);
}

namespace mb2 {
int split_f16(const float *w, int64_t rows, int64_t cols, void *out, cudaStream_t st) {
    char *ob = static_cast<char *>(out);
    float *parts = reinterpret_cast<float *>(ob + 2048);
    int nparts = 0;
    MB2_TRY(amax_parts(w, cols, rows, cols, parts, &nparts, st));
    __half *hi = reinterpret_cast<__half *>(ob + kF16Header);
    const int64_t n = rows * cols;
    split_f16_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(w, n, parts, nparts, hi, hi + n,
                                                                 reinterpret_cast<float *>(ob));
    return check_launch("split_f16_kernel");
}
}  // namespace mb2

extern "C" int mb2_split_f16(const float *w, int64_t rows, int64_t cols, void *out,
                             mb2_stream_t stream) {
    MB2_REQUIRE(rows >= 0 && cols >= 0, MB2_ERR_SHAPE, "split_f16: negative size");
    MB2_REQUIRE(out && mb2::aligned(out, 256), MB2_ERR_ALIGN,
                "split_f16: output must be 256-byte aligned");
    if (rows * cols == 0) return MB2_OK;
    MB2_REQUIRE(w, MB2_ERR_ARG, "split_f16: null pointer");
    return mb2::split_f16(w, rows, cols, out, (cudaStream_t)stream);
}

extern "C" size_t mb2_linear_f16_scratch_bytes(void) {
    return mb2::tc::F16Cfg::AMAX_PARTS * sizeof(float);
}

extern "C" int mb2_linear_f16(const float *x, int64_t ld_x, const void *w_f16, const float *bias,
                              float *y, int64_t ld_y, int64_t M, int64_t N, int64_t K,
                              int epilogue, int sm_pair, void *scratch, mb2_stream_t stream) {
    MB2_REQUIRE(sm_pair >= -1 && sm_pair <= 1, MB2_ERR_ARG, "linear_f16: sm_pair must be -1, 0 or 1");
    MB2_REQUIRE(epilogue == MB2_EPI_NONE || epilogue == MB2_EPI_SOFTPLUS, MB2_ERR_ARG,
                "linear_f16: bad epilogue");
    MB2_REQUIRE(M >= 0 && N >= 0 && K >= 0, MB2_ERR_SHAPE, "linear_f16: negative size");
    MB2_REQUIRE(ld_x >= K && ld_y >= N, MB2_ERR_SHAPE, "linear_f16: leading dimension too small");
    if (M == 0 || N == 0) return MB2_OK;
    MB2_REQUIRE(x && w_f16 && y && scratch, MB2_ERR_ARG, "linear_f16: null pointer");
    MB2_REQUIRE(N >= 16 && K >= 16 && K % 8 == 0, MB2_ERR_UNSUPPORTED,
                "linear_f16: needs N >= 16, K >= 16 and K a multiple of 8 (got N %lld, K %lld)",
                (long long)N, (long long)K);
    MB2_REQUIRE(mb2::aligned(x, 16) && (ld_x * 4) % 16 == 0 && mb2::aligned(w_f16, 256),
                MB2_ERR_ALIGN, "linear_f16: x rows must be 16-byte aligned, the split weight "
                "256-byte aligned");
    bool used = false;
    MB2_TRY(mb2::gemm_f16x3(x, ld_x, w_f16, bias, y, ld_y, M, N, K, N, 0, N, 0, epilogue,
                            (cudaStream_t)stream, &used, mb2::EpiExtra{},
                            static_cast<float *>(scratch), sm_pair));
    MB2_REQUIRE(used, MB2_ERR_UNSUPPORTED, "linear_f16: operands not supported");
    return MB2_OK;
}

// ------------------------------------------------------------- TF32 split ---
// hi = tf32_rn(w), lo = tf32_rn(w - hi): w == hi + lo up to 2^-22 |w|.  A
// derived cache of fp32 weights for the 3-term TF32 tensor-core GEMM.
namespace mb2 {
__global__ void split_tf32_kernel(const float *__restrict__ w, float *__restrict__ out,
                                  int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = w[i];
    const float h = tc::tf32_rn(v);
    out[i] = h;
    out[n + i] = tc::tf32_rn(v - h);
}
}  // namespace mb2

extern "C" int mb2_split_tf32(const float *w, float *out, int64_t numel, mb2_stream_t stream) {
    MB2_REQUIRE(numel >= 0, MB2_ERR_SHAPE, "split_tf32: negative size");
    if (numel == 0) return MB2_OK;
    MB2_REQUIRE(w && out, MB2_ERR_ARG, "split_tf32: null pointer");
    mb2::split_tf32_kernel<<<(unsigned)mb2::ceil_div(numel, 256), 256, 0, (cudaStream_t)stream>>>(
        w, out, numel);
    return mb2::check_launch("split_tf32_kernel");
}

extern "C" int mb2_device_status(int *code, int clear) {
    MB2_REQUIRE(code, MB2_ERR_ARG, "device_status: null pointer");
    cudaError_t e = cudaMemcpyFromSymbol(code, mb2::g_mb2_device_error, sizeof(int));
    if (e != cudaSuccess) return mb2::fail(MB2_ERR_CUDA, "device_status: %s", cudaGetErrorString(e));
    if (clear) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(mb2::g_mb2_device_error, &zero, sizeof(int));
        if (e != cudaSuccess) return mb2::fail(MB2_ERR_CUDA, "device_status: %s", cudaGetErrorString(e));
    }
    return MB2_OK;
}
