// fp32-faithful GEMM on the fp16 tensor cores ("F16X3"), included by gemm_tc.cu
// inside namespace mb2::tc (it shares that file's primitives and device status).
//
// y = x W^T for fp32 x (M, K) and W (N, K), to fp32 accuracy:
//
//   * Scaled fp16 split.  x and W are each multiplied by a power of two (one per
//     tensor: x by 2^ex so that max|x| 2^ex lies in [2^14, 2^15), W likewise by
//     2^ew, fixed when W is split) and written as hi = fp16_rn(v), lo =
//     fp16_rn(v - hi): 11 + 11 significant bits, the precision of the TF32
//     split, and with the scale no element overflows fp16, while the smallest
//     ones lose only what lies 2^-40 below the tensor's largest element.  W's
//     halves are a derived cache (mb2_split_f16); x is split on the fly by four
//     transform warps that write both halves into tensor memory.
//   * Three kind::f16 MMAs per K step (x_hi W_hi, x_hi W_lo, x_lo W_hi) at the
//     fp16 rate, twice the TF32 rate: the same work as the 3xTF32 path in half
//     the tensor-pipe time.
//   * Bounded accumulation error.  The tensor core truncates when it adds into
//     an fp32 accumulator, so every MMA issued into an accumulator adds up to
//     one ulp of the running sum.  The big x_hi W_hi products go to one of two
//     TMEM accumulators P0 / P1 for a segment of SEG k-blocks only (16 MMAs);
//     the epilogue warps then drain the segment into fp32 registers (round to
//     nearest) while the next segment accumulates into the other one.  The two
//     cross terms, 2^-11 of the result, accumulate over the whole K in a third
//     accumulator Q, where their truncation is 2^-11 smaller again.  The result
//     is 2^-(ex+ew) (sum of segments + Q): exact scalings.
//
// Warps: 0 TMA producer, 1 TMEM owner + MMA issuer, 2-5 transform, 6-13
// epilogue (segment drains, output staging and TMA stores; warps w and w + 4
// share TMEM lane quarter w % 4, one taking columns 0-63, the other 64-127).  TMEM: P0 | P1 | Q
// (128 columns each) | two A slots of 64 columns (hi 32 | lo 32: 64 fp16 of K
// per row, two per 32-bit column).  Shared memory: 3 stages of (A fp32 as two
// 128-row x 32-float boxes | W_hi | W_lo, 128 rows x 64 fp16 each) = 192 KB,
// plus 32 KB of output staging (4 KB per epilogue warp).  Every mbarrier wait
// is bounded.

struct F16Cfg {
    static constexpr int BN = 128;
    static constexpr int BK = 64;              // fp16 K elements per k-block
    static constexpr int SEG = 4;              // k-blocks per hi*hi segment (16 MMAs)
    // 14 warps: registers are allocated in groups of four warps, so the block
    // counts as 16 warps and every thread may use 128 registers
    static constexpr int WARPS = 14;
    static constexpr int EPI0 = 6;             // 8 epilogue warps, two per TMEM lane quarter
    static constexpr int EPI_THREADS = 256;
    static constexpr uint32_t COL_P = 0;       // P0 at 0, P1 at 128
    static constexpr uint32_t COL_Q = 256;
    static constexpr uint32_t COL_A = 384;     // A slot l at 384 + 64 l
    static constexpr int ECOLS = 64;           // accumulator columns per epilogue warp
    static constexpr int AMAX_PARTS = 512;     // partial maxima of x (mb2_amax_parts)
};
// Per-CTA stage geometry.  One SM: a 128 x 128 tile per CTA, 3 stages of
// (A 32 KB | W_hi 16 KB | W_lo 16 KB).  A pair of SMs (cta_group::2): a
// 256 x 128 tile per pair, each CTA loading its 128 rows of A and 64 of the
// 128 rows of W (the MMAs read the two halves from the two CTAs), so a stage
// is 48 KB and 4 of them fit: 25 % fewer bytes from L2 per multiply-add and a
// third more work in flight.
// CODES: the weight operand is a quantised weight's integer codes as fp16
// (exact: |q| <= 127), one plane instead of hi / lo, so a stage is 48 KB and
// 4 fit.
template <bool PAIR, bool CODES = false> struct F16Stage {
    static constexpr int STAGES = (PAIR || CODES) ? 4 : 3;
    static constexpr int WROWS = PAIR ? 64 : 128;        // W rows per CTA
    static constexpr uint32_t W_BYTES = WROWS * 128;
    static constexpr uint32_t STAGE_BYTES = 2 * TILE_BYTES + (CODES ? 1 : 2) * W_BYTES;
};

// output staging: 32 rows x 32 fp32 columns (one 128B-swizzled box) per epilogue warp
constexpr size_t f16_staging_bytes() { return (size_t)8 * 32 * 32 * sizeof(float); }
template <bool PAIR, bool CODES = false> constexpr size_t f16_smem_bytes() {
    return 1024 + (size_t)F16Stage<PAIR, CODES>::STAGES * F16Stage<PAIR, CODES>::STAGE_BYTES +
           f16_staging_bytes() + 256;
}
static_assert(f16_smem_bytes<false>() <= 232448 && f16_smem_bytes<true>() <= 232448 &&
                  f16_smem_bytes<false, true>() <= 232448,
              "F16X3 shared memory above the 227 KB per CTA");

struct F16Params {
    Params g;                       // shapes, output, epilogue terms (split-K unused)
    const float *x_parts;           // partial maxima of |x| (float bits of non-negative values)
    int n_parts;
    const float *w_inv;             // 2^-ew (header of the split weight)
    const float *col_scale;         // CODES: the quantised weight's scale per output column
    const float *x_row_inv;         // x split by rows (split_rows_kernel): 2^-e of each row
};

// Exponent e with amax * 2^e in [2^14, 2^15); 0 for zero or non-finite amax.
__device__ __forceinline__ int f16_scale_exp(float amax) {
    const uint32_t bits = __float_as_uint(amax) & 0x7FFFFFFFu;
    const int be = (int)(bits >> 23);
    if (bits == 0 || be == 0xFF) return 0;
    int e = be == 0 ? 126 : 141 - be;          // 14 - (be - 127); subnormal: as far as allowed
    return e > 126 ? 126 : e;                   // 2^e and 2^-e stay normal
}
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

// max over the partial maxima, reduced by one warp (every lane gets it)
__device__ __forceinline__ float warp_amax(const float *parts, int n) {
    float m = 0.0f;
    for (int i = (int)(threadIdx.x & 31); i < n; i += 32) m = fmaxf(m, parts[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    return m;
}

__device__ __forceinline__ uint32_t pack_h2(float lo_elem, float hi_elem) {
    const __half2 h = __floats2half2_rn(lo_elem, hi_elem);   // .x (low half) = lo_elem
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ float2 unpack_h2(uint32_t v) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&v));
}

// kind::f16 MMA (fp16 A and B, fp32 accumulator), A from tensor memory; in a
// pair (cta_group::2) one MMA computes the pair's 256 rows: A's rows 0-127 and
// D's rows 0-127 in the first CTA's TMEM, 128-255 in the second's, B's 128
// rows split 64 / 64 between the two CTAs' shared memory at the same offset.
template <bool PAIR>
__device__ __forceinline__ void mma_ts_f16(uint32_t tmem_d, uint32_t tmem_a, uint64_t db,
                                           uint32_t accum) {
    // D F32 (bits 4-5 = 1), A / B F16 (0), K-major, N >> 3 at 17, M >> 4 at 24
    constexpr uint32_t idesc = (1u << 4) | ((uint32_t)(F16Cfg::BN >> 3) << 17) |
                               ((uint32_t)((PAIR ? 2 * BM : BM) >> 4) << 24);
    if constexpr (PAIR)
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
            ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(accum));
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
            ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(accum));
}

// Arrive (once MMAs complete) on the barrier at this offset in both CTAs of
// the pair, or in this CTA.
template <bool PAIR>
__device__ __forceinline__ void mma_commit_to(uint32_t bar) {
    if constexpr (PAIR)
        asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster"
                     ".multicast::cluster.b64 [%0], %1;" ::"r"(bar), "h"((uint16_t)3) : "memory");
    else
        mma_commit(bar);
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// the shared::cluster address of `local` (a shared::cta address) in CTA `rank`
__device__ __forceinline__ uint32_t peer_addr(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];"
                 ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
                 ::: "memory");
}

// CODES (single SMs only): W is a quantised weight's codes as fp16 and the
// epilogue multiplies column n by its scale: y = 2^-ex (x_hi + x_lo) q^T s,
// two MMAs per K step (x_hi q, x_lo q) -- the codes are exact, so no W_lo
// term -- and half the weight bytes of the dequantised split.
template <bool EXTRA, bool PAIR, bool CODES = false>
__global__ void __launch_bounds__(F16Cfg::WARPS * 32, 1)
gemm_f16x3_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_wh,
                  const __grid_constant__ CUtensorMap map_wl, const __grid_constant__ CUtensorMap map_y,
                  const F16Params fp) {
    static_assert(!(PAIR && CODES), "codes run on single SMs");
    using C = F16Cfg;
    using G = F16Stage<PAIR, CODES>;
    constexpr int BN = C::BN;
    constexpr int TM = PAIR ? 2 * BM : BM;              // tile rows (per pair)
    const Params &p = fp.g;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *gbase = smem_raw + (base - raw);
    const uint32_t out_base = base + G::STAGES * G::STAGE_BYTES;
    const uint32_t bars = out_base + (uint32_t)f16_staging_bytes();
    // full[S] empty[S] xform[S] peer[S] a_empty[2] seg_full[2] seg_empty[2] q_full q_empty; tmem slot
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (G::STAGES + s); };
    auto xform = [&](int s) { return bars + 8u * (2 * G::STAGES + s); };
    auto peer = [&](int s) { return bars + 8u * (3 * G::STAGES + s); };
    auto a_empty = [&](int l) { return bars + 8u * (4 * G::STAGES + l); };
    auto seg_full = [&](int b) { return bars + 8u * (4 * G::STAGES + 2 + b); };
    auto seg_empty = [&](int b) { return bars + 8u * (4 * G::STAGES + 4 + b); };
    const uint32_t q_full = bars + 8u * (4 * G::STAGES + 6);
    const uint32_t q_empty = bars + 8u * (4 * G::STAGES + 7);
    const uint32_t tmem_slot = bars + 8u * (4 * G::STAGES + 8);
    uint32_t *tmem_slot_ptr = reinterpret_cast<uint32_t *>(gbase + (tmem_slot - base));
    // stage s: A box 0 (k 0-31) | A box 1 (k 32-63) | W_hi | W_lo
    auto tile_a = [&](int s, int box) { return base + (uint32_t)(s * G::STAGE_BYTES + box * TILE_BYTES); };
    auto tile_w = [&](int s, int lo) {
        return base + (uint32_t)(s * G::STAGE_BYTES + 2 * TILE_BYTES + lo * G::W_BYTES);
    };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // pair: rank 0 issues the MMAs; rank 1 relays that its stages are ready
    const uint32_t rank = PAIR ? cluster_rank() : 0;
    const int unit0 = PAIR ? (int)cluster_id() : (int)blockIdx.x;     // first tile
    const int units = PAIR ? (int)cluster_count() : (int)gridDim.x;   // tile stride
    const int num_n = (int)ceil_div(p.N, BN);
    const int num_tiles = (int)ceil_div(p.M, TM) * num_n;
    const int nk = (int)ceil_div(p.K, C::BK);
    const int nseg = (nk + C::SEG - 1) / C::SEG;      // segments per tile
    // the epilogue's drained-accumulator barriers live in rank 0 and count
    // both CTAs' epilogue threads
    constexpr int DRAINERS = (PAIR ? 2 : 1) * C::EPI_THREADS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < G::STAGES; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
            mbar_init(xform(s), 128);
            mbar_init(peer(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(a_empty(b), 1);
            mbar_init(seg_full(b), 1);
            mbar_init(seg_empty(b), DRAINERS);
        }
        mbar_init(q_full, 1);
        mbar_init(q_empty, DRAINERS);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                         ::"r"(tmem_slot), "r"(512));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                         ::"r"(tmem_slot), "r"(512));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    if constexpr (PAIR) cluster_sync();      // both CTAs' barriers exist before any remote use
    else __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot_ptr;

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            for (int t = unit0; t < num_tiles && ok; t += units) {
                const int64_t m0 = (int64_t)(t / num_n) * TM + (int64_t)rank * BM;
                const int64_t n0 = (int64_t)(t % num_n) * BN + (int64_t)rank * G::WROWS;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % G::STAGES;
                    const uint32_t ph = (g / G::STAGES) & 1;
                    if (!mbar_wait(empty(s), ph ^ 1, 11)) { ok = false; break; }
                    mbar_expect_tx(full(s), G::STAGE_BYTES);
                    const int32_t kc = kb * C::BK;
                    tma_load_2d(tile_a(s, 0), &map_a, full(s), kc, (int32_t)m0);
                    tma_load_2d(tile_a(s, 1), &map_a, full(s), kc + 32, (int32_t)m0);
                    tma_load_2d(tile_w(s, 0), &map_wh, full(s), kc, (int32_t)n0);
                    if (!CODES) tma_load_2d(tile_w(s, 1), &map_wl, full(s), kc, (int32_t)n0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && PAIR && rank != 0) {
            // ------------------------------------------ pair: relay (rank 1)
            // a stage of this CTA is ready for the pair's MMAs once it has
            // landed and its A has been split into TMEM
            uint32_t g = 0;
            bool ok = true;
            const uint32_t leader_peer0 = peer_addr(peer(0), 0);
            for (int t = unit0; t < num_tiles && ok; t += units) {
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % G::STAGES;
                    const uint32_t ph = (g / G::STAGES) & 1;
                    ok = mbar_wait(full(s), ph, 22) && mbar_wait(xform(s), ph, 23);
                    if (!ok) break;
                    mbar_arrive_cluster(leader_peer0 + 8u * s);
                }
            }
        } else if (lane == 0) {
            // ----------------------------------------------------- MMA issuer
            uint32_t g = 0, gs = 0;
            int it = 0;
            bool ok = true;
            for (int t = unit0; t < num_tiles && ok; t += units, ++it) {
                uint32_t pcol = 0;
                for (int kb = 0; kb < nk && ok; ++kb, ++g) {
                    const int rel = kb % C::SEG;
                    if (rel == 0) {
                        // this segment's accumulator was drained two segments ago
                        // (in a pair: by both CTAs' epilogues, the other one remotely)
                        ok = mbar_wait_cluster(seg_empty(gs & 1), ((gs >> 1) & 1) ^ 1, 12);
                        if (ok && kb == 0) ok = mbar_wait_cluster(q_empty, (it & 1) ^ 1, 13);
                        if (!ok) break;
                        pcol = C::COL_P + (gs & 1) * BN;
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    }
                    const int s = g % G::STAGES;
                    const uint32_t ph = (g / G::STAGES) & 1;
                    ok = mbar_wait(full(s), ph, 14) && mbar_wait(xform(s), ph, 15) &&
                         (!PAIR || mbar_wait_cluster(peer(s), ph, 24));
                    if (!ok) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                    for (int kk = 0; kk < C::BK / 16; ++kk) {
                        const uint32_t ah = tmem + C::COL_A + (g & 1) * 64 + kk * 8;
                        const uint64_t bh = smem_desc(tile_w(s, 0) + kk * 32);
                        mma_ts_f16<PAIR>(tmem + pcol, ah, bh, (rel > 0 || kk > 0) ? 1u : 0u);
                        if (CODES) {
                            mma_ts_f16<PAIR>(tmem + C::COL_Q, ah + 32, bh, (kb > 0 || kk > 0) ? 1u : 0u);
                        } else {
                            const uint64_t bl = smem_desc(tile_w(s, 1) + kk * 32);
                            mma_ts_f16<PAIR>(tmem + C::COL_Q, ah, bl, (kb > 0 || kk > 0) ? 1u : 0u);
                            mma_ts_f16<PAIR>(tmem + C::COL_Q, ah + 32, bh, 1u);
                        }
                    }
                    mma_commit_to<PAIR>(empty(s));        // stages free once these MMAs read them
                    mma_commit_to<PAIR>(a_empty(g & 1));  // and the A slots
                    if (rel == C::SEG - 1 || kb == nk - 1) {
                        mma_commit_to<PAIR>(seg_full(gs & 1));
                        ++gs;
                    }
                }
                if (ok) mma_commit_to<PAIR>(q_full);
            }
        }
    } else if (warp < C::EPI0) {
        // --------------------------------------- x split into TMEM (scaled fp16)
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const float sx = pow2f(f16_scale_exp(warp_amax(fp.x_parts, fp.n_parts)));
        uint32_t g = 0;
        bool ok = true;
        for (int t = unit0; t < num_tiles && ok; t += units) {
            for (int kb = 0; kb < nk; ++kb, ++g) {
                const int s = g % G::STAGES;
                const uint32_t ph = (g / G::STAGES) & 1;
                bool w = mbar_wait(full(s), ph, 18);
                if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
                uint32_t hi[32], lo[32];
#pragma unroll
                for (int box = 0; box < 2; ++box) {
                    // this thread's row of the 128B-swizzled box: logical 16-byte
                    // chunk c at physical chunk c ^ (row & 7)
                    const uint8_t *arow = gbase + (tile_a(s, box) - base) + row * 128;
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const float4 v = *reinterpret_cast<const float4 *>(arow + ((c ^ (row & 7)) << 4));
                        const float a0 = v.x * sx, a1 = v.y * sx, a2 = v.z * sx, a3 = v.w * sx;
                        const uint32_t h01 = pack_h2(a0, a1), h23 = pack_h2(a2, a3);
                        const float2 f01 = unpack_h2(h01), f23 = unpack_h2(h23);
                        const int j = box * 16 + c * 2;          // column of elements 2j, 2j + 1
                        hi[j] = h01;
                        hi[j + 1] = h23;
                        lo[j] = pack_h2(a0 - f01.x, a1 - f01.y);
                        lo[j + 1] = pack_h2(a2 - f23.x, a3 - f23.y);
                    }
                }
                w = mbar_wait(a_empty(g & 1), ((g >> 1) & 1) ^ 1, 19);
                if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + C::COL_A + (g & 1) * 64;
                tmem_st32(ta, hi);
                tmem_st32(ta + 32, lo);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                mbar_arrive(xform(s));
            }
        }
    } else {
        // ----------------------------------------------------------- epilogue
        const int q = warp & 3;                          // TMEM lane quarter
        const int ch = (warp - C::EPI0) >> 2;            // column half: 0 or 1
        const uint32_t lanes = (uint32_t)(q * 32) << 16;
        const uint32_t ccol = (uint32_t)(ch * C::ECOLS);
        const float inv_x = pow2f(-f16_scale_exp(warp_amax(fp.x_parts, fp.n_parts)));
        const float inv_w = CODES ? 1.0f : *fp.w_inv;
        const uint32_t wst = out_base + (uint32_t)((warp - C::EPI0) * 32 * 128);  // one box
        uint8_t *wst_g = gbase + (wst - base);
        float *Y = static_cast<float *>(p.y);
        const float *bias = static_cast<const float *>(p.bias);
        float acc[C::ECOLS];
        // add this warp's 64 columns of an accumulator into acc, 32 at a time
        auto drain = [&](uint32_t col) {
            uint32_t r[32];
#pragma unroll
            for (int cb = 0; cb < C::ECOLS / 32; ++cb) {
                tmem_ld32_async(tmem + lanes + col + ccol + cb * 32, r);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[cb * 32 + j] += __uint_as_float(r[j]);
            }
        };
        // drained accumulators are reported to rank 0's barriers
        const uint32_t seg_empty0 = PAIR ? peer_addr(seg_empty(0), 0) : seg_empty(0);
        const uint32_t q_empty0 = PAIR ? peer_addr(q_empty, 0) : q_empty;
        auto drained = [&](uint32_t local, uint32_t remote) {
            if (PAIR && rank != 0) mbar_arrive_cluster(remote);
            else mbar_arrive(local);
        };
        uint32_t gs = 0;
        int it = 0;
        bool ok = true;
        for (int t = unit0; t < num_tiles && ok; t += units, ++it) {
            const int64_t m0 = (int64_t)(t / num_n) * TM + (int64_t)rank * BM;
            const int64_t n0 = (int64_t)(t % num_n) * BN;
#pragma unroll
            for (int j = 0; j < C::ECOLS; ++j) acc[j] = 0.0f;
            for (int sg = 0; sg < nseg; ++sg, ++gs) {
                if (sg == nseg - 1) {
                    // Q first: the MMA warp waits for it before the next tile
                    const bool w = mbar_wait(q_full, it & 1, 20);
                    if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    drain(C::COL_Q);
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    drained(q_empty, q_empty0);
                }
                const bool w = mbar_wait(seg_full(gs & 1), (gs >> 1) & 1, 21);
                if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                drain(C::COL_P + (gs & 1) * BN);
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                drained(seg_empty(gs & 1), seg_empty0 + 8u * (gs & 1));
            }
            if (!ok) break;
            const int64_t m_row = m0 + q * 32 + lane;
            const bool row_ok = m_row < p.M;
            const float rscale = (EXTRA && p.row_scale && row_ok) ? p.row_scale[m_row] : 1.0f;
            const float *rrow = static_cast<const float *>(p.resid) + (row_ok ? m_row : 0) * p.ld_r;
#pragma unroll
            for (int cb = 0; cb < C::ECOLS / 32; ++cb) {
                const int64_t c0 = n0 + ch * C::ECOLS + cb * 32;   // first output column
                float *v = acc + cb * 32;        // in place (constant offsets once unrolled)
                if (CODES) {
                    // column c0 + j's scale: loaded by lane j, broadcast by shuffles
                    const float my_s = c0 + lane < p.N ? fp.col_scale[c0 + lane] : 0.0f;
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        v[j] = (v[j] * inv_x) * __shfl_sync(0xffffffffu, my_s, j);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = v[j] * inv_x * inv_w;
                }
                if (EXTRA && p.row_scale) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] *= rscale;
                }
                if (bias) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] += (c0 + j < p.N) ? bias[c0 + j] : 0.0f;
                }
                if (EXTRA && p.epi == MB2_EPI_SOFTPLUS) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = softplus_f(v[j]);
                }
                if (EXTRA && p.silu_from >= 0 && c0 + 31 >= p.silu_from) {
                    // in_proj's z half: SiLU(z)
                    if (c0 >= p.silu_from) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = silu_f(v[j]);
                    } else {
                        for (int j = 0; j < 32; ++j)
                            if (c0 + j >= p.silu_from) v[j] = silu_f(v[j]);
                    }
                }
                if (EXTRA && p.resid && row_ok) {
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        if (c0 + c * 4 < p.N) {
                            const float4 u = *reinterpret_cast<const float4 *>(rrow + c0 + c * 4);
                            v[c * 4] += u.x; v[c * 4 + 1] += u.y;
                            v[c * 4 + 2] += u.z; v[c * 4 + 3] += u.w;
                        }
                    }
                }
                // the previous store from this warp's box must have read it
                if (lane == 0) bulk_wait_read0();
                __syncwarp();
                // row `lane` of the box: its 16-byte chunks at c ^ (row & 7)
                uint8_t *rowp = wst_g + lane * 128;
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    *reinterpret_cast<float4 *>(rowp + ((c ^ (lane & 7)) << 4)) =
                        make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
                if (p.tma_store) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0 && c0 < p.N) {      // boxes wholly right of N store nothing
                        tma_store_2d(&map_y, wst, (int32_t)c0, (int32_t)(m0 + q * 32));
                        bulk_commit();
                    }
                } else {
                    // plain stores with the column remap: row rr of this warp's slab
                    __syncwarp();
                    const int64_t n = c0 + lane;
                    const int64_t dst = n + (n >= p.n1 ? p.off1 : 0) + (n >= p.n2 ? p.off2 : 0);
                    for (int rr = 0; rr < 32; ++rr) {
                        const int64_t m = m0 + q * 32 + rr;
                        if (m >= p.M) break;
                        if (n < p.N)
                            Y[m * p.ld_y + dst] = *(reinterpret_cast<const float *>(
                                wst_g + rr * 128 + (((lane >> 2) ^ (rr & 7)) << 4)) + (lane & 3));
                    }
                    __syncwarp();
                }
            }
        }
        if (lane == 0) bulk_wait0();
    }
    // every role is done with TMEM (bounded waits: also after an expired one)
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    __syncwarp();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if constexpr (PAIR)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
    // neither CTA of a pair leaves while the other may still signal its barriers
    __syncwarp();
    if constexpr (PAIR) cluster_sync();
}
