// F16X3 on 128 x 256 tiles ("wide"), included by gemm_tc.cu inside namespace
// mb2::tc after gemm_f16x3.cuh (it shares that file's scaled fp16 split, the
// accumulation scheme and its helpers).
//
// The same arithmetic as gemm_f16x3_kernel -- x and W scaled by powers of two
// and split into fp16 hi + lo, three kind::f16 MMAs per K step (x_hi W_hi into
// a segment accumulator P drained into fp32 registers every SEG k-blocks,
// x_hi W_lo + x_lo W_hi into Q over the whole K) -- with 256-wide MMAs: a
// 128 x 256 x 16 MMA does twice the work of a 128 x 128 x 16 one in about
// 1.2x its time on the B200 (measured with the MMAs alone), which is what
// bounds the 128-wide kernel.
//
// What changes with the width:
//   * TMEM holds P (256 columns) and Q (256 columns) only, so x's split goes
//     to shared memory and the MMAs read both operands from there (SS form).
//     The split is made in place: a k-block of 32 fp32 K values per row
//     (128 B, 128B swizzle, as TMA loads it) becomes x_hi and x_lo rows of 32
//     fp16 (64 B each, 64B swizzle) in the same 16 KB; the transform warps
//     read their rows, meet at a named barrier, then write.  Or x arrives
//     split already (see XFW below).
//   * P is single-buffered: at a segment boundary inside a tile the MMA warp
//     issues the k-block's Q MMAs first and waits for P's drain only before
//     its P MMAs; at a tile boundary it issues P first and waits for Q's drain
//     before the Q MMAs, so the drains overlap MMAs either way.
//   * 16 epilogue warps (four per TMEM lane quarter) drain 64 accumulator
//     columns each into fp32 running sums.
// Shared memory: 4 stages of (A fp32 -> x_hi | x_lo, 16 KB | W_hi 256 x 32
// fp16, 16 KB | W_lo, 16 KB) = 192 KB, plus 32 KB of output staging (2 KB a
// warp: 32 rows x 16 columns per TMA store).  Every mbarrier wait is bounded.

template <int XFW = 2, bool CODES = false> struct F16WCfg {
    static constexpr int BN = 256;
    static constexpr int BK = 32;              // fp32 K values per k-block (one 128 B TMA box)
    static constexpr int SEG = 8;              // k-blocks per hi*hi segment (16 MMAs, as F16X3)
    // CODES: the weight is one plane of a quantised weight's integer codes
    // (exact in fp16), so a stage is 32 KB and 6 fit
    static constexpr int STAGES = CODES ? 6 : 4;
    static constexpr int XF0 = 2;              // transform warps from 2
    static constexpr int XF_WARPS = XFW;
    static constexpr int XF_THREADS = 32 * XF_WARPS;
    static constexpr int RPT = XF_WARPS ? 128 / XF_THREADS : 0;   // rows a transform thread splits
    static constexpr int EPI0 = XF0 + XF_WARPS;    // 16 epilogue warps after them
    static constexpr int WARPS = EPI0 + 16;
    static constexpr int EPI_WARPS = 16;
    static constexpr int EPI_THREADS = 512;
    static constexpr int ECOLS = 64;           // accumulator columns per epilogue warp
    static constexpr uint32_t COL_P = 0;
    static constexpr uint32_t COL_Q = 256;
    static constexpr uint32_t A_BYTES = 128 * 128;       // 128 rows x 32 fp32
    static constexpr uint32_t W_BYTES = 256 * 64;        // 256 rows x 32 fp16
    static constexpr uint32_t STAGE_BYTES = A_BYTES + (CODES ? 1 : 2) * W_BYTES;
};
// output staging: 32 rows x 16 fp32 columns (one 64B-swizzled box) per epilogue warp
constexpr size_t f16w_staging_bytes() { return (size_t)F16WCfg<>::EPI_WARPS * 32 * 16 * sizeof(float); }
template <bool CODES = false> constexpr size_t f16w_smem_bytes() {
    return 1024 + (size_t)F16WCfg<2, CODES>::STAGES * F16WCfg<2, CODES>::STAGE_BYTES +
           f16w_staging_bytes() + 256;
}
static_assert(f16w_smem_bytes<false>() <= 232448 && f16w_smem_bytes<true>() <= 232448,
              "wide F16X3 shared memory above the 227 KB per CTA");

// Shared-memory matrix descriptor of a K-major operand in the 64B-swizzled
// layout (64-byte rows, 8-row atoms of 512 bytes; layout type 4).
__device__ __forceinline__ uint64_t smem_desc64(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | (32ull << 32) | (1ull << 46) |
           (4ull << 61);
}

// kind::f16 MMA, 128 x 256 x 16, both operands from shared memory
__device__ __forceinline__ void mma_ss_f16w(uint32_t tmem_d, uint64_t da, uint64_t db,
                                            uint32_t accum) {
    // D F32 (bits 4-5 = 1), A / B F16 (0), K-major, N >> 3 at 17, M >> 4 at 24
    constexpr uint32_t idesc = (1u << 4) | ((uint32_t)(F16WCfg<>::BN >> 3) << 17) |
                               ((uint32_t)(BM >> 4) << 24);
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accum));
}

// XFW transform warps: 2 (two rows a thread, 20 warps of 96 registers) or 4
// (one row a thread, 22 warps of 80 registers: a faster split, a tighter
// epilogue); the host picks 4 for long K, where the split's latency matters
// more than the epilogue's registers.  XFW = 0: x arrives split already
// (split_rows_kernel: x_hi | x_lo fp16 planes with one power-of-two scale per
// row); TMA loads both halves into the stage as the split would have left
// them, no transform warps run, and the epilogue scales row m by its own
// 2^-e_m (map_al: the x_lo plane; map_a the x_hi plane).
// CODES: W is a quantised weight's codes as fp16 (map_wh; map_wl unused) and
// column n is multiplied by col_scale[n] in the epilogue, as in the 128-wide
// kernel's CODES form: two MMAs per K step (x_hi q, x_lo q).
template <bool EXTRA, int XFW, bool CODES = false>
__global__ void __launch_bounds__(F16WCfg<XFW, CODES>::WARPS * 32, 1)
gemm_f16w_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_wh,
                 const __grid_constant__ CUtensorMap map_wl, const __grid_constant__ CUtensorMap map_y,
                 const __grid_constant__ CUtensorMap map_al, const F16Params fp) {
    constexpr bool PRE = XFW == 0;
    using C = F16WCfg<XFW, CODES>;
    constexpr int BN = C::BN;
    const Params &p = fp.g;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *gbase = smem_raw + (base - raw);
    const uint32_t out_base = base + C::STAGES * C::STAGE_BYTES;
    const uint32_t bars = out_base + (uint32_t)f16w_staging_bytes();
    // full[S] empty[S] xform[S] seg_full seg_empty q_full q_empty; tmem slot
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (C::STAGES + s); };
    auto xform = [&](int s) { return bars + 8u * (2 * C::STAGES + s); };
    const uint32_t seg_full = bars + 8u * (3 * C::STAGES);
    const uint32_t seg_empty = seg_full + 8u;
    const uint32_t q_full = seg_full + 16u;
    const uint32_t q_empty = seg_full + 24u;
    const uint32_t tmem_slot = seg_full + 32u;
    uint32_t *tmem_slot_ptr = reinterpret_cast<uint32_t *>(gbase + (tmem_slot - base));
    // stage s: A (fp32, then x_hi at +0 and x_lo at +8 KB) | W_hi | W_lo
    auto tile_a = [&](int s) { return base + (uint32_t)(s * C::STAGE_BYTES); };
    auto tile_w = [&](int s, int lo) {
        return base + (uint32_t)(s * C::STAGE_BYTES + C::A_BYTES + lo * C::W_BYTES);
    };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_n = (int)ceil_div(p.N, BN);
    const int num_tiles = (int)ceil_div(p.M, BM) * num_n;
    const int nk = (int)ceil_div(p.K, C::BK);
    const int nseg = (nk + C::SEG - 1) / C::SEG;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
            mbar_init(xform(s), C::XF_THREADS);
        }
        mbar_init(seg_full, 1);
        mbar_init(seg_empty, C::EPI_THREADS);
        mbar_init(q_full, 1);
        mbar_init(q_empty, C::EPI_THREADS);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(tmem_slot), "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot_ptr;

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                const int64_t m0 = (int64_t)(t / num_n) * BM;
                const int64_t n0 = (int64_t)(t % num_n) * BN;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % C::STAGES;
                    const uint32_t ph = (g / C::STAGES) & 1;
                    if (!mbar_wait(empty(s), ph ^ 1, 31)) { ok = false; break; }
                    mbar_expect_tx(full(s), C::STAGE_BYTES);
                    const int32_t kc = kb * C::BK;
                    if (PRE) {
                        tma_load_2d(tile_a(s), &map_a, full(s), kc, (int32_t)m0);
                        tma_load_2d(tile_a(s) + C::A_BYTES / 2, &map_al, full(s), kc, (int32_t)m0);
                    } else {
                        tma_load_2d(tile_a(s), &map_a, full(s), kc, (int32_t)m0);
                    }
                    tma_load_2d(tile_w(s, 0), &map_wh, full(s), kc, (int32_t)n0);
                    if (!CODES) tma_load_2d(tile_w(s, 1), &map_wl, full(s), kc, (int32_t)n0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------------------------------------------- MMA issuer
            uint32_t g = 0, gs = 0;
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
                for (int kb = 0; kb < nk && ok; ++kb, ++g) {
                    const int rel = kb % C::SEG;
                    const int s = g % C::STAGES;
                    const uint32_t ph = (g / C::STAGES) & 1;
                    ok = mbar_wait(full(s), ph, 32) && (PRE || mbar_wait(xform(s), ph, 33));
                    if (!ok) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t ahi = tile_a(s), alo = ahi + C::A_BYTES / 2;
                    const uint32_t bh = tile_w(s, 0), bl = tile_w(s, 1);
                    auto issue_p = [&]() {
#pragma unroll
                        for (int kk = 0; kk < C::BK / 16; ++kk)
                            mma_ss_f16w(tmem + C::COL_P, smem_desc64(ahi + kk * 32),
                                        smem_desc64(bh + kk * 32), (rel > 0 || kk > 0) ? 1u : 0u);
                    };
                    auto issue_q = [&]() {
#pragma unroll
                        for (int kk = 0; kk < C::BK / 16; ++kk) {
                            if (CODES) {        // x_lo q (the codes are exact: no W_lo)
                                mma_ss_f16w(tmem + C::COL_Q, smem_desc64(alo + kk * 32),
                                            smem_desc64(bh + kk * 32), (kb > 0 || kk > 0) ? 1u : 0u);
                            } else {
                                mma_ss_f16w(tmem + C::COL_Q, smem_desc64(ahi + kk * 32),
                                            smem_desc64(bl + kk * 32), (kb > 0 || kk > 0) ? 1u : 0u);
                                mma_ss_f16w(tmem + C::COL_Q, smem_desc64(alo + kk * 32),
                                            smem_desc64(bh + kk * 32), 1u);
                            }
                        }
                    };
                    if (rel != 0) {
                        issue_p();
                        issue_q();
                    } else if (kb == 0) {
                        // tile start: P (drained with the previous tile's last
                        // segment) first, then Q once its drain is done
                        ok = mbar_wait(seg_empty, (gs & 1) ^ 1, 34);
                        if (!ok) break;
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        issue_p();
                        ok = mbar_wait(q_empty, (it & 1) ^ 1, 35);
                        if (!ok) break;
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        issue_q();
                    } else {
                        // a segment boundary inside the tile: Q first, P once drained
                        issue_q();
                        ok = mbar_wait(seg_empty, (gs & 1) ^ 1, 36);
                        if (!ok) break;
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        issue_p();
                    }
                    mma_commit(empty(s));           // stage free once these MMAs read it
                    if (rel == C::SEG - 1 || kb == nk - 1) {
                        mma_commit(seg_full);
                        ++gs;
                    }
                }
                if (ok) mma_commit(q_full);
            }
        }
    } else if (!PRE && warp < C::EPI0) {
        // ------------------- x split in place: fp32 rows -> x_hi | x_lo (fp16)
        // thread rows r0 + XF_THREADS h, h < RPT
        const int r0 = (warp - C::XF0) * 32 + lane;
        const float sx = pow2f(f16_scale_exp(warp_amax(fp.x_parts, fp.n_parts)));
        uint32_t g = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            for (int kb = 0; kb < nk; ++kb, ++g) {
                const int s = g % C::STAGES;
                const uint32_t ph = (g / C::STAGES) & 1;
                bool w = mbar_wait(full(s), ph, 37);
                if (!__all_sync(0xffffffffu, w)) ok = false;
                // both transform warps reach the named barrier below, also after
                // an expired wait (they then convert whatever is there)
                uint32_t hi[C::RPT > 0 ? C::RPT : 1][16], lo[C::RPT > 0 ? C::RPT : 1][16];
                uint8_t *a = gbase + (tile_a(s) - base);
#pragma unroll
                for (int h = 0; h < C::RPT; ++h) {
                    // fp32 row r: 128 B, 16-byte chunk c at c ^ (r & 7)
                    const int r = r0 + C::XF_THREADS * h;
                    const uint8_t *arow = a + r * 128;
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const float4 v = *reinterpret_cast<const float4 *>(arow + ((c ^ (r & 7)) << 4));
                        const float a0 = v.x * sx, a1 = v.y * sx, a2 = v.z * sx, a3 = v.w * sx;
                        const uint32_t h01 = pack_h2(a0, a1), h23 = pack_h2(a2, a3);
                        const float2 f01 = unpack_h2(h01), f23 = unpack_h2(h23);
                        hi[h][2 * c] = h01;
                        hi[h][2 * c + 1] = h23;
                        lo[h][2 * c] = pack_h2(a0 - f01.x, a1 - f01.y);
                        lo[h][2 * c + 1] = pack_h2(a2 - f23.x, a3 - f23.y);
                    }
                }
                // all 128 rows read before any is overwritten
                asm volatile("bar.sync 1, %0;" ::"n"(C::XF_THREADS) : "memory");
#pragma unroll
                for (int h = 0; h < C::RPT; ++h) {
                    // x_hi row r at +0, x_lo at +8 KB: 64 B each, 16-byte chunk c
                    // at c ^ ((r >> 1) & 3) (64B swizzle)
                    const int r = r0 + C::XF_THREADS * h;
                    uint8_t *hrow = a + r * 64;
                    uint8_t *lrow = hrow + C::A_BYTES / 2;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint32_t off = (uint32_t)((c ^ ((r >> 1) & 3)) << 4);
                        *reinterpret_cast<uint4 *>(hrow + off) =
                            make_uint4(hi[h][4 * c], hi[h][4 * c + 1], hi[h][4 * c + 2], hi[h][4 * c + 3]);
                        *reinterpret_cast<uint4 *>(lrow + off) =
                            make_uint4(lo[h][4 * c], lo[h][4 * c + 1], lo[h][4 * c + 2], lo[h][4 * c + 3]);
                    }
                }
                // the tensor core reads the split through the async proxy
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(xform(s));
                if (!ok) break;
            }
        }
    } else {
        // ----------------------------------------------------------- epilogue
        const int q = warp & 3;                          // TMEM lane quarter
        const int ch = (warp - C::EPI0) >> 2;            // column quarter: 0-3
        const uint32_t lanes = (uint32_t)(q * 32) << 16;
        const uint32_t ccol = (uint32_t)(ch * C::ECOLS);
        const float inv_x_tensor = PRE ? 1.0f : pow2f(-f16_scale_exp(warp_amax(fp.x_parts, fp.n_parts)));
        const float inv_w = CODES ? 1.0f : *fp.w_inv;
        const uint32_t wst = out_base + (uint32_t)((warp - C::EPI0) * 32 * 64);  // one box
        uint8_t *wst_g = gbase + (wst - base);
        float *Y = static_cast<float *>(p.y);
        const float *bias = static_cast<const float *>(p.bias);
        float acc[C::ECOLS];
        // 16 columns per TMEM load: 64 running sums + 16 loaded values fit the
        // 96 registers a thread of 20 warps gets
        auto drain = [&](uint32_t col) {
            uint32_t r[16];
#pragma unroll
            for (int cb = 0; cb < C::ECOLS / 16; ++cb) {
                tmem_ld16_async(tmem + lanes + col + ccol + cb * 16, r);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) acc[cb * 16 + j] += __uint_as_float(r[j]);
            }
        };
        uint32_t gs = 0;
        int it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
            const int64_t m0 = (int64_t)(t / num_n) * BM;
            const int64_t n0 = (int64_t)(t % num_n) * BN;
#pragma unroll
            for (int j = 0; j < C::ECOLS; ++j) acc[j] = 0.0f;
            for (int sg = 0; sg < nseg; ++sg, ++gs) {
                const bool w = mbar_wait(seg_full, gs & 1, 38);
                if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                drain(C::COL_P);
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                mbar_arrive(seg_empty);
            }
            if (!ok) break;
            {
                const bool w = mbar_wait(q_full, it & 1, 39);
                if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                drain(C::COL_Q);
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                mbar_arrive(q_empty);
            }
            const int64_t m_row = m0 + q * 32 + lane;
            const bool row_ok = m_row < p.M;
            const float rscale = (EXTRA && p.row_scale && row_ok) ? p.row_scale[m_row] : 1.0f;
            const float *rrow = static_cast<const float *>(p.resid) + (row_ok ? m_row : 0) * p.ld_r;
            // x's scale: one per tensor, or (pre-split) this row's own
            const float inv_x = PRE ? (row_ok ? fp.x_row_inv[m_row] : 0.0f) : inv_x_tensor;
#pragma unroll
            for (int cb = 0; cb < C::ECOLS / 32; ++cb) {
                const int64_t c0 = n0 + ch * C::ECOLS + cb * 32;   // first output column
                float *v = acc + cb * 32;
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
                // two stores of 16 columns through this warp's 2 KB box
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const int64_t cs = c0 + 16 * hh;
                    // the previous store from the box must have read it
                    if (lane == 0) bulk_wait_read0();
                    __syncwarp();
                    // row `lane` of the box: 64 B, 16-byte chunk c at c ^ ((row >> 1) & 3)
                    uint8_t *rowp = wst_g + lane * 64;
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        *reinterpret_cast<float4 *>(rowp + ((c ^ ((lane >> 1) & 3)) << 4)) =
                            make_float4(v[16 * hh + 4 * c], v[16 * hh + 4 * c + 1],
                                        v[16 * hh + 4 * c + 2], v[16 * hh + 4 * c + 3]);
                    if (p.tma_store) {
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        __syncwarp();
                        if (lane == 0 && cs < p.N) {
                            tma_store_2d(&map_y, wst, (int32_t)cs, (int32_t)(m0 + q * 32));
                            bulk_commit();
                        }
                    } else {
                        // plain stores with the column remap: lanes 0-15 take
                        // the box's even rows, 16-31 the odd ones
                        __syncwarp();
                        const int cl = lane & 15;
                        const int64_t n = cs + cl;
                        const int64_t dst = n + (n >= p.n1 ? p.off1 : 0) + (n >= p.n2 ? p.off2 : 0);
                        for (int rr = lane >> 4; rr < 32; rr += 2) {
                            const int64_t m = m0 + q * 32 + rr;
                            if (m >= p.M) break;
                            if (n < p.N)
                                Y[m * p.ld_y + dst] = *(reinterpret_cast<const float *>(
                                    wst_g + rr * 64 + (((cl >> 2) ^ ((rr >> 1) & 3)) << 4)) + (cl & 3));
                        }
                        __syncwarp();
                    }
                }
            }
        }
        if (lane == 0) bulk_wait0();
    }
    // every role is done with TMEM (bounded waits: also after an expired one)
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}
