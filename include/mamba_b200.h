/*
 * mamba_b200.h -- C ABI of the B200 (sm_100a) Mamba S6 block library.
 *
 * Every entry point takes DEVICE pointers (caller-allocated inputs, outputs
 * and workspace), int64 shapes, a cudaStream_t, and returns an int status
 * (MB2_OK == 0).  Nothing here allocates device memory (except
 * mb2_peer_alloc, whose purpose that is).  On failure
 * mb2_last_error() returns a thread-local message; the Python host layer
 * turns it into RuntimeError / ValueError like the reference's TORCH_CHECK.
 *
 * Layouts are row-major with the last index contiguous.  Activations are
 * token-major: row n = b * seqlen + t.
 *
 * dtype codes: MB2_F32 (float) or MB2_BF16 (__nv_bfloat16 bits as uint16).
 * Scan state h is always float32; conv state is in the activation dtype,
 * matching src/cpu_mamba/_mamba.py:87-101.
 */
#ifndef MAMBA_B200_H
#define MAMBA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *mb2_stream_t; /* == cudaStream_t */

enum mb2_status {
    MB2_OK = 0,
    MB2_ERR_ARG = 1,          /* null pointer / bad enum */
    MB2_ERR_SHAPE = 2,        /* inconsistent or unsupported sizes */
    MB2_ERR_ALIGN = 3,        /* pointer or leading dimension misaligned */
    MB2_ERR_UNSUPPORTED = 4,  /* valid request this build does not handle */
    MB2_ERR_CUDA = 5,         /* launch / runtime error */
    MB2_ERR_WORKSPACE = 6     /* workspace too small */
};

enum mb2_dtype { MB2_F32 = 0, MB2_BF16 = 1 };

/* Linear-layer epilogues: none, or softplus(y) (beta 1, threshold 20) as
 * dt_proj is followed by in src/cpu_mamba/_mamba.py:219-220. */
enum mb2_epilogue { MB2_EPI_NONE = 0, MB2_EPI_SOFTPLUS = 1 };

/* Quantisation schemes of src/cpu_mamba/quant.py:47-53 (QuantConfig.scheme). */
enum mb2_scheme { MB2_Q_NONE = 0, MB2_Q_INT8 = 1, MB2_Q_INT4 = 2, MB2_Q_NF4 = 3 };

/* Library identity and the last error message of the calling thread. */
int mb2_version(void);
const char *mb2_last_error(void);

/* Device-side status of the current device: 0, or the code of the first
 * bounded wait inside a kernel that expired (the kernel then abandoned its
 * tile instead of hanging).  clear != 0 resets it.  Synchronous. */
int mb2_device_status(int *code, int clear);

/* ------------------------------------------------------------------------
 * Selective scan -- drop-in for selective_scan_cpu(x, dt, A, B, C, D) -> y
 * (src/cpu_mamba/selective_scan_cpu.cpp:19-26, bound at
 * src/cpu_mamba/_mamba.py:37-43 and called at :244).
 *   x, dt: (batch, seqlen, d_inner)  A: (d_inner, d_state) (negative)
 *   B, C:  (batch, seqlen, d_state)  D: (d_inner)
 *   y:     (batch, seqlen, d_inner)  -- fully overwritten
 * All contiguous float32; 1 <= d_state <= 256 as in the reference (cpp:39).
 * h0 (batch, d_inner, d_state) may be NULL (zero initial state); h_last may
 * be NULL, else receives the final state (the time loop of
 * forward_with_final_state, src/cpu_mamba/_mamba.py:191-199).
 * ------------------------------------------------------------------------ */
int mb2_selective_scan(const float *x, const float *dt, const float *A,
                       const float *B, const float *C, const float *D,
                       float *y, int64_t batch, int64_t seqlen,
                       int64_t d_inner, int64_t d_state, const float *h0,
                       float *h_last, mb2_stream_t stream);

/* ------------------------------------------------------------------------
 * Causal depthwise conv1d + bias + SiLU over the x half of in_proj's output
 * (src/cpu_mamba/_mamba.py:211-215).
 *   x_in: (batch*seqlen, ld_in) rows, channels [0, d_inner) are read
 *   w: (d_inner, d_conv)  bias: (d_inner) or NULL
 *   xc: (batch*seqlen, ld_out)
 *   conv_tail (batch, d_inner, d_conv-1) or NULL: the last d_conv-1 pre-conv
 *   inputs, zero-left-padded when seqlen < d_conv-1 (_mamba.py:180).
 * ------------------------------------------------------------------------ */
int mb2_conv1d_silu(int dtype, const void *x_in, int64_t ld_in,
                    const void *w, const void *bias, void *xc, int64_t ld_out,
                    void *conv_tail, int64_t batch, int64_t seqlen,
                    int64_t d_inner, int64_t d_conv, mb2_stream_t stream);

/* ------------------------------------------------------------------------
 * Fused scan stage of the block, one kernel: dt = softplus(dt_low W_dt^T +
 * b_dt) (dt_proj, _mamba.py:219-220), A = -exp(A_log) (:222), selective scan
 * + D skip (selective_scan_cpu.cpp:68-83), cast to the activation dtype and
 * SiLU(z) gate (_mamba.py:263-264).
 *   xc:     (N, ld_xc) conv+SiLU output
 *   dt_low, B, C: (N, ld_*) rows of dt_rank / d_state / d_state values
 *           (the three column segments of x_proj's output)
 *   z:      (N, ld_z) gate input (the z half of in_proj's output)
 *   w_dt:   (d_inner, dt_rank), b_dt: (d_inner), A_log: (d_inner, d_state),
 *   D: (d_inner) -- all in the activation dtype
 *   y:      (N, ld_y) gated output; may alias xc (each element of xc is read
 *           before the same element of y is written)
 *   h0 / h_last: optional (batch, d_inner, d_state) float32 initial / final
 *   state (h0 may alias h_last: the single-token step updates h in place).
 * bf16 rows must start on 4-byte boundaries.
 * ------------------------------------------------------------------------ */
int mb2_scan_fused(int dtype, const void *xc, int64_t ld_xc,
                   const void *dt_low, int64_t ld_dl, const void *B,
                   int64_t ld_b, const void *C, int64_t ld_c, const void *z,
                   int64_t ld_z, const void *w_dt, const void *b_dt,
                   const void *A_log, const void *D, const float *h0,
                   float *h_last, void *y, int64_t ld_y, int64_t batch,
                   int64_t seqlen, int64_t d_inner, int64_t d_state,
                   int64_t dt_rank, mb2_stream_t stream);

/* The same stage given dt_proj's output (dt_low W_dt^T + b_dt, e.g. from
 * mb2_linear, which the block forward runs on the tensor cores): the kernel
 * applies the softplus.  dt_pre (N, ld_dt) in the activation dtype; the other
 * arguments as mb2_scan_fused.  y may alias xc. */
int mb2_scan_gated(int dtype, const void *xc, int64_t ld_xc, const void *dt_pre,
                   int64_t ld_dt, const void *B, int64_t ld_b, const void *C,
                   int64_t ld_c, const void *z, int64_t ld_z, const void *A_log,
                   const void *D, const float *h0, float *h_last, void *y,
                   int64_t ld_y, int64_t batch, int64_t seqlen, int64_t d_inner,
                   int64_t d_state, mb2_stream_t stream);

/* mb2_scan_gated with a workspace of mb2_scan_workspace_bytes(batch, seqlen,
 * d_inner, d_state) bytes (0 = none needed): long sequences over few
 * (batch, channel) chains then run in T segments in parallel (segment
 * summaries, a carry pass, the outputs), as the block forward does. */
size_t mb2_scan_workspace_bytes(int64_t batch, int64_t seqlen, int64_t d_inner,
                                int64_t d_state);
int mb2_scan_gated_ws(int dtype, const void *xc, int64_t ld_xc, const void *dt_pre,
                      int64_t ld_dt, const void *B, int64_t ld_b, const void *C,
                      int64_t ld_c, const void *z, int64_t ld_z, const void *A_log,
                      const void *D, const float *h0, float *h_last, void *y,
                      int64_t ld_y, int64_t batch, int64_t seqlen, int64_t d_inner,
                      int64_t d_state, void *workspace, size_t workspace_bytes,
                      mb2_stream_t stream);

/* First-order linear recurrence h[t] = a[t] * h[t-1] + b[t], h[-1] = 0, over
 * the time axis of contiguous (batch, seqlen, inner) tensors: the primitive
 * of the reference's associative scans (src/cpu_mamba/scan_assoc.py:24-55,
 * _associative_prefix_scan, whose trailing dims are flattened into inner).
 * fp32 state; a, b, h all F32 or all BF16.  h may not alias a or b. */
int mb2_linear_recurrence(int dtype, const void *a, const void *b, void *h, int64_t batch,
                          int64_t seqlen, int64_t inner, mb2_stream_t stream);

/* ------------------------------------------------------------------------
 * Linear layer y = x W^T (+ bias): nn.Linear as used by in_proj, x_proj,
 * dt_proj, out_proj (_mamba.py:67,74-75,84).
 *   x: (M, ld_x)  W: (N, K) row-major  bias: (N) or NULL  y: (M, ld_y)
 * dtype F32: fp32-faithful.  With w_split (the TF32 halves of W from
 *   mb2_split_tf32) the tensor cores compute x_hi W_hi + x_hi W_lo + x_lo W_hi;
 *   with w_split == NULL the CUDA-core fp32 FMA kernel runs.
 * dtype BF16: bf16 operands, fp32 accumulation, bf16 output.
 * ------------------------------------------------------------------------ */
int mb2_linear(int dtype, const void *x, int64_t ld_x, const void *w,
               const float *w_split, const void *bias, void *y, int64_t ld_y,
               int64_t M, int64_t N, int64_t K, int epilogue,
               mb2_stream_t stream);

/* Split an fp32 tensor of numel elements into its TF32 halves:
 * out[0:numel] = hi = tf32_rn(w), out[numel:2 numel] = lo = tf32_rn(w - hi),
 * so w == hi + lo to within 2^-22 |w|.  A derived cache of the weights for
 * mb2_linear's F32 tensor-core path (not module state). */
int mb2_split_tf32(const float *w, float *out, int64_t numel,
                   mb2_stream_t stream);

/* fp32-faithful linear layer on the fp16 tensor cores (F16X3): the same
 * y = x W^T (+ bias) as mb2_linear's F32 path, in half its tensor-pipe time.
 * x and W are each scaled by a power of two (x per call from its largest
 * magnitude, W when split) and split into fp16 halves hi + lo (11 + 11
 * significant bits); the MMAs form x_hi W_hi + x_hi W_lo + x_lo W_hi with the
 * big products accumulated in segments of 256 of K that are added up in fp32
 * round-to-nearest, so the rounding error stays that of an fp32 GEMM at any K.
 *   x: (M, ld_x) float32, rows 16-byte aligned   y: (M, ld_y) float32
 *   w_f16: mb2_split_f16's output for W (N, K), 256-byte aligned; K % 8 == 0
 *   sm_pair: -1 (the default, what mb2_block_forward uses) = 128 x 256 output
 *   tiles with 256-wide MMAs when N >= 256, else as 0; 0 = 128 x 128 tiles on
 *   single SMs; 1 = 256 x 128 tiles on pairs of SMs (cta_group::2: each SM of
 *   a pair loads half of W's tile; bit-identical with 0, 8-13 % slower).  All
 *   are fp32-faithful (same segment sums of the same products).
 *   scratch: mb2_linear_f16_scratch_bytes() of device memory (x's partial maxima)
 * No counterpart in the reference (its projections are torch's fp32 GEMMs,
 * _mamba.py:67,74,84); mb2_block_forward uses it for in_proj, x_proj and
 * out_proj when the descriptor carries weight_f16. */
size_t mb2_split_f16_bytes(int64_t rows, int64_t cols);
int mb2_split_f16(const float *w, int64_t rows, int64_t cols, void *out,
                  mb2_stream_t stream);
size_t mb2_linear_f16_scratch_bytes(void);
int mb2_linear_f16(const float *x, int64_t ld_x, const void *w_f16, const float *bias,
                   float *y, int64_t ld_y, int64_t M, int64_t N, int64_t K,
                   int epilogue, int sm_pair, void *scratch, mb2_stream_t stream);

/* ------------------------------------------------------------------------
 * Weight-only quantisation (src/cpu_mamba/quant.py:60-134), bit-exact.
 *   w: (rows, cols) float32
 *   int8: weight_q int8 (rows, cols);  int4 / nf4: uint8 (rows, (cols+1)/2),
 *   even element in the high nibble, odd cols padded (int4 code 0 -> nibble 7,
 *   nf4 index 0).  scale: (rows) float32.
 * ------------------------------------------------------------------------ */
int mb2_quantize(int scheme, const float *w, int64_t rows, int64_t cols,
                 void *weight_q, float *scale, mb2_stream_t stream);

/* dequantize_{int8,int4,nf4} (quant.py:68-69, 90-101, 124-134): w_out (rows, in_dim) f32. */
int mb2_dequantize(int scheme, const void *weight_q, const float *scale,
                   int64_t rows, int64_t in_dim, float *w_out,
                   mb2_stream_t stream);

/* QuantizedLinear.forward (quant.py:188-190): y = x deq(W)^T (+ bias).
 *   x: (M, ld_x) in dtype; y: (M, ld_y) in dtype; weight_q/scale as above. */
int mb2_qlinear(int scheme, int dtype, const void *x, int64_t ld_x,
                const void *weight_q, const float *scale, const void *bias,
                void *y, int64_t ld_y, int64_t M, int64_t N, int64_t K,
                int epilogue, mb2_stream_t stream);

/* Blockwise (grouped) variants -- the reference's roadmap "blockwise NF4
 * (group_size=64)" (README.md:115, :201; not in the reference's code): the
 * formulas above applied to each run of group_size consecutive input columns
 * of a row, scale (rows, ceil(cols / group_size)).  group_size 0 equals the
 * per-row functions; 4-bit schemes need an even group_size. */
int mb2_quantize_grouped(int scheme, const float *w, int64_t rows, int64_t cols,
                         int64_t group_size, void *weight_q, float *scale,
                         mb2_stream_t stream);
int mb2_dequantize_grouped(int scheme, const void *weight_q, const float *scale,
                           int64_t rows, int64_t in_dim, int64_t group_size,
                           float *w_out, mb2_stream_t stream);
int mb2_qlinear_grouped(int scheme, int64_t group_size, int dtype, const void *x,
                        int64_t ld_x, const void *weight_q, const float *scale,
                        const void *bias, void *y, int64_t ld_y, int64_t M,
                        int64_t N, int64_t K, int epilogue, mb2_stream_t stream);

/* ------------------------------------------------------------------------
 * Whole block.  Weights follow the mamba_ssm state_dict (_mamba.py:67-84);
 * a quantised linear passes weight_q/scale instead of weight.
 * ------------------------------------------------------------------------ */
typedef struct mb2_linear_w {
    const void *weight;     /* (out, in) in dtype, or NULL when quantised   */
    const float *weight_split; /* optional (2, out, in) TF32 halves (F32 path)  */
    const void *weight_q;   /* quantised codes, or NULL                      */
    const float *scale;     /* quantised: (out) per-channel scale, or        */
                            /* (out, ceil(in / group_size)) per group        */
    const void *bias;       /* (out) or NULL                                 */
    int scheme;             /* mb2_scheme                                    */
    int64_t group_size;     /* 0: one scale per row (quant.py); else columns */
                            /* per scale group (blockwise, e.g. 64)          */
    const void *weight_f16; /* optional scaled fp16 split of W (mb2_split_f16):  */
                            /* F32 projections of >= 256 rows run on the fp16 */
                            /* tensor cores (mb2_linear_f16)                  */
} mb2_linear_w;

typedef struct mb2_block {
    int64_t d_model, d_inner, d_state, d_conv, dt_rank;
    int dtype;                      /* mb2_dtype of activations and weights */
    mb2_linear_w in_proj, x_proj, dt_proj, out_proj;
    const void *conv_w;             /* (d_inner, d_conv) */
    const void *conv_b;             /* (d_inner) or NULL */
    const void *A_log;              /* (d_inner, d_state) */
    const void *D;                  /* (d_inner) */
} mb2_block;

/* Bytes of workspace mb2_block_forward needs for (batch, seqlen). */
size_t mb2_block_workspace_bytes(const mb2_block *blk, int64_t batch,
                                 int64_t seqlen);

/* CPUMamba.forward (_mamba.py:204-265); with h_last / conv_tail non-NULL also
 * the state of forward_with_final_state (:165-202) from the same pass.
 *   x, out: (batch, seqlen, d_model) contiguous in dtype.
 * dt_proj runs as a tensor-core GEMM when it can (dense weight; F32 also
 * needs its weight_split; batch*seqlen >= 256), otherwise inside the scan
 * kernel from W_dt's rows. */
int mb2_block_forward(const mb2_block *blk, const void *x, void *out,
                      int64_t batch, int64_t seqlen, float *h_last,
                      void *conv_tail, void *workspace, size_t workspace_bytes,
                      mb2_stream_t stream);

/* Stage timing of mb2_block_forward: the same launches on the same stream,
 * with CUDA events between the six stages; waits for them and writes their
 * durations in ms to stage_ms[0..5] (in_proj, conv1d + SiLU, x_proj, dt_proj
 * + softplus, scan + gate, out_proj).  A profiling aid without a reference
 * counterpart (the reference times whole forwards, bench/bench.py:28-75). */
int mb2_block_forward_profile(const mb2_block *blk, const void *x, void *out,
                              int64_t batch, int64_t seqlen, void *workspace,
                              size_t workspace_bytes, float *stage_ms,
                              mb2_stream_t stream);

/* Bytes of workspace mb2_block_step needs for a batch. */
size_t mb2_step_workspace_bytes(const mb2_block *blk, int64_t batch);

/* CPUMamba.forward_step (_mamba.py:103-163) for one token per sequence.
 * h (batch, d_inner, d_state) f32 and conv_state (batch, d_inner, d_conv-1)
 * are updated IN PLACE.  x, out: (batch, d_model). */
int mb2_block_step(const mb2_block *blk, const void *x, void *out, float *h,
                   void *conv_state, int64_t batch, void *workspace,
                   size_t workspace_bytes, mb2_stream_t stream);

/* ---- residual stack: x <- x + block(RMSNorm(x)) per layer ----------------
 * No single counterpart in the reference (it has no stack); each layer is
 * CPUMamba.forward (_mamba.py:204-265) applied to torch.nn.RMSNorm(x), the
 * composition a Mamba-130M-style model makes around the block. */

/* out = w * norm_weight[col] (rows, cols), rounded to dtype: RMSNorm's weight
 * folded into the columns of the in_proj weight that follows it. */
int mb2_fold_norm(int dtype, const void *w, const void *norm_weight, void *out,
                  int64_t rows, int64_t cols, mb2_stream_t stream);

/* Bytes of workspace mb2_stack_forward needs. */
size_t mb2_stack_workspace_bytes(const mb2_block *layers, int64_t n_layers,
                                 int64_t batch, int64_t seqlen);

/* n_layers pre-norm residual blocks over x (batch, seqlen, d_model), updated
 * IN PLACE: per layer x = x + block(x / sqrt(mean(x^2) + eps) * g).  Each
 * layer's in_proj weight (and its TF32 split for f32) must be the folded
 * weight mb2_fold_norm(W_in, g) of that layer's norm weight g.  The 1/rms
 * factor is applied in in_proj's epilogue and the residual add in out_proj's,
 * so the normalised activations are never materialised. */
int mb2_stack_forward(const mb2_block *layers, int64_t n_layers, float eps, void *x,
                      int64_t batch, int64_t seqlen, void *workspace,
                      size_t workspace_bytes, mb2_stream_t stream);

/* mb2_stack_forward that also leaves each layer's final state, as
 * CPUMamba.forward_with_final_state does for one block (_mamba.py:165-202):
 * h_last[i] (batch, d_inner, d_state) fp32 and conv_tail[i] (batch, d_inner,
 * d_conv-1) of layer i; either array (or an entry) may be NULL. */
int mb2_stack_forward_state(const mb2_block *layers, int64_t n_layers, float eps, void *x,
                            int64_t batch, int64_t seqlen, float *const *h_last,
                            void *const *conv_tail, void *workspace, size_t workspace_bytes,
                            mb2_stream_t stream);

/* One decode step of the stack: x (batch, d_model) is the residual stream,
 * updated in place (x <- x + block_i(RMSNorm_i(x)) for every layer i), each
 * layer's h[i] and conv_state[i] advanced as mb2_block_step does
 * (_mamba.py:103-163 per layer).  layers[i].in_proj.weight is the norm-folded
 * weight, as for mb2_stack_forward. */
size_t mb2_stack_step_workspace_bytes(const mb2_block *layers, int64_t n_layers,
                                      int64_t batch);
int mb2_stack_step(const mb2_block *layers, int64_t n_layers, float eps, void *x,
                   float *const *h, void *const *conv_state, int64_t batch, void *workspace,
                   size_t workspace_bytes, mb2_stream_t stream);

/* ---- d_inner channel shards ------------------------------------------------
 * A block whose d_inner channels are split over ranks (one GPU each): blk
 * describes this rank's shard -- d_inner = its channel count; in_proj rows
 * = its channels of the x half then of the z half; conv1d, dt_proj, A_log and
 * D the channels' rows; x_proj and out_proj the channels' COLUMNS (both
 * contract over d_inner); out_proj's bias on one rank only.  A forward or a
 * step runs in two phases with an all-reduce (sum over ranks) after each:
 *   phase 1: in_proj -> conv -> x_proj's partial x_dbl, left in the workspace
 *            at the offset mb2_block_shard_xdbl gives ((rows, ld) elements of
 *            the activation dtype, pad columns zeroed)  -> all-reduce x_dbl
 *   phase 2: dt_proj -> scan -> gate -> out_proj's partial into out
 *            -> all-reduce out
 * Both phases take the same workspace (mb2_block_workspace_bytes /
 * mb2_step_workspace_bytes of the shard).  h_last / conv_tail (forward) and h
 * / conv_state (step) are the shard's channels.  The split of _mamba.py:204-265
 * / :103-163 over devices; the reference runs on one host. */
int mb2_block_shard_xdbl(const mb2_block *blk, int64_t rows, int step, size_t *offset,
                         int64_t *ld);
int mb2_block_forward_shard(const mb2_block *blk, int phase, const void *x, void *out,
                            int64_t batch, int64_t seqlen, float *h_last, void *conv_tail,
                            void *workspace, size_t workspace_bytes, mb2_stream_t stream);
int mb2_block_step_shard(const mb2_block *blk, int phase, const void *x, void *out, float *h,
                         void *conv_state, int64_t batch, void *workspace,
                         size_t workspace_bytes, mb2_stream_t stream);

/* ---- all-reduce through peer memory ---------------------------------------
 * The sum over ranks (one GPU each, one node) that the shards above need,
 * as one kernel over NVLink: each rank pushes its data (as fp32) into every
 * rank's buffer, raises per-chunk flags there, waits for every rank's flags
 * in its own buffer and sums the contributions in rank order (every rank gets
 * the same bits; bf16 data is summed in fp32 and rounded once).  Buffers come
 * from mb2_peer_alloc (cudaMalloc + a CUDA IPC handle, exchanged by the
 * caller) and mb2_peer_open in the other ranks' processes.  No counterpart in
 * the reference (one host, no collectives).  Every rank must make the same
 * sequence of calls (same counts) on one stream; calls may be captured in a
 * CUDA graph (the call counter lives in the buffer).  A wait that exceeds
 * timeout_ns records MB2_PEER_TIMEOUT in the rank's status word
 * (mb2_peer_status) and the kernel returns; the data is then not the sum. */
#define MB2_PEER_MAX_RANKS 8
#define MB2_PEER_TIMEOUT 0x7e01
#define MB2_PEER_HANDLE_BYTES 64
typedef struct mb2_peer_group {
    int32_t world, rank;
    int64_t slot_elems;                    /* largest count per call */
    int64_t timeout_ns;                    /* bound of every wait */
    void *bufs[MB2_PEER_MAX_RANKS];        /* every rank's buffer, mapped here */
} mb2_peer_group;
size_t mb2_peer_buffer_bytes(int world, int64_t slot_elems);
int mb2_peer_alloc(size_t bytes, void **ptr, void *ipc_handle /* 64 bytes out */);
int mb2_peer_open(const void *ipc_handle, void **ptr);
int mb2_peer_close(void *ptr);
int mb2_peer_free(void *ptr);
int mb2_peer_allreduce(int dtype, void *data, int64_t count, const mb2_peer_group *g,
                       mb2_stream_t stream);
int mb2_peer_status(const mb2_peer_group *g, int *code, int clear);

/* Size of the device array mb2_block_step_static uses as its workspace. */
#define MB2_STEP_STATIC_SCRATCH_BYTES (8u << 20)

/* mb2_block_step for callers that cannot allocate device memory (a plugin
 * whose host application owns the device memory budget, or a serving loop
 * that must not allocate once running).  No counterpart in the reference: its
 * forward_step allocates host tensors freely.  Same arguments and results as
 * mb2_block_step, but the workspace is a fixed MB2_STEP_STATIC_SCRATCH_BYTES
 * (8 MiB) array inside the library, held on every GPU that loads the library
 * until exit; a batch whose mb2_step_workspace_bytes exceeds it returns
 * MB2_ERR_WORKSPACE.  Allocates nothing.  The first call on a device looks the
 * array's address up (cudaGetSymbolAddress) with that device current, so make
 * it before any stream capture.  All calls on a device share the array: calls
 * whose GPU work overlaps race and must be ordered by the caller. */
int mb2_block_step_static(const mb2_block *blk, const void *x, void *out, float *h,
                          void *conv_state, int64_t batch, mb2_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MAMBA_B200_H */
