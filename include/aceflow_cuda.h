/*
 * aceflow_cuda.h — C ABI of the B200 (sm_100a) retention hot path.
 *
 * This is the drop-in boundary under AceFlow's af.nn.MultiScaleRetention /
 * Linear / RMSNorm / SwiGLU, af.ops and AceEngine APIs.  Each entry point
 * names the reference interface it replaces (paths relative to the
 * 42Wor/aceflow checkout).  A Rust `extern "C"` block, a PyO3 method or a
 * Python ctypes stub binds these symbols directly.
 *
 * Conventions
 *  - Every pointer argument except `af_ctx*` and host-side parameters is a
 *    DEVICE pointer on the context's device, owned by the caller.  The
 *    library never frees caller memory.
 *  - Matrices are row-major and contiguous unless a stride argument says
 *    otherwise.  Weights use the PyTorch (out, in) layout that the reference
 *    uses (aceflow/nn/layers.py:19-20, aceflow-core/src/nn/mod.rs:34-39).
 *  - `af_stream_t` is a cudaStream_t (NULL = the legacy default stream).
 *    Every call is asynchronous on that stream.
 *  - Every call returns an af_status.  On failure, af_last_error() gives a
 *    message for the calling thread.  No exception crosses the ABI.  Shape
 *    errors are the analogue of the reference's PyValueError
 *    (aceflow-core/src/cpu/mod.rs:64-68,188-238,615-644).
 *  - Scratch memory comes from the context's workspace, grown on first use
 *    (af_reserve_workspace() sizes it up front, e.g. before graph capture).
 *  - One context per device per host thread.
 */
#ifndef ACEFLOW_CUDA_H_
#define ACEFLOW_CUDA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  AF_OK = 0,
  AF_ERR_ARG = 1,     /* bad shape, null pointer, unsupported size */
  AF_ERR_CUDA = 2,    /* a CUDA runtime/driver call failed */
  AF_ERR_NCCL = 3,    /* reserved for collective calls */
  AF_ERR_TIMEOUT = 4, /* a bounded device-side wait gave up */
  AF_ERR_STATE = 5    /* context misuse (wrong device, destroyed context) */
} af_status;

typedef struct af_ctx af_ctx;
typedef void *af_stream_t;

/* ------------------------------------------------------------------ context */
int af_abi_version(void);
const char *af_last_error(void);
/* Creates a context on `device` (no reference counterpart: the reference's
 * CPU engine needs none; its GPU context is wgpu/context.rs:54-91). */
int af_cuda_init(int device, af_ctx **ctx);
int af_cuda_destroy(af_ctx *ctx);
int af_reserve_workspace(af_ctx *ctx, size_t bytes);
/* Synchronises the device and reads the context's device error word: a
 * kernel whose bounded wait gave up sets bit AF_ERR_TIMEOUT instead of
 * hanging.  Returns AF_ERR_TIMEOUT if set; `flags` (may be NULL) receives the
 * word; `reset` clears it.  ctx == NULL reads (and with `reset` clears) the
 * error word of af_msr_decode_step_f32_noalloc on the current device, which
 * takes no context. */
int af_check_device(af_ctx *ctx, int *flags, int reset);
/* Runs the bounded-wait error path on purpose, with no fault: one thread
 * waits (the kernels' own mbarrier wait, limit `limit_ns`, 1 us .. 2 s) on a
 * barrier phase nothing completes, gives up and sets AF_ERR_TIMEOUT in the
 * context's error word (ctx == NULL: the word of
 * af_msr_decode_step_f32_noalloc on the current device), which
 * af_check_device then reports.  No reference counterpart: the reference's
 * failures are host-side PyValueErrors (aceflow-core/src/cpu/mod.rs:188-238). */
int af_selftest_bounded_wait(af_ctx *ctx, int64_t limit_ns, af_stream_t stream);
/* Tuning switches of a context (no reference counterpart):
 *   "decode_head_groups" 1..8  head groups pipelined by the split decode step (default 1)
 *   "allow_split_k"      0/1   small-M GEMMs may split K with fp32 atomics (default 1;
 *                              0 makes results bitwise reproducible run to run)
 *   "decode_slice_rows"  >= 0  batch slices of af_msr_decode_step_f32 (default 0: none)
 *   "chunk_len"          64/128 tokens per chunk of the chunkwise prefill when a call passes
 *                              chunk 0, and of af_decoder_layer_prefill (default 64)
 *   "chunkwise_segments" >= 0  sequence segments per stream in the chunkwise prefill
 *                              (default 0: enough to put one CTA on every SM; 1: none)
 *   "sharded_head_groups" 0..8 head groups af_prefill_head_sharded pipelines against
 *                              its all-gather (default 0 = 1: measured not to pay)
 *   "sharded_row_slabs"  0..8  row slabs af_prefill_head_sharded_rows pipelines, the all-to-all of
 *                              slab j+1 under the W_o GEMM of slab j (default 0 = 1:
 *                              measured not to pay at 2 GPUs)
 *   "comm_reserve_sms"   0..64 SMs the overlapped kernels leave to the collective (default 16)
 *   "decode_transposed"  0..15 bf16 af_decoder_layer_decode projections computed as
 *                              W . x^T (bit 0 QKV, 1 W_o, 2 gate/up, 3 down; default 15)
 *   "pdl"                0/1   decode chains as programmatic dependent launches (default 1)
 *   "gemm_pair"          0/1   large bf16 GEMMs on CTA pairs, 256 x 256 tiles (default 1)
 *   "decode_pairs"       0/1   the decode step's projections on CTA pairs (default 1)
 *   "gemm_producers"     1..4  TMA producer threads per tensor-core GEMM CTA (default 1)
 *   "phase_marks"        0/1   record timing events at the prefill phases (af_phase_times) */
int af_set_option(af_ctx *ctx, const char *name, int64_t value);
/* Phase times of the last prefill call made with af_set_option "phase_marks"
 * on (af_msr_prefill_bf16, af_retention_chunkwise_bf16,
 * af_prefill_head_sharded[_rows]): the device time between consecutive phase
 * boundaries on the caller's stream, e.g. "qkv", "chunk_state",
 * "chunk_scan", "chunkwise", "allgather"/"alltoall", "w_o".  Waits for the
 * last boundary.  Fills up to `max` entries; `n` receives the count (0 when
 * marks are off).  No reference counterpart (measurement). */
int af_phase_times(af_ctx *ctx, float *ms, const char **names, int max, int *n);
/* Number of this library's kernel launches issued through `ctx` so far. */
int af_launch_count(af_ctx *ctx, int64_t *count);

/* ------------------------------------------------------------- retention */
/* Recurrent retention step for `batch` independent streams.
 * Replaces retention_step_core (aceflow-core/src/cpu/recurrence.rs:3-42) as
 * called by AceEngine.retention_step / retention_step_packed
 * (aceflow-core/src/cpu/mod.rs:486-545).
 *   state  [batch][num_heads][head_dim][head_dim] fp32, updated in place;
 *          consecutive streams are `state_batch_stride` floats apart.
 *   q,k,v  row b at q + b*qkv_row_stride (fp32), head h at h*head_dim.
 *   out    [batch][num_heads*head_dim] fp32 (o = q . S with the UPDATED S).
 * Any head_dim; multiples of 4 up to 1024 take the vectorised kernel. */
int af_retention_step(af_ctx *ctx, float *state, int64_t state_batch_stride, const float *gamma,
                      const float *q, const float *k, const float *v, int64_t qkv_row_stride,
                      float *out, int batch, int num_heads, int head_dim, af_stream_t stream);

/* Token-serial retention over T tokens for `batch` streams; writes every
 * token's output.  Replaces AceEngine.prefill_recurrent
 * (aceflow-core/src/cpu/mod.rs:547-587), which returns only the last row.
 *   q,k,v  token t of stream b at (b*T + t)*qkv_row_stride.
 *   out    [batch][T][num_heads*head_dim]. */
int af_retention_scan(af_ctx *ctx, float *state, int64_t state_batch_stride, const float *gamma,
                      const float *q, const float *k, const float *v, int64_t qkv_row_stride,
                      float *out, int batch, int T, int num_heads, int head_dim,
                      af_stream_t stream);

/* ----------------------------------------------------------- norms, FFN */
/* y = x / sqrt(mean(x^2) + eps) * w over rows of length d.
 * Replaces RMSNorm.forward / ops.rms_norm (aceflow/nn/layers.py:45-49,
 * aceflow/ops/functional.py:18-25) and rmsnorm_core
 * (aceflow-core/src/cpu/norm.rs:6-59).  If `residual` is non-NULL the input
 * is x + residual, which is also written to `sum_out` when that is non-NULL
 * (the pre-norm residual add of cpu/mod.rs:679-683). */
int af_rmsnorm_f32(af_ctx *ctx, const float *x, const float *residual, const float *w, float *y,
                   float *sum_out, int rows, int d, float eps, af_stream_t stream);
/* Same on bf16 rows (fp32 math, bf16 out); w stays fp32. */
int af_rmsnorm_bf16(af_ctx *ctx, const uint16_t *x, const float *w, uint16_t *y, int rows, int d,
                    float eps, af_stream_t stream);

/* hidden = silu(gate) * up with gate_up packed [rows][2f], gate first.
 * Replaces swiglu_forward (aceflow-core/src/cpu/swiglu.rs:4-18). */
int af_swiglu_packed_f32(af_ctx *ctx, const float *gate_up, float *hidden, int rows, int f,
                         af_stream_t stream);
/* out = silu(gate) * up elementwise (ops.silu when up == NULL,
 * aceflow/ops/functional.py:44-46; SwiGLU.forward's product, layers.py:83-87). */
int af_silu_mul_f32(af_ctx *ctx, const float *gate, const float *up, float *out, int64_t n,
                    af_stream_t stream);

/* out = a + b (b repeats every b_period elements: the bias broadcast of
 * Tensor + bias, aceflow/core/tensor.py:104-118) or a + scalar if b == NULL. */
int af_add_f32(af_ctx *ctx, const float *a, const float *b, float *out, int64_t n, int64_t b_period,
               float scalar, af_stream_t stream);

/* ----------------------------------------------------------------- GEMM */
/* y[M][N] = x[M][K] . W[N][K]^T (+ bias[N]), fp32 in/out with fp32-accurate
 * accumulation.  Replaces Linear.forward (aceflow/nn/layers.py:29-33) ->
 * Tensor::matmul (aceflow-core/src/tensor/mod.rs:182-196) and gemv /
 * batched_gemv (aceflow-core/src/cpu/gemv.rs:164-194). */
int af_linear_f32(af_ctx *ctx, const float *x, const float *w, const float *bias, float *y, int M,
                  int N, int K, af_stream_t stream);
/* Same with bf16 x [M][K] and W [N][K] on the bf16 tensor cores, fp32
 * accumulation; y is fp32 (y_bf16 == 0) or bf16 (y_bf16 != 0).  The bf16
 * path of Linear.forward for the tensor-core prefill. */
int af_linear_bf16(af_ctx *ctx, const uint16_t *x, const uint16_t *w, const float *bias, void *y,
                   int y_bf16, int M, int N, int K, af_stream_t stream);

/* Reorders the fused QKV weight [3d][d] (rows q, k, v as in AceEngine's
 * w_qkv, aceflow-core/src/cpu/mod.rs:201-207) into head-major rows
 * [H][q|k|v][head_dim][d], so each head group's projection weights are one
 * contiguous block.  elem_bytes 2 or 4. */
int af_pack_qkv_heads(af_ctx *ctx, const void *src, void *dst, int d_model, int num_heads,
                      int elem_bytes, af_stream_t stream);

/* Splits fp32 values into an exact tf32 part (low 13 mantissa bits cleared)
 * and the remainder: hi + lo == src exactly.  Prepares weights for
 * af_msr_decode_step_f32_split (done once, at weight-load time). */
int af_split_tf32(af_ctx *ctx, const float *src, float *hi, float *lo, int64_t n, af_stream_t stream);

/* General bf16 tensor-core GEMM with strided operands and the fused
 * epilogue: C = rowscale * (A[M][K] . B[N][K]^T) (+ bias) (+ residual), with
 * A row stride lda, B row stride ldb (elements), output row stride ldo
 * (replaces the gemm of aceflow-core/src/tensor/ops.rs:71-90 for bf16).
 * a_kblock > 0: A is K-blocked, K/a_kblock blocks [M][a_kblock] stored one
 * after another (what an all-gather of per-rank column slices produces);
 * a_kblock must divide K and be a multiple of 64.  0: plain [M][K].
 * rowscale[m] = 1/sqrt(sum_p row_sumsq(m, p) * inv_d + eps) when row_sumsq
 * is non-NULL (the RMSNorm of a retention output), else 1; row_sumsq is
 * [M][nparts], or with parts_block > 0 nparts/parts_block blocks
 * [M][parts_block] one after another.  accumulate != 0 adds into out (fp32)
 * instead of overwriting it.  The head-sharded prefill's output projection
 * is this GEMM over the gathered head outputs. */
int af_gemm_bf16(af_ctx *ctx, const uint16_t *A, int64_t lda, int a_kblock, const uint16_t *B,
                 int64_t ldb, int M, int N, int K, void *out, int64_t ldo, int out_bf16,
                 const float *bias, const float *residual, int64_t ldr, const float *row_sumsq,
                 int nparts, int parts_block, float inv_d, float eps, int accumulate,
                 af_stream_t stream);

/* af_linear_f32 from operands split by af_split_tf32 (x_hi + x_lo == x,
 * w_hi + w_lo == W): the tensor cores read ready-made tf32 operands.
 * K % 4 == 0, all pointers 16-byte aligned. */
int af_linear_f32_split(af_ctx *ctx, const float *x_hi, const float *x_lo, const float *w_hi,
                        const float *w_lo, const float *bias, float *y, int M, int N, int K,
                        af_stream_t stream);

/* ------------------------------------------------------- fused MSR layer */
/* One recurrent decode step of a MultiScaleRetention layer for `batch`
 * streams: qkv = x W_qkv^T; retention step; RMSNorm(eps, ret_norm_w) over
 * d_model; out = normed W_o^T.  The recurrent counterpart of
 * MultiScaleRetention.forward_parallel (aceflow/nn/retention.py:44-66), i.e.
 * AceEngine.forward_layer_internal's retention half
 * (aceflow-core/src/cpu/mod.rs:651-678).
 *   x [batch][d] fp32; w_qkv [3d][d] (rows q, k, v); w_o [d][d];
 *   state [batch][H][d/H][d/H] fp32 in place; out [batch][d] fp32.
 * Uses workspace scratch of (4*d + H) * batch floats. */
int af_msr_decode_step_f32(af_ctx *ctx, const float *x, float *state, const float *gamma,
                           const float *w_qkv, const float *w_o, const float *ret_norm_w,
                           float eps, int batch, int d_model, int num_heads, float *out,
                           af_stream_t stream);

/* af_msr_decode_step_f32 with the projection weights prepared beforehand
 * (once, at weight-load time): w_qkv packed head-major by af_pack_qkv_heads
 * and then split by af_split_tf32 into w_qkv_hi + w_qkv_lo; w_o split by
 * af_split_tf32 as it is.  The tensor cores read ready-made tf32 operands
 * (fp32-exact weights; twice the weight bytes are read).  Optionally
 * (af_set_option "decode_head_groups") the step runs as a pipeline over head
 * groups: one group's QKV projection overlapping the previous group's state
 * stream and the one before's W_o product.
 * For 64 < batch <= 256 the QKV projection runs transposed (W_qkv . x^T:
 * every weight tile read by one CTA) with split-K partial buffers that the
 * state-stream kernel sums while it loads q, k, v.
 * head_dim 64/128/256, all pointers 16-byte aligned.
 * Workspace: batch*(17*d_model + num_heads) + 64 floats. */
int af_msr_decode_step_f32_split(af_ctx *ctx, const float *x, float *state, const float *gamma,
                                 const float *w_qkv_hi, const float *w_qkv_lo, const float *w_o_hi,
                                 const float *w_o_lo, const float *ret_norm_w, float eps, int batch,
                                 int d_model, int num_heads, float *out, af_stream_t stream);

/* The same decode step for callers that cannot allocate device memory when
 * they run it: a server whose device memory is carved up front by its own
 * arena allocator, or a plugin inside a host that owns the device-memory
 * budget.  No reference counterpart: the reference's CPU engine preallocates
 * its host buffers in AceEngine::new.  Scratch comes from a fixed 16 MiB
 * array inside the library (2^22 floats; the step needs
 * batch*(4*d_model + num_heads) of them, i.e. batch <= 511 at d_model 2048),
 * held on every GPU that loads the library until the process exits; larger
 * sizes return AF_ERR_ARG.  The call allocates nothing and takes no context;
 * the current device is used.  The first call on a device looks up the
 * array's device address (and loads the library's kernels there, a one-time
 * set-up); do not call the entry point again after cudaDeviceReset.  All calls on a device share the array and keep the last
 * call's contents, so calls that overlap on the GPU (concurrent streams)
 * race: at most one call in flight per device.  A bounded-wait timeout in its
 * kernels is reported by af_check_device(NULL, ...). */
int af_msr_decode_step_f32_noalloc(const float *x, float *state, const float *gamma,
                                   const float *w_qkv, const float *w_o, const float *ret_norm_w,
                                   float eps, int batch, int d_model, int num_heads, float *out,
                                   af_stream_t stream);

/* Chunkwise-parallel retention core on the bf16 tensor cores (head_dim 256,
 * chunks of `chunk` = 64 or 128 tokens; 0 takes the context's "chunk_len").
 * The parallel form (aceflow/nn/retention.py:51-61) computed chunk by chunk
 * with the carried state of recurrence.rs:28-39; the result does not depend
 * on the chunk length beyond rounding.
 *   qkv       [batch*T][3*H*256] bf16: q | k | v per row (a QKV projection).
 *   state_in  [batch][H][256][256] fp32 initial state, or NULL for zeros.
 *   state_out same layout, the state after the last token, or NULL.
 *   out       [batch*T][H*256] bf16: retention output times norm_w (or 1).
 *   sumsq     [batch*T][P*H] fp32 partial sums of the unscaled output's
 *             squares (row r's RMS is sqrt(sum(sumsq[r]) / d)), or NULL;
 *             P = 2 for chunk 64, 4 for chunk 128.
 * When batch*H*2 CTAs cannot fill the GPU, each stream is cut into sequence
 * segments (af_chunkwise_plan): a state pass, a scan over segment states
 * and the full pass from each segment's state; workspace
 * batch*nseg*H*256 KiB when nseg > 1. */
int af_retention_chunkwise_bf16(af_ctx *ctx, const uint16_t *qkv, int batch, int T, int num_heads,
                                const float *gamma, const float *state_in, float *state_out,
                                uint16_t *out, const float *norm_w, float *sumsq, int chunk, af_stream_t stream);

/* Backward of af_retention_chunkwise_bf16 for training: given the forward's
 * qkv [batch*T][3*H*256] bf16 (q | k | v), its initial state (state_in,
 * [batch][H][256][256] fp32, or NULL for zeros) and the gradient of the
 * retention output dout [batch*T][H*256] bf16 (the output before norm_w),
 * writes dqkv [batch*T][3*H*256] bf16 (dQ | dK | dV) and, if dstate_in is
 * non-NULL, the gradient of the initial state [batch][H][256][256] fp32.
 * The loss is taken to depend on the outputs only (not on the final state).
 * Each gradient is a retention form of its own (dQ = Retention(dO, V, K)
 * from S_0^T; dK and dV are Retention(V, dO, Q) and Retention(K, Q, dO) over
 * reversed time), so three passes of the 128-token tensor-core kernel do
 * the work; bf16 results, fp32 accumulation.  No reference counterpart: the
 * reference trains through PyTorch only (aceflow/trainers).  Workspace
 * batch*T*6*d bytes (+ batch*H*256 KiB with a state, + segment states). */
int af_retention_chunkwise_backward_bf16(af_ctx *ctx, const uint16_t *qkv, const uint16_t *dout, int batch, int T,
                                         int num_heads, const float *gamma, const float *state_in, uint16_t *dqkv,
                                         float *dstate_in, af_stream_t stream);

/* The sequence segmentation the chunkwise prefill uses for `batch` streams
 * of T tokens and `num_heads` heads on a GPU with num_sms SMs (host-only,
 * needs no GPU).  nseg_req > 0 forces that many segments (capped by the
 * chunk count); 0 picks enough for one CTA per SM.  Outputs the segment
 * count and length (a multiple of `chunk` tokens, 64 or 128, 0 = 64; the
 * last segment may be shorter). */
int af_chunkwise_plan(int num_sms, int batch, int T, int num_heads, int nseg_req, int chunk, int *nseg,
                      int *seg_len);

/* MultiScaleRetention forward over a prompt on the bf16 tensor cores:
 * x [batch*T][d] bf16 -> out [batch*T][d] (fp32, or bf16 if out_bf16).
 * Replaces MultiScaleRetention.forward_parallel (aceflow/nn/retention.py:44-66)
 * for bf16 inputs (fp32 accumulation, tolerance 2e-2) and the token-serial
 * AceEngine.prefill_recurrent (aceflow-core/src/cpu/mod.rs:547-587).
 *   w_qkv [3d][d] bf16 (rows q, k, v); w_o [d][d] bf16; ret_norm_w [d] fp32;
 *   state_in/state_out and chunk as for af_retention_chunkwise_bf16.
 * head_dim must be 256.  Workspace: batch*T*(8*d + 16*H) bytes. */
int af_msr_prefill_bf16(af_ctx *ctx, const uint16_t *x, const uint16_t *w_qkv, const uint16_t *w_o,
                        const float *ret_norm_w, const float *gamma, float eps, int batch, int T,
                        int d_model, int num_heads, const float *state_in, float *state_out,
                        void *out, int out_bf16, int chunk, af_stream_t stream);

/* ------------------------------------------------- gated MSR (opt-in mode)
 * RetNet's gate and per-head GroupNorm (Sun et al. 2023, eq. 8):
 *   out = (swish(x W_g^T) (.) GroupNorm_H(Retention(x))) W_o^T
 * in place of the reference's RMSNorm(Retention(x)) W_o^T.  No reference
 * counterpart: the reference has neither a gate nor a group norm
 * (aceflow/nn/retention.py:44-66); these entry points are an extension,
 * checked against their own float64 restatement. */
/* y = swish(g) * (gn_weight * (o - mean_h) / sqrt(var_h + eps) + gn_bias) for
 * each row and head h (mean and variance over the head's d/H values); o, g, y
 * fp32 or bf16 (the *_bf16 flags) [rows][d]; gn_weight/gn_bias [d] or NULL
 * (1 / 0).  y must not overlap o or g.  head_dim a multiple of 8, <= 1024. */
int af_group_norm_gate(af_ctx *ctx, const void *o, int o_bf16, const void *g, int g_bf16, const float *gn_weight,
                       const float *gn_bias, void *y, int y_bf16, int64_t rows, int d_model, int num_heads, float eps,
                       af_stream_t stream);
/* One recurrent decode step of the gated layer (fp32, 3xTF32 projections):
 * x [batch][d]; w_qkv [3d][d] (rows q, k, v); w_g [d][d]; w_o [d][d];
 * state [batch][H][d/H][d/H] in place; out [batch][d].  Workspace 6*batch*d
 * floats. */
int af_msr_gated_decode_step_f32(af_ctx *ctx, const float *x, float *state, const float *gamma, const float *w_qkv,
                                 const float *w_g, const float *w_o, const float *gn_weight, const float *gn_bias,
                                 float eps, int batch, int d_model, int num_heads, float *out, af_stream_t stream);
/* The gated layer over a prompt on the bf16 tensor cores (head_dim 256):
 * x [batch*T][d] bf16, weights bf16, state_in/state_out and chunk as for
 * af_retention_chunkwise_bf16; out fp32 (or bf16 if out_bf16). */
int af_msr_gated_prefill_bf16(af_ctx *ctx, const uint16_t *x, const uint16_t *w_qkv, const uint16_t *w_g,
                              const uint16_t *w_o, const float *gn_weight, const float *gn_bias, const float *gamma,
                              float eps, int batch, int T, int d_model, int num_heads, const float *state_in,
                              float *state_out, void *out, int out_bf16, int chunk, af_stream_t stream);

/* ------------------------------------------------------- decoder stack */
/* Weights of one decoder layer (AceEngine's LayerWeights,
 * aceflow-core/src/cpu/mod.rs:18-28), device pointers.  Matrices are fp32 or
 * bf16 (one dtype per layer), (out, in) layout.  w_gate_up must be in the
 * 16-row interleave produced by af_pack_gate_up from AceEngine's
 * [gate rows; up rows] layout.  Norm weights are fp32. */
typedef struct {
  const void *w_qkv;     /* [3d][d], rows q, k, v */
  const void *w_o;       /* [d][d] */
  const void *w_gate_up; /* [2f][d], interleaved */
  const void *w_down;    /* [d][f] */
  const float *norm1, *norm2, *ret_norm; /* [d] */
} af_layer_weights;

/* Row permutation [gate; up] -> (16 gate rows, 16 up rows) groups, the
 * layout the fused SwiGLU epilogue reads.  f % 16 == 0; elem_bytes 2 or 4. */
int af_pack_gate_up(af_ctx *ctx, const void *src, void *dst, int f, int d, int elem_bytes,
                    af_stream_t stream);

/* One decoder layer at one token for `batch` streams, in place on x [batch][d]
 * fp32 and the layer's state slice (streams `state_batch_stride` floats
 * apart).  AceEngine.forward_layer (aceflow-core/src/cpu/mod.rs:423-444 ->
 * 646-706) batched.  weights_bf16 selects bf16 weights (bf16 tensor cores,
 * bf16 activations into the GEMMs) or fp32 weights (3xTF32, fp32 accuracy).
 * head_dim 64, 128 or 256; f % 16 == 0. */
int af_decoder_layer_decode(af_ctx *ctx, const af_layer_weights *w, int weights_bf16, float *x,
                            float *state, int64_t state_batch_stride, const float *gamma, float eps,
                            int batch, int d_model, int num_heads, int d_ffn, af_stream_t stream);

/* One decoder layer over T prompt tokens per stream (bf16 weights, tensor-core
 * chunkwise retention), in place on x [batch*T][d] fp32; replaces running
 * forward_layer_internal token by token over the prompt
 * (generate_stream_internal, cpu/mod.rs:721-730).  state_in/state_out
 * [batch][H][256][256] fp32 (either may be NULL: zeros / not written). */
int af_decoder_layer_prefill(af_ctx *ctx, const af_layer_weights *w, float *x, const float *state_in,
                             float *state_out, const float *gamma, float eps, int batch, int T,
                             int d_model, int num_heads, int d_ffn, af_stream_t stream);

/* x[r] = table[tokens[r]] (fp32 or bf16 table [vocab][d] -> fp32 rows).  An
 * out-of-range prompt id keeps the previous row of its sequence (cpu/mod.rs:
 * 721-726); zero_oob = 1 gives the generated-token rule (zeros, 757-763).
 * Rows form sequences of T. */
int af_embed_gather(af_ctx *ctx, const void *table, int table_bf16, const int32_t *tokens, float *x,
                    int rows, int T, int vocab, int d, int zero_oob, af_stream_t stream);

/* y = bf16(RMSNorm(x) * w) for fp32 rows; w == NULL gives a plain cast. */
int af_rmsnorm_to_bf16(af_ctx *ctx, const float *x, const float *w, uint16_t *y, int rows, int d,
                       float eps, af_stream_t stream);

/* Greedy pick per row, first maximum wins (sampler.rs:118-128). */
int af_argmax_rows(af_ctx *ctx, const float *logits, int rows, int vocab, int32_t *out,
                   af_stream_t stream);

/* logits [batch][vocab] = table . RMSNorm_final(x) (tied LM head,
 * project_logits, sampler.rs:67-81; final_norm may be NULL as in AceEngine's
 * default), then tokens[b] = argmax.  table fp32 or bf16 [vocab][d]. */
int af_lm_head_argmax(af_ctx *ctx, const float *x, const float *final_norm, float eps,
                      const void *table, int table_bf16, int batch, int vocab, int d,
                      float *logits, int32_t *tokens, af_stream_t stream);

/* tokens[r] = one draw from row r of logits [rows][vocab] (fp32), as
 * sample_token_from_logits (aceflow-core/src/cpu/sampler.rs:104-180):
 * repetition penalty over the distinct in-range tokens of row r's context
 * (apply_repetition_penalty, sampler.rs:83-102): context_tokens[r *
 * context_stride + 0 .. context_len) (ids < 0 or >= vocab are skipped, so -1
 * pads shorter contexts; context_len 0: none), then greedy when
 * temperature <= 1e-4, else logits /
 * max(temperature, 1e-5), the top_k largest (0 = all), a softmax over them,
 * the sorted prefix through the first place where the running sum exceeds
 * top_p, and the first item of that prefix where the running sum reaches
 * uniforms[r] * (its mass).  uniforms [rows] in [0, 1) take the place of the
 * reference's clock-seeded generator (sampler.rs:8-35); they may be NULL
 * when greedy.  Equal logits are ordered by lowest index.  logits is not
 * modified; vocab <= AF_SAMPLE_MAX_VOCAB. */
#define AF_SAMPLE_MAX_VOCAB 50000
int af_sample_rows(af_ctx *ctx, const float *logits, int rows, int vocab, const int32_t *context_tokens,
                   int64_t context_stride, int context_len, float temperature, int top_k, float top_p,
                   float repetition_penalty, const float *uniforms, int32_t *out, af_stream_t stream);

/* ------------------------------------------------------- multi-GPU prefill
 * One process per GPU.  Rank 0 creates an id with af_comm_unique_id, the
 * ranks share it out of band (torch.distributed, MPI, a file), then every
 * rank calls af_comm_init with its context (collective: blocks until all
 * ranks joined).  NCCL is loaded at run time (libnccl.so.2).  No reference
 * counterpart: the reference runs on one CPU or one wgpu device. */
#define AF_COMM_ID_BYTES 128
int af_comm_unique_id(void *id_out /* AF_COMM_ID_BYTES */);
int af_comm_init(af_ctx *ctx, int nranks, int rank, const void *unique_id);
int af_comm_destroy(af_ctx *ctx);

/* Head-sharded MultiScaleRetention prefill (the layer of af_msr_prefill_bf16
 * split over the ranks of the context's communicator; aceflow/nn/
 * retention.py:44-66 for the math).  Rank r owns heads [r*H/g, (r+1)*H/g)
 * and output columns [r*dl, (r+1)*dl), dl = d/g:
 *   x           [batch*T][d] bf16, the same on every rank
 *   w_qkv_local [3*dl][d] bf16: rows of W_q, then W_k, then W_v for its heads
 *   w_o_rows    [dl][d] bf16: rows r*dl..(r+1)*dl-1 of W_o
 *   ret_norm_w  [d] fp32 and gamma [H] fp32: the full vectors
 *   state_in/state_out [batch][H/g][256][256] fp32 for its heads, or NULL
 *   out         [batch*T][dl] fp32 (or bf16 if out_bf16): its columns of
 *               the layer output.
 * One ncclAllGather of the head outputs (bf16) and of the per-row partial
 * sums of squares precedes the output projection; with head groups
 * (af_set_option "sharded_head_groups"; batch 1 or no state) each group's
 * gather runs on a side stream under the next group's compute.  Every rank must make the
 * same call.  head_dim 256; H divisible by the rank count.  Workspace
 * batch*T*(6*dl + 2*d + 8*H) bytes plus segment states. */
int af_prefill_head_sharded(af_ctx *ctx, const uint16_t *x, const uint16_t *w_qkv_local,
                            const uint16_t *w_o_rows, const float *ret_norm_w, const float *gamma,
                            float eps, int batch, int T, int d_model, int num_heads,
                            const float *state_in, float *state_out, void *out, int out_bf16, int chunk,
                            af_stream_t stream);

/* The same layer, row-sharded: the exchange is an all-to-all (ncclSend /
 * ncclRecv pairs) instead of the all-gather, so each rank receives only
 * (g-1)/g^2 of the head outputs, and holds the complete rows
 * [r*c, r*c + n_r) (c = ceil(batch*T / g)) on which it applies the RMSNorm
 * and the FULL W_o.
 *   w_qkv_local [3*dl][d] bf16 as above; w_o [d][d] bf16 (all of it);
 *   out [n_r][d] fp32 (or bf16): rows r*c .. r*c + n_r - 1 of the layer
 *   output [batch*T][d] (n_r = 0 on ranks past the last row).
 * Every rank must make the same call.  head_dim 256; H divisible by the rank
 * count.  Workspace batch*T*(6*dl + 2*dl/g + 8*H/g*(1 + 1/g)) bytes plus
 * segment states. */
int af_prefill_head_sharded_rows(af_ctx *ctx, const uint16_t *x, const uint16_t *w_qkv_local, const uint16_t *w_o,
                                 const float *ret_norm_w, const float *gamma, float eps, int batch, int T,
                                 int d_model, int num_heads, const float *state_in, float *state_out, void *out,
                                 int out_bf16, int chunk, af_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* ACEFLOW_CUDA_H_ */
