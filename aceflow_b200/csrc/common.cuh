// Shared host/device helpers for the sm_100a retention kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cstdio>
#include <cstdarg>

#include "../../include/aceflow_cuda.h"

#include <atomic>
#include <utility>

struct af_ctx {
  int device = 0;
  int num_sms = 0;
  uint32_t magic = 0;
  void *workspace = nullptr;
  size_t workspace_bytes = 0;
  int64_t launches = 0;
  int *dev_err = nullptr;  // device error word: bit AF_ERR_TIMEOUT set by bounded waits
  // side streams + events for the overlapped decode step (fork/join on the
  // caller's stream, so the pattern is also valid under graph capture)
  cudaStream_t side[2] = {nullptr, nullptr};
  static constexpr int kMaxSlices = 8;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  cudaEvent_t ev_a[kMaxSlices] = {}, ev_b[kMaxSlices] = {};
  int allow_split_k = 1;        // small-M GEMMs may split K (fp32 atomics: not bitwise reproducible)
  // head groups pipelined in the split decode step; 1 = sequential, the
  // fastest measured on B200 (the state stream fills every SM, so the
  // pipelined GEMMs cannot co-reside and only add launches)
  int decode_head_groups = 1;
  int decode_slice_rows = 0;  // batch rows per overlapped slice; 0 = one sequential pass (faster today)
  int chunk_segments = 0;     // sequence segments per stream in the chunkwise prefill; 0 = fill the SMs
  int chunk_len = 64;         // tokens per chunk of the chunkwise prefill when a call passes 0 (64 or 128)
  // NCCL communicator of the head-sharded prefill (sharded_prefill.cu)
  void *comm = nullptr;
  int comm_nranks = 0, comm_rank = 0;
  int pdl = 1;  // decode chains use programmatic dependent launch
  int gemm_pair = 1;  // large bf16 GEMMs on CTA pairs (cta_group::2, 256 x 256 tiles)
  int decode_pairs = 1;  // decode-step projections on CTA pairs (256-row tiles)
  int gemm_producers = 1;  // TMA producer threads per tensor-core GEMM CTA (1..4)
  // bf16 decode layer projections run transposed (bit 0 QKV, 1 W_o, 2 gate/up, 3 down)
  int decode_transposed = 15;
  int sharded_head_groups = 0;  // head groups pipelined against the all-gather (0: auto; 1: one gather)
  int comm_reserve_sms = 16;    // SMs the overlapped kernels leave to NCCL
  // row slabs af_prefill_head_sharded_rows pipelines (slab j+1's all-to-all
  // under slab j's W_o GEMM); 0: auto, 1: one exchange
  int sharded_row_slabs = 0;
  // Phase marks (af_set_option "phase_marks"): timing events the prefill
  // entry points record on the caller's stream at their phase boundaries,
  // read back by af_phase_times.
  static constexpr int kMaxMarks = 16;
  int phase_marks = 0;
  int nmarks = 0;
  cudaEvent_t mark_ev[kMaxMarks] = {};
  const char *mark_name[kMaxMarks] = {};
};

constexpr uint32_t kCtxMagic = 0xACEF1011u;

namespace af {

// Thread-local message for af_last_error().
void set_error(const char *fmt, ...);

inline int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_error("%s", buf);
  return code;
}

// Validates the context and makes its device current.
int enter(af_ctx *ctx, const char *fn);

// Grows the context workspace to at least `bytes` (256-byte aligned base).
int workspace(af_ctx *ctx, size_t bytes, void **out, const char *fn);

// Checks the launch that was just issued and counts it.
inline int launched(af_ctx *ctx, const char *fn) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(AF_ERR_CUDA, "%s: launch failed: %s", fn, cudaGetErrorString(e));
  ctx->launches++;
  return AF_OK;
}

// Epilogue of the tensor-core GEMM (gemm_tc.cu).
struct GemmEpilogueArgs {
  void *out = nullptr;
  int64_t ldo = 0;
  int out_bf16 = 0;
  const float *bias = nullptr;
  const float *row_parts = nullptr;  // per-row partial sums of squares -> 1/rms scale
  int nparts = 0;
  float inv_d = 0.f, eps = 0.f;
  const float *residual = nullptr;  // fp32 [M][ldr] added after scaling
  int64_t ldr = 0;
  int swiglu = 0;  // (16 gate, 16 up) column groups -> silu(g)*u, N/2 outputs
  int accumulate = 0;  // add (atomically) into out, which the caller initialised
  int a_kblock = 0;    // A stored as K/a_kblock blocks [M][a_kblock] back to back (0: plain)
  int parts_block = 0; // row_parts stored as blocks [M][parts_block] (0: plain [M][nparts])
  int trans = 0;       // store C^T: element (m, n) at out[n * ldo + m] (plain fp32 only)
  int64_t split_stride = 0;  // split-K z stores its partial at out + z * split_stride (no atomics)
  int max_partials = 1;      // partial buffers available at out (split_stride != 0)
  int force_bn = 0, force_splits = 0;  // tile width / split count chosen by the caller (0: dispatch decides)
  // Programmatic dependent launch: operand (1 = A, 2 = B) that does not depend
  // on the previous kernel (the weights) and is prefetched before the wait;
  // 0 = none.  pdl = launch with the attribute.
  int pdl = 0, pre_operand = 0;
  int pair = 0;  // run on CTA pairs (256-row tiles; width and splits from force_bn / force_splits)
  int scale_residual = 0;  // the row scale multiplies the residual too: out = (acc + residual) * scale
  int max_ctas = 0;        // persistent kernel: at most this many CTAs (SMs left to a concurrent kernel); 0: all
};

bool tc_gemm_ok(const void *A, int64_t lda, const void *B, int64_t ldb, int K, bool fp32);
int tc_gemm(af_ctx *ctx, const void *A, int64_t lda, const void *B, int64_t ldb, int M, int N, int K, bool fp32,
            const GemmEpilogueArgs &a, cudaStream_t st, const char *fn);
int tc_gemm_presplit(af_ctx *ctx, const float *A_hi, const float *A_lo, int64_t lda, const float *B_hi,
                     const float *B_lo, int64_t ldb, int M, int N, int K, const GemmEpilogueArgs &a, cudaStream_t st,
                     const char *fn);
// hi = tf32 part of src, lo = src - hi (exact); `zero` (n floats, may be
// NULL) is cleared in the same pass.
int split_tf32(af_ctx *ctx, const float *src, float *hi, float *lo, int64_t n, cudaStream_t st, const char *fn,
               float *zero = nullptr, bool pdl = false);
// bf16(RMSNorm(x) * w) rows (decoder.cu); pdl: programmatic dependent launch.
int rmsnorm_to_bf16(af_ctx *ctx, const float *x, const float *w, uint16_t *y, int rows, int d, float eps,
                    cudaStream_t st, const char *fn, bool pdl);

// Chunkwise prefill (retention_chunkwise.cu).  A plan cuts each stream into
// nseg segments of seg_len tokens (seg_len a multiple of the chunk length).
struct ChunkPlan {
  int nseg, seg_len;
  int chunk;  // tokens per chunk: 64 or 128
};
ChunkPlan chunkwise_plan(int num_sms, int B, int T, int H, int nseg_req, int chunk);
size_t chunkwise_seg_state_bytes(int B, int H, const ChunkPlan &pl);
// ldo: output row stride (0: H*256); out_reverse: token t of each stream is
// written to row T-1-t.  Both need pl.chunk == 128.
int retention_chunkwise_bf16(af_ctx *ctx, const void *qkv, int B, int T, int H, const float *gamma,
                             const float *state_in, float *state_out, void *out, const float *norm_w, float *sumsq,
                             const ChunkPlan &pl, float *seg_states, cudaStream_t st, const char *fn, int64_t ldo = 0,
                             bool out_reverse = false);
// The same with q, k and v read from separate bf16 row-major buffers: row
// b*T + t of each, head h's columns h*256.. after the pointer, rows ldq / ldk
// / ldv elements apart (16-byte aligned pointers, strides multiples of 8).
struct ChunkSrc {
  const void *q, *k, *v;
  int64_t ldq, ldk, ldv;
};
int retention_chunkwise_bf16(af_ctx *ctx, const ChunkSrc &src, int B, int T, int H, const float *gamma,
                             const float *state_in, float *state_out, void *out, const float *norm_w, float *sumsq,
                             const ChunkPlan &pl, float *seg_states, cudaStream_t st, const char *fn, int64_t ldo,
                             bool out_reverse);
int chunkwise_head_dim();
// Per-head partial sums of squares per output row for that chunk length.
int chunkwise_parts(int chunk);
// The context's chunk length (af_set_option "chunk_len"; 64 or 128).
int chunkwise_default_chunk(const af_ctx *ctx);
// The chunk length of a call (0: the context's), checked.
int resolve_chunk(const af_ctx *ctx, int chunk, int *out, const char *fn);

// af_check_device(NULL, ...): the allocation-free decode step's error word on
// the current device (decode_noalloc.cu).
int noalloc_check_device(int *flags, int reset);
// Device address of that error word on the current device.
int noalloc_error_word(int **word, const char *fn);

// Releases the context's communicator, if any (sharded_prefill.cu).
void comm_release(af_ctx *ctx);

// One decode token of retention for `batch` streams (retention_decode.cu).
// hn > 0 selects heads [h0, h0 + hn) with q/k/v of consecutive heads qkv_hs
// floats apart; nsplit > 1 sums q/k/v over partial buffers split_stride
// floats apart (split-K projection output).
int launch_retention_step(af_ctx *ctx, float *state, int64_t state_bs, const float *gamma, const float *q,
                          const float *k, const float *v, int64_t qs, float *out, int64_t out_rs, int batch, int H,
                          int dh, const float *norm_w, float *sumsq, cudaStream_t st, const char *fn, int out_bf16,
                          float *out_lo = nullptr, int h0 = 0, int hn = 0, int64_t qkv_hs = 0, int nsplit = 1,
                          int64_t split_stride = 0, bool pdl = false);

inline cudaStream_t stream_of(af_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Phase marks: `mark_begin` starts a call's list, `mark` closes the phase
// named `name` (no-ops unless the context has phase_marks on; the events were
// created when it was switched on).
inline void mark(af_ctx *ctx, const char *name, cudaStream_t st) {
  if (!ctx->phase_marks || ctx->nmarks >= af_ctx::kMaxMarks || !ctx->mark_ev[ctx->nmarks]) return;
  cudaEventRecord(ctx->mark_ev[ctx->nmarks], st);
  ctx->mark_name[ctx->nmarks++] = name;
}
inline void mark_begin(af_ctx *ctx, cudaStream_t st) {
  ctx->nmarks = 0;
  mark(ctx, "begin", st);
}

// Raises a kernel's dynamic shared-memory limit on the context's device,
// once per device (the attribute is per device; `done` is the call site's
// device bitmask - setting it twice is harmless, so the check may race).
inline int smem_attr(af_ctx *ctx, const void *kernel, size_t bytes, std::atomic<unsigned long long> &done,
                     const char *fn) {
  const unsigned long long bit = 1ull << (ctx->device & 63);
  if (done.load(std::memory_order_relaxed) & bit) return AF_OK;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return fail(AF_ERR_CUDA, "%s: shared-memory attribute: %s", fn, cudaGetErrorString(e));
  done.fetch_or(bit, std::memory_order_relaxed);
  return AF_OK;
}

// Launches `kernel`, optionally as a programmatic dependent launch: it may
// start while the previous kernel on the stream drains and must execute
// griddep_wait() before it reads that kernel's results or writes anything.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 bool pdl, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace af

#define AF_ENTER(ctx, fn)                       \
  do {                                          \
    int _rc = af::enter((ctx), (fn));           \
    if (_rc != AF_OK) return _rc;               \
  } while (0)

#define AF_REQUIRE(cond, fn, ...)                                      \
  do {                                                                 \
    if (!(cond)) return af::fail(AF_ERR_ARG, fn ": " __VA_ARGS__);     \
  } while (0)

#define AF_CUDA(call, fn)                                                               \
  do {                                                                                  \
    cudaError_t _e = (call);                                                            \
    if (_e != cudaSuccess) return af::fail(AF_ERR_CUDA, "%s: %s: %s", fn, #call,        \
                                           cudaGetErrorString(_e));                     \
  } while (0)

// ------------------------------------------------------------------ device
// Programmatic dependent launch: wait until the previous kernel on the
// stream has completed and its memory is visible (a no-op otherwise).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel on the stream (a programmatic dependent launch) be
// scheduled once every CTA of this grid has executed it: its CTAs then take
// free SMs and run their prologue (barriers, TMEM, the first weight tiles)
// while this grid works, and block in griddep_wait() before touching this
// grid's results.  Issued after a CTA's own TMEM allocation, so a dependent
// CTA never holds TMEM that a CTA of this grid still has to allocate.
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float4 ld_stream(const float4 *p) {
  float4 v;
  asm volatile("ld.global.cs.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_stream(float4 *p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
