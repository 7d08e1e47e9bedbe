// Context, workspace and error plumbing of the C ABI (include/aceflow_cuda.h).
#include "common.cuh"

#include <cstdlib>
#include <cstring>
#include <new>

namespace af {

static thread_local char g_error[1024] = "";

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

int enter(af_ctx *ctx, const char *fn) {
  if (ctx == nullptr || ctx->magic != kCtxMagic)
    return fail(AF_ERR_STATE, "%s: invalid or destroyed af_ctx", fn);
  int cur = -1;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return fail(AF_ERR_CUDA, "%s: cudaGetDevice: %s", fn, cudaGetErrorString(e));
  if (cur != ctx->device) {
    e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return fail(AF_ERR_CUDA, "%s: cudaSetDevice: %s", fn, cudaGetErrorString(e));
  }
  return AF_OK;
}

int workspace(af_ctx *ctx, size_t bytes, void **out, const char *fn) {
  bytes = (bytes + 255) & ~size_t(255);
  if (bytes > ctx->workspace_bytes) {
    if (ctx->workspace) {
      cudaError_t e = cudaFree(ctx->workspace);
      ctx->workspace = nullptr;
      ctx->workspace_bytes = 0;
      if (e != cudaSuccess) return fail(AF_ERR_CUDA, "%s: cudaFree(workspace): %s", fn, cudaGetErrorString(e));
    }
    cudaError_t e = cudaMalloc(&ctx->workspace, bytes);
    if (e != cudaSuccess)
      return fail(AF_ERR_CUDA, "%s: cudaMalloc(workspace, %zu): %s", fn, bytes, cudaGetErrorString(e));
    ctx->workspace_bytes = bytes;
  }
  *out = ctx->workspace;
  return AF_OK;
}

}  // namespace af

extern "C" {

int af_abi_version(void) { return 2; }

const char *af_last_error(void) { return af::g_error; }

int af_cuda_init(int device, af_ctx **out) {
  if (out == nullptr) return af::fail(AF_ERR_ARG, "af_cuda_init: out is NULL");
  *out = nullptr;
  int n = 0;
  AF_CUDA(cudaGetDeviceCount(&n), "af_cuda_init");
  if (device < 0 || device >= n)
    return af::fail(AF_ERR_ARG, "af_cuda_init: device %d out of range (%d devices)", device, n);
  AF_CUDA(cudaSetDevice(device), "af_cuda_init");
  cudaDeviceProp prop;
  AF_CUDA(cudaGetDeviceProperties(&prop, device), "af_cuda_init");
  if (prop.major != 10)
    return af::fail(AF_ERR_ARG, "af_cuda_init: device %d is sm_%d%d; this library is built for sm_100a",
                    device, prop.major, prop.minor);
  af_ctx *ctx = new (std::nothrow) af_ctx();
  if (!ctx) return af::fail(AF_ERR_ARG, "af_cuda_init: out of host memory");
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  cudaError_t e = cudaMalloc(&ctx->dev_err, 256);
  if (e == cudaSuccess) e = cudaMemset(ctx->dev_err, 0, 256);
  if (e != cudaSuccess) {
    delete ctx;
    return af::fail(AF_ERR_CUDA, "af_cuda_init: device error word: %s", cudaGetErrorString(e));
  }
  int lo_prio = 0, hi_prio = 0;
  if (e == cudaSuccess) e = cudaDeviceGetStreamPriorityRange(&lo_prio, &hi_prio);
  if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&ctx->side[0], cudaStreamNonBlocking, hi_prio);
  if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&ctx->side[1], cudaStreamNonBlocking, lo_prio);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_fork, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_join, cudaEventDisableTiming);
  for (int i = 0; i < af_ctx::kMaxSlices && e == cudaSuccess; ++i) {
    e = cudaEventCreateWithFlags(&ctx->ev_a[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_b[i], cudaEventDisableTiming);
  }
  if (e != cudaSuccess) {
    af_ctx *tmp = ctx;
    ctx->magic = kCtxMagic;
    af_cuda_destroy(tmp);
    return af::fail(AF_ERR_CUDA, "af_cuda_init: streams/events: %s", cudaGetErrorString(e));
  }
  if (const char *env = getenv("AF_DECODE_SLICE_ROWS")) ctx->decode_slice_rows = atoi(env);
  if (const char *env = getenv("AF_DECODE_HEAD_GROUPS")) ctx->decode_head_groups = atoi(env);
  if (const char *env = getenv("AF_SHARDED_HEAD_GROUPS")) ctx->sharded_head_groups = atoi(env);
  if (const char *env = getenv("AF_PDL")) ctx->pdl = atoi(env) != 0;
  if (const char *env = getenv("AF_GEMM_PAIR")) ctx->gemm_pair = atoi(env) != 0;
  if (const char *env = getenv("AF_DECODE_PAIRS")) ctx->decode_pairs = atoi(env) != 0;
  if (const char *env = getenv("AF_GEMM_PRODUCERS")) {
    const int v = atoi(env);
    if (v >= 1 && v <= 4) ctx->gemm_producers = v;
  }
  if (const char *env = getenv("AF_COMM_RESERVE_SMS")) ctx->comm_reserve_sms = atoi(env);
  if (const char *env = getenv("AF_SHARDED_ROW_SLABS")) ctx->sharded_row_slabs = atoi(env);
  ctx->magic = kCtxMagic;
  *out = ctx;
  return AF_OK;
}

int af_cuda_destroy(af_ctx *ctx) {
  AF_ENTER(ctx, "af_cuda_destroy");
  af::comm_release(ctx);
  if (ctx->workspace) cudaFree(ctx->workspace);
  if (ctx->dev_err) cudaFree(ctx->dev_err);
  for (int i = 0; i < 2; ++i)
    if (ctx->side[i]) cudaStreamDestroy(ctx->side[i]);
  if (ctx->ev_fork) cudaEventDestroy(ctx->ev_fork);
  if (ctx->ev_join) cudaEventDestroy(ctx->ev_join);
  for (int i = 0; i < af_ctx::kMaxSlices; ++i) {
    if (ctx->ev_a[i]) cudaEventDestroy(ctx->ev_a[i]);
    if (ctx->ev_b[i]) cudaEventDestroy(ctx->ev_b[i]);
  }
  for (int i = 0; i < af_ctx::kMaxMarks; ++i)
    if (ctx->mark_ev[i]) cudaEventDestroy(ctx->mark_ev[i]);
  ctx->magic = 0;
  delete ctx;
  return AF_OK;
}

int af_reserve_workspace(af_ctx *ctx, size_t bytes) {
  AF_ENTER(ctx, "af_reserve_workspace");
  void *p = nullptr;
  return af::workspace(ctx, bytes, &p, "af_reserve_workspace");
}

int af_check_device(af_ctx *ctx, int *flags, int reset) {
  if (ctx == nullptr) return af::noalloc_check_device(flags, reset);
  AF_ENTER(ctx, "af_check_device");
  int h = 0;
  AF_CUDA(cudaMemcpy(&h, ctx->dev_err, sizeof(int), cudaMemcpyDeviceToHost), "af_check_device");
  if (reset && h) AF_CUDA(cudaMemset(ctx->dev_err, 0, sizeof(int)), "af_check_device");
  if (flags) *flags = h;
  if (h & (1 << AF_ERR_TIMEOUT))
    return af::fail(AF_ERR_TIMEOUT, "af_check_device: a device-side wait timed out (flags 0x%x)", h);
  return AF_OK;
}

int af_set_option(af_ctx *ctx, const char *name, int64_t value) {
  AF_ENTER(ctx, "af_set_option");
  if (!name) return af::fail(AF_ERR_ARG, "af_set_option: name is NULL");
  if (!strcmp(name, "decode_head_groups")) {
    if (value < 1 || value > af_ctx::kMaxSlices) return af::fail(AF_ERR_ARG, "af_set_option: decode_head_groups 1..8");
    ctx->decode_head_groups = (int)value;
  } else if (!strcmp(name, "allow_split_k")) {
    ctx->allow_split_k = value != 0;
  } else if (!strcmp(name, "decode_pairs")) {
    ctx->decode_pairs = value != 0;
  } else if (!strcmp(name, "gemm_pair")) {
    ctx->gemm_pair = value != 0;
  } else if (!strcmp(name, "gemm_producers")) {
    if (value < 1 || value > 4) return af::fail(AF_ERR_ARG, "af_set_option: gemm_producers must be 1..4");
    ctx->gemm_producers = (int)value;
  } else if (!strcmp(name, "pdl")) {
    ctx->pdl = value != 0;
  } else if (!strcmp(name, "decode_transposed")) {
    if (value < 0 || value > 15) return af::fail(AF_ERR_ARG, "af_set_option: decode_transposed 0..15");
    ctx->decode_transposed = (int)value;
  } else if (!strcmp(name, "sharded_head_groups")) {
    if (value < 0 || value > af_ctx::kMaxSlices) return af::fail(AF_ERR_ARG, "af_set_option: sharded_head_groups 0..8");
    ctx->sharded_head_groups = (int)value;
  } else if (!strcmp(name, "sharded_row_slabs")) {
    if (value < 0 || value > af_ctx::kMaxSlices) return af::fail(AF_ERR_ARG, "af_set_option: sharded_row_slabs 0..8");
    ctx->sharded_row_slabs = (int)value;
  } else if (!strcmp(name, "comm_reserve_sms")) {
    if (value < 0 || value > 64) return af::fail(AF_ERR_ARG, "af_set_option: comm_reserve_sms 0..64");
    ctx->comm_reserve_sms = (int)value;
  } else if (!strcmp(name, "chunk_len")) {
    if (value != 64 && value != 128) return af::fail(AF_ERR_ARG, "af_set_option: chunk_len must be 64 or 128");
    ctx->chunk_len = (int)value;
  } else if (!strcmp(name, "chunkwise_segments")) {
    if (value < 0 || value > 4096) return af::fail(AF_ERR_ARG, "af_set_option: chunkwise_segments 0..4096");
    ctx->chunk_segments = (int)value;
  } else if (!strcmp(name, "phase_marks")) {
    for (int i = 0; value && i < af_ctx::kMaxMarks; ++i)
      if (!ctx->mark_ev[i]) AF_CUDA(cudaEventCreate(&ctx->mark_ev[i]), "af_set_option(phase_marks)");
    ctx->phase_marks = value != 0;
    ctx->nmarks = 0;
  } else if (!strcmp(name, "decode_slice_rows")) {
    if (value < 0) return af::fail(AF_ERR_ARG, "af_set_option: decode_slice_rows >= 0");
    ctx->decode_slice_rows = (int)value;
  } else {
    return af::fail(AF_ERR_ARG, "af_set_option: unknown option '%s'", name);
  }
  return AF_OK;
}

int af_phase_times(af_ctx *ctx, float *ms, const char **names, int max, int *n) {
  AF_ENTER(ctx, "af_phase_times");
  if (!ms || !names || !n || max < 0) return af::fail(AF_ERR_ARG, "af_phase_times: null output or bad max");
  *n = 0;
  if (!ctx->phase_marks || ctx->nmarks < 2) return AF_OK;
  AF_CUDA(cudaEventSynchronize(ctx->mark_ev[ctx->nmarks - 1]), "af_phase_times");
  for (int i = 1; i < ctx->nmarks && *n < max; ++i) {
    float t = 0.f;
    AF_CUDA(cudaEventElapsedTime(&t, ctx->mark_ev[i - 1], ctx->mark_ev[i]), "af_phase_times");
    ms[*n] = t;
    names[*n] = ctx->mark_name[i];
    ++*n;
  }
  return AF_OK;
}

int af_launch_count(af_ctx *ctx, int64_t *count) {
  AF_ENTER(ctx, "af_launch_count");
  if (!count) return af::fail(AF_ERR_ARG, "af_launch_count: count is NULL");
  *count = ctx->launches;
  return AF_OK;
}

}  // extern "C"
