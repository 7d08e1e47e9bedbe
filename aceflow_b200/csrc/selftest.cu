// Self-test of the bounded-wait error path.
//
// Every device-side wait in this library (mbarrier phases of the tcgen05
// kernels) gives up after a time limit, records AF_ERR_TIMEOUT in a device
// error word and lets its kernel return, instead of hanging the GPU.  This
// entry point runs that path on purpose, without any fault: one thread waits,
// with the same sm100::mbar_wait the kernels use and a caller-chosen short
// limit, on an mbarrier phase that nothing ever completes.  The host then
// reads AF_ERR_TIMEOUT through af_check_device and the context stays usable.
#include "common.cuh"
#include "sm100.cuh"

namespace {

__global__ void bounded_wait_selftest_kernel(int *err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);  // one arrival completes phase 0; none comes
    sm100::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !sm100::mbar_wait(&bar, 0, limit_ns)) atomicOr(err, 1 << AF_ERR_TIMEOUT);
}

}  // namespace

extern "C" int af_selftest_bounded_wait(af_ctx *ctx, int64_t limit_ns, af_stream_t stream) {
  const char *fn = "af_selftest_bounded_wait";
  AF_REQUIRE(limit_ns >= 1000 && limit_ns <= 2000000000LL, "af_selftest_bounded_wait",
             "limit_ns must be in [1 us, 2 s], got %lld", (long long)limit_ns);
  int *err = nullptr;
  if (ctx) {
    AF_ENTER(ctx, fn);
    err = ctx->dev_err;
  } else {
    int rc = af::noalloc_error_word(&err, fn);
    if (rc) return rc;
  }
  bounded_wait_selftest_kernel<<<1, 32, 0, af::stream_of(stream)>>>(err, (uint64_t)limit_ns);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return af::fail(AF_ERR_CUDA, "%s: launch failed: %s", fn, cudaGetErrorString(e));
  if (ctx) ctx->launches++;
  return AF_OK;
}
