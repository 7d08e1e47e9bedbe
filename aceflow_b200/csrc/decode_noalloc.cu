// Decode step for callers that cannot allocate device memory.
//
// af_msr_decode_step_f32 takes its scratch (the packed q/k/v projection, the
// retention output and the per-head sums of squares) from the context's
// workspace, which grows with cudaMalloc on first use.  Some callers cannot
// allocate at that point: serving processes whose device memory is carved up
// front by their own arena allocator (a library cudaMalloc would break their
// accounting or fail outright once the arena holds the free memory), plugins
// loaded into a host that owns the device-memory budget, and loops that must
// not take cudaMalloc's implicit synchronisation.  For them,
// af_msr_decode_step_f32_noalloc runs the very same kernels, with its scratch
// in a fixed array compiled into this library (kNoallocScratchFloats floats,
// 16 MiB, held on every GPU that loads the library until the process exits)
// and with no context argument, so a call allocates nothing.
//
// The array's name is a host-side stand-in in host code, not a device
// address: the device address is looked up with cudaGetSymbolAddress once
// per device, with that device current, by the first call made on it.  The cached
// address belongs to the device's current primary context: after
// cudaDeviceReset the entry point must not be called again in the process.
//
// The kernels' bounded waits report a timeout in this file's own device
// error word (there is no context to hold one); af_check_device(NULL, ...)
// reads and clears it for the current device.
#include "common.cuh"

#include <mutex>

namespace af {
size_t msr_decode_scratch_floats(int batch, int d, int H);
int msr_decode_step_impl(af_ctx *ctx, const float *x, float *state, const float *gamma, const float *w_qkv,
                         const float *w_o, const float *ret_norm_w, float eps, int B, int d, int H, float *out,
                         float *scratch, cudaStream_t st, const char *fn);
int check_msr_decode(const char *fn, const float *x, float *state, const float *gamma, const float *w_qkv,
                     const float *w_o, const float *ret_norm_w, int B, int d, int H, const float *out);
}  // namespace af

namespace {

constexpr size_t kNoallocScratchFloats = size_t(1) << 22;  // 16 MiB of fp32 scratch
constexpr int kMaxDevices = 64;

// Shared by every call on a device; nothing in it needs to start at zero
// (each call writes the scratch it reads), except the error word, which
// device globals start with.
static __device__ __align__(256) float g_noalloc_scratch[kNoallocScratchFloats];
static __device__ __align__(256) int g_noalloc_err[64];

struct DeviceSetup {
  float *scratch = nullptr;  // device address of g_noalloc_scratch on this device
  int *err = nullptr;        // device address of g_noalloc_err
  int num_sms = 0;
  bool ready = false;
};
DeviceSetup g_setup[kMaxDevices];
std::mutex g_setup_mu;

// Once per device, with that device current: resolve the arrays' device
// addresses (this also loads the library's module on the device).
int setup_device(int dev, DeviceSetup *out, const char *fn) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  DeviceSetup &s = g_setup[dev];
  if (!s.ready) {
    void *p = nullptr, *pe = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return af::fail(AF_ERR_CUDA, "%s: cudaGetSymbolAddress(scratch): %s", fn, cudaGetErrorString(e));
    e = cudaGetSymbolAddress(&pe, g_noalloc_err);
    if (e != cudaSuccess) return af::fail(AF_ERR_CUDA, "%s: cudaGetSymbolAddress(error word): %s", fn, cudaGetErrorString(e));
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return af::fail(AF_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(e));
    s.scratch = static_cast<float *>(p);
    s.err = static_cast<int *>(pe);
    s.num_sms = sms;
    s.ready = true;
  }
  *out = s;
  return AF_OK;
}

}  // namespace

namespace af {
// Device address of the error word on the current device (set-up included).
int noalloc_error_word(int **word, const char *fn) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(AF_ERR_CUDA, "%s: cudaGetDevice: %s", fn, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(AF_ERR_ARG, "%s: device %d out of range", fn, dev);
  DeviceSetup s;
  int rc = setup_device(dev, &s, fn);
  if (rc) return rc;
  *word = s.err;
  return AF_OK;
}

// af_check_device(NULL, ...): the allocation-free entry point's error word on
// the current device.  cudaMemcpyFromSymbol synchronises the device first.
int noalloc_check_device(int *flags, int reset) {
  const char *fn = "af_check_device(NULL)";
  int h = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&h, g_noalloc_err, sizeof(int));
  if (e != cudaSuccess) return fail(AF_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(e));
  if (reset && h) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_noalloc_err, &zero, sizeof(int));
    if (e != cudaSuccess) return fail(AF_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(e));
  }
  if (flags) *flags = h;
  if (h & (1 << AF_ERR_TIMEOUT))
    return fail(AF_ERR_TIMEOUT, "%s: a device-side wait of the allocation-free decode step timed out (flags 0x%x)",
                fn, h);
  return AF_OK;
}
}  // namespace af

extern "C" int af_msr_decode_step_f32_noalloc(const float *x, float *state, const float *gamma, const float *w_qkv,
                                              const float *w_o, const float *ret_norm_w, float eps, int B, int d,
                                              int H, float *out, af_stream_t stream) {
  const char *fn = "af_msr_decode_step_f32_noalloc";
  int rc = af::check_msr_decode(fn, x, state, gamma, w_qkv, w_o, ret_norm_w, B, d, H, out);
  if (rc) return rc;
  const size_t need = af::msr_decode_scratch_floats(B, d, H);
  if (need > kNoallocScratchFloats)
    return af::fail(AF_ERR_ARG,
                    "%s: batch %d x d_model %d needs %zu floats of scratch; the static array holds %zu "
                    "(use af_msr_decode_step_f32 for larger batches)",
                    fn, B, d, need, kNoallocScratchFloats);
  if (B == 0) return AF_OK;
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return af::fail(AF_ERR_CUDA, "%s: cudaGetDevice: %s", fn, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return af::fail(AF_ERR_ARG, "%s: device %d out of range", fn, dev);
  DeviceSetup s;
  rc = setup_device(dev, &s, fn);
  if (rc) return rc;
  // A context on the stack: no workspace, no side streams (sequential step).
  af_ctx ctx;
  ctx.device = dev;
  ctx.num_sms = s.num_sms;
  ctx.magic = kCtxMagic;
  ctx.dev_err = s.err;
  ctx.decode_slice_rows = 0;
  return af::msr_decode_step_impl(&ctx, x, state, gamma, w_qkv, w_o, ret_norm_w, eps, B, d, H, out, s.scratch,
                                  af::stream_of(stream), fn);
}
