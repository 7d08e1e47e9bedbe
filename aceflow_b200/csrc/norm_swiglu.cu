// RMSNorm and SwiGLU: bandwidth-bound row kernels.
//
// RMSNorm (aceflow/nn/layers.py:45-49; aceflow-core/src/cpu/norm.rs:6-59):
//   y = x * (1 / sqrt(mean(x^2) + eps)) * w
// One CTA per row; the row is read once into shared memory (16-byte vector
// loads when aligned), the sum of squares is a warp-shuffle tree, and the
// scaled row is written once.  The optional residual input gives the pre-norm
// residual add of AceEngine (cpu/mod.rs:679-683) in the same pass.
//
// SwiGLU (aceflow-core/src/cpu/swiglu.rs:4-18): h = g / (1 + exp(-g)) * u.
#include "common.cuh"

namespace {

__device__ __forceinline__ float block_sum(float v, float *red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) red[wid] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = 0.f;
  for (int w = 0; w < nw; ++w) t += red[w];
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(256)
    rmsnorm_f32_kernel(const float *__restrict__ x, const float *__restrict__ res, const float *__restrict__ w,
                       float *__restrict__ y, float *__restrict__ sum_out, int d, float eps, bool vec) {
  extern __shared__ float row[];
  __shared__ float red[32];
  const size_t off = (size_t)blockIdx.x * d;
  float ss = 0.f;
  if (vec) {
    const float4 *x4 = reinterpret_cast<const float4 *>(x + off);
    const float4 *r4 = res ? reinterpret_cast<const float4 *>(res + off) : nullptr;
    float4 *s4 = reinterpret_cast<float4 *>(row);
    for (int i = threadIdx.x; i < d / 4; i += blockDim.x) {
      float4 a = x4[i];
      if (r4) {
        const float4 b = r4[i];
        a.x += b.x;
        a.y += b.y;
        a.z += b.z;
        a.w += b.w;
        if (sum_out) reinterpret_cast<float4 *>(sum_out + off)[i] = a;
      }
      s4[i] = a;
      ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
    }
  } else {
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
      float a = x[off + i];
      if (res) {
        a += res[off + i];
        if (sum_out) sum_out[off + i] = a;
      }
      row[i] = a;
      ss += a * a;
    }
  }
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)d + eps);
  if (vec) {
    const float4 *s4 = reinterpret_cast<const float4 *>(row);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    float4 *y4 = reinterpret_cast<float4 *>(y + off);
    for (int i = threadIdx.x; i < d / 4; i += blockDim.x) {
      const float4 a = s4[i], ww = w4[i];
      y4[i] = make_float4(a.x * (inv * ww.x), a.y * (inv * ww.y), a.z * (inv * ww.z), a.w * (inv * ww.w));
    }
  } else {
    for (int i = threadIdx.x; i < d; i += blockDim.x) y[off + i] = row[i] * (inv * w[i]);
  }
}

__global__ void __launch_bounds__(256)
    rmsnorm_bf16_kernel(const __nv_bfloat16 *__restrict__ x, const float *__restrict__ w,
                        __nv_bfloat16 *__restrict__ y, int d, float eps) {
  extern __shared__ float row[];
  __shared__ float red[32];
  const size_t off = (size_t)blockIdx.x * d;
  float ss = 0.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float a = __bfloat162float(x[off + i]);
    row[i] = a;
    ss += a * a;
  }
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)d + eps);
  for (int i = threadIdx.x; i < d; i += blockDim.x) y[off + i] = __float2bfloat16(row[i] * (inv * w[i]));
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

__global__ void swiglu_packed_kernel(const float *__restrict__ gu, float *__restrict__ h, int rows, int f) {
  const int64_t n = (int64_t)rows * f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / f, j = i - r * f;
    const float g = gu[r * 2 * f + j], u = gu[r * 2 * f + f + j];
    h[i] = silu(g) * u;
  }
}

__global__ void silu_mul_kernel(const float *__restrict__ g, const float *__restrict__ u, float *__restrict__ o,
                                int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    o[i] = u ? silu(g[i]) * u[i] : silu(g[i]);
}

__global__ void add_kernel(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ o,
                           int64_t n, int64_t period, float scalar) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    o[i] = a[i] + (b ? b[i % period] : scalar);
}

unsigned grid_for(int64_t n, const af_ctx *ctx) {
  int64_t blocks = (n + 255) / 256;
  const int64_t cap = (int64_t)ctx->num_sms * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (unsigned)blocks;
}

}  // namespace

namespace af {
int launch_rmsnorm_f32(af_ctx *ctx, const float *x, const float *res, const float *w, float *y, float *sum_out,
                       int rows, int d, float eps, cudaStream_t st, const char *fn) {
  if (rows == 0) return AF_OK;
  const bool vec = d % 4 == 0 && aligned16(x) && aligned16(w) && aligned16(y) && (!res || aligned16(res)) &&
                   (!sum_out || aligned16(sum_out));
  const size_t smem = (size_t)d * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(rmsnorm_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(AF_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(e));
  }
  rmsnorm_f32_kernel<<<rows, 256, smem, st>>>(x, res, w, y, sum_out, d, eps, vec);
  return launched(ctx, fn);
}
}  // namespace af

extern "C" {

int af_rmsnorm_f32(af_ctx *ctx, const float *x, const float *residual, const float *w, float *y, float *sum_out,
                   int rows, int d, float eps, af_stream_t stream) {
  const char *fn = "af_rmsnorm_f32";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(x && w && y, "af_rmsnorm_f32", "null pointer");
  AF_REQUIRE(rows >= 0 && d > 0 && d <= 56 * 1024, "af_rmsnorm_f32", "bad sizes rows=%d d=%d", rows, d);
  return af::launch_rmsnorm_f32(ctx, x, residual, w, y, sum_out, rows, d, eps, af::stream_of(stream), fn);
}

int af_rmsnorm_bf16(af_ctx *ctx, const uint16_t *x, const float *w, uint16_t *y, int rows, int d, float eps,
                    af_stream_t stream) {
  const char *fn = "af_rmsnorm_bf16";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(x && w && y, "af_rmsnorm_bf16", "null pointer");
  AF_REQUIRE(rows >= 0 && d > 0 && d <= 48 * 1024 / 4, "af_rmsnorm_bf16", "bad sizes rows=%d d=%d", rows, d);
  if (rows == 0) return AF_OK;
  rmsnorm_bf16_kernel<<<rows, 256, (size_t)d * sizeof(float), af::stream_of(stream)>>>(
      reinterpret_cast<const __nv_bfloat16 *>(x), w, reinterpret_cast<__nv_bfloat16 *>(y), d, eps);
  return af::launched(ctx, fn);
}

int af_swiglu_packed_f32(af_ctx *ctx, const float *gate_up, float *hidden, int rows, int f, af_stream_t stream) {
  const char *fn = "af_swiglu_packed_f32";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(gate_up && hidden, "af_swiglu_packed_f32", "null pointer");
  AF_REQUIRE(rows >= 0 && f > 0, "af_swiglu_packed_f32", "bad sizes rows=%d f=%d", rows, f);
  if (rows == 0) return AF_OK;
  swiglu_packed_kernel<<<grid_for((int64_t)rows * f, ctx), 256, 0, af::stream_of(stream)>>>(gate_up, hidden, rows, f);
  return af::launched(ctx, fn);
}

int af_silu_mul_f32(af_ctx *ctx, const float *gate, const float *up, float *out, int64_t n, af_stream_t stream) {
  const char *fn = "af_silu_mul_f32";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(gate && out && n >= 0, "af_silu_mul_f32", "bad arguments");
  if (n == 0) return AF_OK;
  silu_mul_kernel<<<grid_for(n, ctx), 256, 0, af::stream_of(stream)>>>(gate, up, out, n);
  return af::launched(ctx, fn);
}

int af_add_f32(af_ctx *ctx, const float *a, const float *b, float *out, int64_t n, int64_t b_period, float scalar,
               af_stream_t stream) {
  const char *fn = "af_add_f32";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(a && out && n >= 0, "af_add_f32", "bad arguments");
  AF_REQUIRE(!b || (b_period > 0 && n % b_period == 0), "af_add_f32", "b_period %lld must divide n %lld",
             (long long)b_period, (long long)n);
  if (n == 0) return AF_OK;
  add_kernel<<<grid_for(n, ctx), 256, 0, af::stream_of(stream)>>>(a, b, out, n, b_period, scalar);
  return af::launched(ctx, fn);
}

}  // extern "C"
