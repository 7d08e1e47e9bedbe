// fp32 SIMT GEMM  y[M][N] = rowscale[m] * (x[M][K] . W[N][K]^T) + bias[N].
//
// Full fp32 accuracy on the CUDA cores: the generic path for odd shapes and
// the correctness baseline for the tensor-core GEMMs.  64x64 output tile per
// CTA, 16-deep K slices staged in shared memory (transposed so each thread
// reads its 4 rows / 4 columns as two float4), 4x4 register micro-tile.
//
// The optional row scale is the fused RMSNorm of the retention output
// (aceflow/nn/retention.py:64-65): rowscale[m] = 1/sqrt(sum_p part[m][p] / d + eps)
// where part[m][p] are per-head sums of o^2 written by the retention kernel.
#include "common.cuh"

namespace {

constexpr int BM = 64, BN = 64, BK = 16;

__global__ void __launch_bounds__(256)
    sgemm_nt_kernel(const float *__restrict__ x, const float *__restrict__ w, const float *__restrict__ bias,
                    float *__restrict__ y, int M, int N, int K, const float *__restrict__ parts, int nparts,
                    float inv_d, float eps) {
  __shared__ __align__(16) float As[BK][BM + 4];
  __shared__ __align__(16) float Ws[BK][BN + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[4][4] = {};
  // loader mapping: 256 threads x 4 elements = 64 rows x 16 k
  const int lr = threadIdx.x / 4, lk = (threadIdx.x % 4) * 4;
  for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int kk = k0 + lk + u;
      const int am = m0 + lr, wn = n0 + lr;
      As[lk + u][lr] = (am < M && kk < K) ? x[(size_t)am * K + kk] : 0.f;
      Ws[lk + u][lr] = (wn < N && kk < K) ? w[(size_t)wn * K + kk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      const float4 a = *reinterpret_cast<const float4 *>(&As[kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4 *>(&Ws[kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
    float scale = 1.f;
    if (parts) {
      float s = 0.f;
      for (int p = 0; p < nparts; ++p) s += parts[(size_t)m * nparts + p];
      scale = 1.0f / sqrtf(s * inv_d + eps);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n < N) y[(size_t)m * N + n] = acc[i][j] * scale + (bias ? bias[n] : 0.f);
    }
  }
}

}  // namespace

namespace af {
int launch_sgemm_nt(af_ctx *ctx, const float *x, const float *w, const float *bias, float *y, int M, int N, int K,
                    const float *parts, int nparts, float inv_d, float eps, cudaStream_t st, const char *fn) {
  if (M == 0 || N == 0) return AF_OK;
  const dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
  sgemm_nt_kernel<<<grid, 256, 0, st>>>(x, w, bias, y, M, N, K, parts, nparts, inv_d, eps);
  return launched(ctx, fn);
}
// fp32 GEMM dispatch: the 3xTF32 tensor-core kernel when the operands meet
// TMA's alignment rules, else the SIMT kernel.  Optional fused row scale.
int linear_f32(af_ctx *ctx, const float *x, int64_t ldx, const float *w, int64_t ldw, const float *bias, float *y,
               int64_t ldy, int M, int N, int K, const float *parts, int nparts, float inv_d, float eps,
               cudaStream_t st, const char *fn) {
  if (M == 0 || N == 0) return AF_OK;
  if (tc_gemm_ok(x, ldx, w, ldw, K, true) && M <= 65535 * 128) {
    GemmEpilogueArgs ep;
    ep.out = y;
    ep.ldo = ldy;
    ep.bias = bias;
    ep.row_parts = parts;
    ep.nparts = nparts;
    ep.inv_d = inv_d;
    ep.eps = eps;
    return tc_gemm(ctx, x, ldx, w, ldw, M, N, K, true, ep, st, fn);
  }
  if (ldx != K || ldw != K || ldy != N) return fail(AF_ERR_ARG, "%s: strided operands need 16-byte alignment", fn);
  return launch_sgemm_nt(ctx, x, w, bias, y, M, N, K, parts, nparts, inv_d, eps, st, fn);
}

}  // namespace af

extern "C" int af_linear_f32(af_ctx *ctx, const float *x, const float *w, const float *bias, float *y, int M, int N,
                             int K, af_stream_t stream) {
  const char *fn = "af_linear_f32";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(x && w && y, "af_linear_f32", "null pointer");
  AF_REQUIRE(M >= 0 && N >= 0 && K > 0, "af_linear_f32", "bad sizes M=%d N=%d K=%d", M, N, K);
  AF_REQUIRE(M <= 65535 * 64, "af_linear_f32", "M=%d too large", M);
  return af::linear_f32(ctx, x, K, w, K, bias, y, N, M, N, K, nullptr, 0, 0.f, 0.f, af::stream_of(stream), fn);
}

extern "C" int af_linear_bf16(af_ctx *ctx, const uint16_t *x, const uint16_t *w, const float *bias, void *y,
                              int y_bf16, int M, int N, int K, af_stream_t stream) {
  const char *fn = "af_linear_bf16";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(x && w && y, "af_linear_bf16", "null pointer");
  AF_REQUIRE(M >= 0 && N >= 0 && K > 0, "af_linear_bf16", "bad sizes M=%d N=%d K=%d", M, N, K);
  AF_REQUIRE(af::tc_gemm_ok(x, K, w, K, K, false), "af_linear_bf16",
             "K=%d must be a multiple of 8 and x, W 16-byte aligned", K);
  AF_REQUIRE(M <= 65535 * 128, "af_linear_bf16", "M=%d too large", M);
  af::GemmEpilogueArgs ep;
  ep.out = y;
  ep.ldo = N;
  ep.out_bf16 = y_bf16;
  ep.bias = bias;
  return af::tc_gemm(ctx, x, K, w, K, M, N, K, false, ep, af::stream_of(stream), fn);
}
