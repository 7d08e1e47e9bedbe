// Gated MultiScaleRetention (opt-in mode; no counterpart in the reference).
//
// The reference's layer is RMSNorm(Retention(X)) W_o^T (aceflow/nn/
// retention.py:44-66).  RetNet as published (Sun et al. 2023, "Retentive
// Network: A Successor to Transformer for Large Language Models", eq. 8)
// adds a gate projection and a per-head GroupNorm:
//     Y   = GroupNorm_H(Retention(X))        (each head's d_h values: mean 0,
//                                             variance 1, then weight/bias per channel)
//     out = (swish(X W_G^T) (.) Y) W_O^T      swish(g) = g * sigmoid(g)
// The retention itself stays the reference's (no 1/sqrt(d_h) scaling).
// Here the gate and the group norm are one fused pass over each token row
// (one warp per (row, head)), between the retention kernel and the W_O GEMM:
//   decode:  qkv GEMM (3xTF32), g GEMM, the fp32 state stream, group norm +
//            gate, W_O GEMM
//   prefill: qkv GEMM and g GEMM (bf16 tensor cores), the chunkwise kernel,
//            group norm + gate (bf16), W_O GEMM.
#include "common.cuh"

namespace af {
int linear_f32(af_ctx *ctx, const float *x, int64_t ldx, const float *w, int64_t ldw, const float *bias, float *y,
               int64_t ldy, int M, int N, int K, const float *parts, int nparts, float inv_d, float eps,
               cudaStream_t st, const char *fn);
}  // namespace af

namespace {

__device__ __forceinline__ void load8(const float *p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4 *>(p)[0], b = reinterpret_cast<const float4 *>(p)[1];
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16 *p, float (&v)[8]) {
  const uint4 r = *reinterpret_cast<const uint4 *>(p);
  const __nv_bfloat162 *e = reinterpret_cast<const __nv_bfloat162 *>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(e[i]);
    v[2 * i] = f.x, v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void store8(float *p, const float (&v)[8]) {
  reinterpret_cast<float4 *>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4 *>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void store8(__nv_bfloat16 *p, const float (&v)[8]) {
  uint4 r;
  __nv_bfloat162 *e = reinterpret_cast<__nv_bfloat162 *>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) e[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4 *>(p) = r;
}

constexpr int kMaxChunks = 4;  // 8-element chunks per lane: head_dim <= 1024

// One warp per (row, head): y = swish(g) * (gn_w * (o - mean) / sqrt(var + eps) + gn_b)
// over the head's dh values (two passes over registers: mean, then variance).
template <typename TO, typename TG, typename TY>
__global__ void __launch_bounds__(256) group_norm_gate_kernel(const TO *__restrict__ o, const TG *__restrict__ g,
                                                              const float *__restrict__ w,
                                                              const float *__restrict__ bias, TY *__restrict__ y,
                                                              int64_t rows, int d, int H, float eps) {
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (wid >= rows * H) return;
  const int64_t r = wid / H;
  const int h = (int)(wid % H);
  const int dh = d / H, nch = dh / 8;
  const size_t base = (size_t)r * d + (size_t)h * dh;
  float v[kMaxChunks][8];
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int ch = lane + 32 * c;
    if (ch < nch) {
      load8(o + base + 8 * ch, v[c]);
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[c][i];
    }
  }
  s = warp_sum(s);
  const float mean = s / (float)dh;
  float q = 0.f;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int ch = lane + 32 * c;
    if (ch < nch) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[c][i] -= mean;
        q = fmaf(v[c][i], v[c][i], q);
      }
    }
  }
  q = warp_sum(q);
  const float inv = rsqrtf(q / (float)dh + eps);
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int ch = lane + 32 * c;
    if (ch < nch) {
      float gv[8], out[8];
      load8(g + base + 8 * ch, gv);
      const int col = h * dh + 8 * ch;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float yn = v[c][i] * inv * (w ? w[col + i] : 1.f) + (bias ? bias[col + i] : 0.f);
        out[i] = yn * (gv[i] / (1.f + expf(-gv[i])));
      }
      store8(y + base + 8 * ch, out);
    }
  }
}

template <typename TO, typename TG, typename TY>
int launch_gn_gate(af_ctx *ctx, const void *o, const void *g, const float *w, const float *b, void *y, int64_t rows,
                   int d, int H, float eps, cudaStream_t st, const char *fn) {
  const int64_t warps = rows * H;
  group_norm_gate_kernel<TO, TG, TY><<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(
      static_cast<const TO *>(o), static_cast<const TG *>(g), w, b, static_cast<TY *>(y), rows, d, H, eps);
  return af::launched(ctx, fn);
}

int group_norm_gate(af_ctx *ctx, const void *o, int o_bf16, const void *g, int g_bf16, const float *w,
                    const float *b, void *y, int y_bf16, int64_t rows, int d, int H, float eps, cudaStream_t st,
                    const char *fn) {
  using B16 = __nv_bfloat16;
  const int key = (o_bf16 ? 4 : 0) | (g_bf16 ? 2 : 0) | (y_bf16 ? 1 : 0);
  switch (key) {
    case 0: return launch_gn_gate<float, float, float>(ctx, o, g, w, b, y, rows, d, H, eps, st, fn);
    case 1: return launch_gn_gate<float, float, B16>(ctx, o, g, w, b, y, rows, d, H, eps, st, fn);
    case 2: return launch_gn_gate<float, B16, float>(ctx, o, g, w, b, y, rows, d, H, eps, st, fn);
    case 3: return launch_gn_gate<float, B16, B16>(ctx, o, g, w, b, y, rows, d, H, eps, st, fn);
    case 4: return launch_gn_gate<B16, float, float>(ctx, o, g, w, b, y, rows, d, H, eps, st, fn);
    case 5: return launch_gn_gate<B16, float, B16>(ctx, o, g, w, b, y, rows, d, H, eps, st, fn);
    case 6: return launch_gn_gate<B16, B16, float>(ctx, o, g, w, b, y, rows, d, H, eps, st, fn);
    default: return launch_gn_gate<B16, B16, B16>(ctx, o, g, w, b, y, rows, d, H, eps, st, fn);
  }
}

inline size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

}  // namespace

extern "C" {

int af_group_norm_gate(af_ctx *ctx, const void *o, int o_bf16, const void *g, int g_bf16, const float *gn_weight,
                       const float *gn_bias, void *y, int y_bf16, int64_t rows, int d_model, int num_heads, float eps,
                       af_stream_t stream) {
  const char *fn = "af_group_norm_gate";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(o && g && y && rows >= 0 && num_heads > 0 && d_model % num_heads == 0, "af_group_norm_gate",
             "null pointer or bad sizes (rows %lld, d_model %d, heads %d)", (long long)rows, d_model, num_heads);
  const int dh = d_model / num_heads;
  AF_REQUIRE(dh % 8 == 0 && dh <= 8 * 32 * 4, "af_group_norm_gate", "head_dim %d must be a multiple of 8, <= 1024",
             dh);
  AF_REQUIRE(af::aligned16(o) && af::aligned16(g) && af::aligned16(y), "af_group_norm_gate",
             "o, g and y must be 16-byte aligned");
  if (rows == 0) return AF_OK;
  return group_norm_gate(ctx, o, o_bf16, g, g_bf16, gn_weight, gn_bias, y, y_bf16, rows, d_model, num_heads, eps,
                         af::stream_of(stream), fn);
}

int af_msr_gated_decode_step_f32(af_ctx *ctx, const float *x, float *state, const float *gamma, const float *w_qkv,
                                 const float *w_g, const float *w_o, const float *gn_weight, const float *gn_bias,
                                 float eps, int B, int d, int H, float *out, af_stream_t stream) {
  const char *fn = "af_msr_gated_decode_step_f32";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(x && state && gamma && w_qkv && w_g && w_o && out, "af_msr_gated_decode_step_f32", "null pointer");
  AF_REQUIRE(B >= 0 && H > 0 && d % H == 0 && (d / H) % 8 == 0 && d / H <= 1024, "af_msr_gated_decode_step_f32",
             "bad sizes batch %d d_model %d heads %d (head_dim a multiple of 8, <= 1024)", B, d, H);
  AF_REQUIRE(af::aligned16(x) && af::aligned16(state) && af::aligned16(out), "af_msr_gated_decode_step_f32",
             "x, state and out must be 16-byte aligned");
  if (B == 0) return AF_OK;
  const int dh = d / H;
  const size_t qkv_b = align256((size_t)B * 3 * d * 4), g_b = align256((size_t)B * d * 4),
               o_b = align256((size_t)B * d * 4), y_b = align256((size_t)B * d * 4);
  void *ws = nullptr;
  int rc = af::workspace(ctx, qkv_b + g_b + o_b + y_b, &ws, fn);
  if (rc) return rc;
  uint8_t *p = static_cast<uint8_t *>(ws);
  float *qkv = reinterpret_cast<float *>(p), *gg = reinterpret_cast<float *>(p + qkv_b);
  float *o = reinterpret_cast<float *>(p + qkv_b + g_b), *yv = reinterpret_cast<float *>(p + qkv_b + g_b + o_b);
  cudaStream_t st = af::stream_of(stream);
  rc = af::linear_f32(ctx, x, d, w_qkv, d, nullptr, qkv, 3 * d, B, 3 * d, d, nullptr, 0, 0.f, 0.f, st, fn);
  if (rc) return rc;
  rc = af::linear_f32(ctx, x, d, w_g, d, nullptr, gg, d, B, d, d, nullptr, 0, 0.f, 0.f, st, fn);
  if (rc) return rc;
  rc = af::launch_retention_step(ctx, state, (int64_t)H * dh * dh, gamma, qkv, qkv + d, qkv + 2 * d, 3 * (int64_t)d,
                                 o, d, B, H, dh, nullptr, nullptr, st, fn, 0);
  if (rc) return rc;
  rc = group_norm_gate(ctx, o, 0, gg, 0, gn_weight, gn_bias, yv, 0, B, d, H, eps, st, fn);
  if (rc) return rc;
  return af::linear_f32(ctx, yv, d, w_o, d, nullptr, out, d, B, d, d, nullptr, 0, 0.f, 0.f, st, fn);
}

int af_msr_gated_prefill_bf16(af_ctx *ctx, const uint16_t *x, const uint16_t *w_qkv, const uint16_t *w_g,
                              const uint16_t *w_o, const float *gn_weight, const float *gn_bias, const float *gamma,
                              float eps, int B, int T, int d, int H, const float *state_in, float *state_out,
                              void *out, int out_bf16, int chunk, af_stream_t stream) {
  const char *fn = "af_msr_gated_prefill_bf16";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(x && w_qkv && w_g && w_o && gamma && out, "af_msr_gated_prefill_bf16", "null pointer");
  AF_REQUIRE(B >= 0 && T >= 0 && H > 0 && d == H * af::chunkwise_head_dim(), "af_msr_gated_prefill_bf16",
             "the tensor-core prefill needs head_dim %d (d_model %d, heads %d)", af::chunkwise_head_dim(), d, H);
  AF_REQUIRE(af::aligned16(x) && af::aligned16(w_qkv) && af::aligned16(w_g) && af::aligned16(w_o) &&
                 af::aligned16(out),
             "af_msr_gated_prefill_bf16", "x, weights and out must be 16-byte aligned");
  AF_REQUIRE((int64_t)B * T <= 65535LL * 128, "af_msr_gated_prefill_bf16", "B*T too large");
  int C = 0;
  if (int rc0 = af::resolve_chunk(ctx, chunk, &C, fn)) return rc0;
  if (B == 0 || T == 0) return AF_OK;
  const int64_t N = (int64_t)B * T;
  const af::ChunkPlan pl = af::chunkwise_plan(ctx->num_sms, B, T, H, ctx->chunk_segments, C);
  const size_t qkv_b = align256((size_t)N * 3 * d * 2), g_b = align256((size_t)N * d * 2),
               o_b = align256((size_t)N * d * 2), seg_b = align256(af::chunkwise_seg_state_bytes(B, H, pl));
  void *ws = nullptr;
  int rc = af::workspace(ctx, qkv_b + g_b + 2 * o_b + seg_b, &ws, fn);
  if (rc) return rc;
  uint8_t *p = static_cast<uint8_t *>(ws);
  void *qkv = p, *gg = p + qkv_b, *o = p + qkv_b + g_b, *yv = p + qkv_b + g_b + o_b;
  float *seg = seg_b ? reinterpret_cast<float *>(p + qkv_b + g_b + 2 * o_b) : nullptr;
  cudaStream_t st = af::stream_of(stream);
  af::mark_begin(ctx, st);
  af::GemmEpilogueArgs e1;
  e1.out = qkv;
  e1.ldo = 3 * d;
  e1.out_bf16 = 1;
  rc = af::tc_gemm(ctx, x, d, w_qkv, d, (int)N, 3 * d, d, false, e1, st, fn);
  if (rc) return rc;
  af::GemmEpilogueArgs eg;
  eg.out = gg;
  eg.ldo = d;
  eg.out_bf16 = 1;
  rc = af::tc_gemm(ctx, x, d, w_g, d, (int)N, d, d, false, eg, st, fn);
  if (rc) return rc;
  af::mark(ctx, "qkv_g", st);
  rc = af::retention_chunkwise_bf16(ctx, qkv, B, T, H, gamma, state_in, state_out, o, nullptr, nullptr, pl, seg, st,
                                    fn);
  if (rc) return rc;
  rc = group_norm_gate(ctx, o, 1, gg, 1, gn_weight, gn_bias, yv, 1, N, d, H, eps, st, fn);
  if (rc) return rc;
  af::mark(ctx, "group_norm_gate", st);
  af::GemmEpilogueArgs e2;
  e2.out = out;
  e2.ldo = d;
  e2.out_bf16 = out_bf16;
  rc = af::tc_gemm(ctx, yv, d, w_o, d, (int)N, d, d, false, e2, st, fn);
  af::mark(ctx, "w_o", st);
  return rc;
}

}  // extern "C"
