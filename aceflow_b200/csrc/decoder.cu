// Decoder-stack kernels: the pieces of AceEngine (aceflow-core/src/cpu/mod.rs)
// around the retention layer, batched over streams.
//
//   embed_gather      embedding rows for token ids (generate_stream_internal,
//                     cpu/mod.rs:721-726 and 757-763)
//   rmsnorm_to_bf16   RMSNorm of the fp32 residual stream into the bf16 A
//                     operand of the next projection (cpu/norm.rs:74-78)
//   argmax_rows       greedy sampling: first maximum wins (sampler.rs:118-128)
//   pack_gate_up      [gate; up] rows -> 16-row interleave for the SwiGLU
//                     GEMM epilogue (swiglu.rs:7-8 layout in, fused layout out)
#include "common.cuh"

namespace {

// x[r] = E[tok[r]] (bf16 or fp32 table -> fp32 rows).  An out-of-range id in
// a prompt keeps the previous row's embedding (the reference copies only
// when the row exists and otherwise leaves `current` unchanged,
// cpu/mod.rs:721-726); `zero_oob` selects the generated-token rule
// (cpu/mod.rs:757-763: zeros).  Rows are grouped in sequences of length T.
__global__ void embed_gather_kernel(const void *__restrict__ table, int table_bf16, const int32_t *__restrict__ tok,
                                    float *__restrict__ x, int rows, int T, int V, int d, int zero_oob) {
  const int r = blockIdx.x;
  if (r >= rows) return;
  int t = tok[r];
  if (t < 0 || t >= V) {
    if (zero_oob) {
      t = -1;
    } else {
      // last in-range id earlier in the same sequence, else zeros
      const int s0 = (r / T) * T;
      t = -1;
      for (int q = r - 1; q >= s0; --q) {
        const int u = tok[q];
        if (u >= 0 && u < V) {
          t = u;
          break;
        }
      }
    }
  }
  float *xo = x + (size_t)r * d;
  if (t < 0) {
    for (int i = threadIdx.x; i < d; i += blockDim.x) xo[i] = 0.f;
    return;
  }
  if (table_bf16) {
    const __nv_bfloat16 *e = reinterpret_cast<const __nv_bfloat16 *>(table) + (size_t)t * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) xo[i] = __bfloat162float(e[i]);
  } else {
    const float *e = reinterpret_cast<const float *>(table) + (size_t)t * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) xo[i] = e[i];
  }
}

__global__ void __launch_bounds__(256)
    rmsnorm_to_bf16_kernel(const float *__restrict__ x, const float *__restrict__ w, __nv_bfloat16 *__restrict__ y,
                           int d, float eps) {
  extern __shared__ float row[];
  __shared__ float red[32];
  const size_t off = (size_t)blockIdx.x * d;
  float ss = 0.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float a = x[off + i];
    row[i] = a;
    ss += a * a;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < (int)(blockDim.x + 31) / 32; ++i) t += red[i];
  if (w == nullptr) {  // plain fp32 -> bf16 conversion
    for (int i = threadIdx.x; i < d; i += blockDim.x) y[off + i] = __float2bfloat16(row[i]);
    return;
  }
  const float inv = 1.0f / sqrtf(t / (float)d + eps);
  for (int i = threadIdx.x; i < d; i += blockDim.x) y[off + i] = __float2bfloat16(row[i] * (inv * w[i]));
}

// The same for rows of d = 1024 * V4 floats, held in registers as float4s
// (V4 per thread, 256 threads): one read of x, one write of y.
template <int V4>
__global__ void __launch_bounds__(256)
    rmsnorm_to_bf16_reg_kernel(const float4 *__restrict__ x, const float4 *__restrict__ w, uint2 *__restrict__ y,
                               float eps) {
  constexpr int D4 = 256 * V4;
  __shared__ float red[8];
  const size_t off = (size_t)blockIdx.x * D4;
  griddep_launch();
  griddep_wait();  // x comes from the kernel before (programmatic launch)
  float4 a[V4];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < V4; ++i) {
    a[i] = x[off + threadIdx.x + i * 256];
    ss += a[i].x * a[i].x + a[i].y * a[i].y + a[i].z * a[i].z + a[i].w * a[i].w;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) t += red[i];
  const float inv = w ? 1.0f / sqrtf(t / (float)(4 * D4) + eps) : 1.f;
#pragma unroll
  for (int i = 0; i < V4; ++i) {
    const int k = threadIdx.x + i * 256;
    const float4 ww = w ? w[k] : make_float4(1.f, 1.f, 1.f, 1.f);
    __nv_bfloat162 lo = __floats2bfloat162_rn(a[i].x * (inv * ww.x), a[i].y * (inv * ww.y));
    __nv_bfloat162 hi = __floats2bfloat162_rn(a[i].z * (inv * ww.z), a[i].w * (inv * ww.w));
    y[off + k] = make_uint2(*reinterpret_cast<uint32_t *>(&lo), *reinterpret_cast<uint32_t *>(&hi));
  }
}

// One CTA per row; ties resolve to the smallest index, NaN never wins (the
// reference's strict `>` scan from index 0).
__global__ void __launch_bounds__(512) argmax_rows_kernel(const float *__restrict__ logits, int V,
                                                          int32_t *__restrict__ out) {
  const float *l = logits + (size_t)blockIdx.x * V;
  float best = l[0];
  int bi = 0;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = l[i];
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  // a NaN at index 0 makes the reference return 0
  __shared__ float sb[512];
  __shared__ int si[512];
  sb[threadIdx.x] = best;
  si[threadIdx.x] = bi;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) {
      const float ob = sb[threadIdx.x + s];
      const int oi = si[threadIdx.x + s];
      if (ob > sb[threadIdx.x] || (ob == sb[threadIdx.x] && oi < si[threadIdx.x])) {
        sb[threadIdx.x] = ob;
        si[threadIdx.x] = oi;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) out[blockIdx.x] = (l[0] != l[0]) ? 0 : si[0];
}

// dst row p: group g = p / 32, j = p % 32; j < 16 -> gate row 16g + j,
// else up row 16g + j - 16 (src rows: gate 0..f-1, then up f..2f-1).
__global__ void pack_gate_up_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int f,
                                    int row_bytes) {
  const int p = blockIdx.x;
  const int g = p / 32, j = p % 32;
  const int s = j < 16 ? 16 * g + j : f + 16 * g + (j - 16);
  const uint8_t *a = src + (size_t)s * row_bytes;
  uint8_t *b = dst + (size_t)p * row_bytes;
  for (int i = threadIdx.x * 16; i < row_bytes; i += blockDim.x * 16)
    *reinterpret_cast<uint4 *>(b + i) = *reinterpret_cast<const uint4 *>(a + i);
}

}  // namespace

extern "C" {

int af_embed_gather(af_ctx *ctx, const void *table, int table_bf16, const int32_t *tokens, float *x, int rows, int T,
                    int vocab, int d, int zero_oob, af_stream_t stream) {
  const char *fn = "af_embed_gather";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(table && tokens && x, "af_embed_gather", "null pointer");
  AF_REQUIRE(rows >= 0 && T > 0 && vocab > 0 && d > 0, "af_embed_gather", "bad sizes");
  if (rows == 0) return AF_OK;
  embed_gather_kernel<<<rows, 256, 0, af::stream_of(stream)>>>(table, table_bf16, tokens, x, rows, T, vocab, d,
                                                               zero_oob);
  return af::launched(ctx, fn);
}

int af_rmsnorm_to_bf16(af_ctx *ctx, const float *x, const float *w, uint16_t *y, int rows, int d, float eps,
                       af_stream_t stream) {
  const char *fn = "af_rmsnorm_to_bf16";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(x && y, "af_rmsnorm_to_bf16", "null pointer");
  AF_REQUIRE(rows >= 0 && d > 0 && d <= 12288, "af_rmsnorm_to_bf16", "bad sizes rows=%d d=%d", rows, d);
  return af::rmsnorm_to_bf16(ctx, x, w, y, rows, d, eps, af::stream_of(stream), fn, false);
}

int af_argmax_rows(af_ctx *ctx, const float *logits, int rows, int V, int32_t *out, af_stream_t stream) {
  const char *fn = "af_argmax_rows";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(logits && out && rows >= 0 && V > 0, "af_argmax_rows", "bad arguments");
  if (rows == 0) return AF_OK;
  argmax_rows_kernel<<<rows, 512, 0, af::stream_of(stream)>>>(logits, V, out);
  return af::launched(ctx, fn);
}

int af_pack_gate_up(af_ctx *ctx, const void *src, void *dst, int f, int d, int elem_bytes, af_stream_t stream) {
  const char *fn = "af_pack_gate_up";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(src && dst && src != dst, "af_pack_gate_up", "src and dst must be distinct buffers");
  AF_REQUIRE(f > 0 && f % 16 == 0, "af_pack_gate_up", "ffn dim %d must be a multiple of 16", f);
  AF_REQUIRE((elem_bytes == 2 || elem_bytes == 4) && ((int64_t)d * elem_bytes) % 16 == 0 && af::aligned16(src) &&
                 af::aligned16(dst),
             "af_pack_gate_up", "rows must be 16-byte aligned");
  pack_gate_up_kernel<<<2 * f, 128, 0, af::stream_of(stream)>>>(static_cast<const uint8_t *>(src),
                                                               static_cast<uint8_t *>(dst), f, d * elem_bytes);
  return af::launched(ctx, fn);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decoder layer (AceEngine.forward_layer_internal, cpu/mod.rs:646-706) for a
// batch of streams:
//   h = RMSNorm1(x); qkv = h W_qkv^T; o = retention(qkv)     (state in place)
//   x += W_o RMSNorm_ret(o)        (1/rms applied per row in the GEMM epilogue,
//                                   residual added in the same epilogue)
//   h = RMSNorm2(x); x += W_down (silu(g) * u),  [g|u] = h W_gate_up^T
//                                  (SwiGLU in the gate/up GEMM epilogue)
namespace af {
int rmsnorm_to_bf16(af_ctx *ctx, const float *x, const float *w, uint16_t *y, int rows, int d, float eps,
                    cudaStream_t st, const char *fn, bool pdl) {
  if (rows == 0) return AF_OK;
  const bool al = aligned16(x) && aligned16(y) && (w == nullptr || aligned16(w));
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  const float4 *w4 = reinterpret_cast<const float4 *>(w);
  uint2 *y4 = reinterpret_cast<uint2 *>(y);
  pdl = pdl && ctx->pdl;
  cudaError_t e = cudaSuccess;
  const dim3 g(rows), b(256);
  if (al && d == 1024) e = launch_kernel(rmsnorm_to_bf16_reg_kernel<1>, g, b, 0, st, pdl, x4, w4, y4, eps);
  else if (al && d == 2048) e = launch_kernel(rmsnorm_to_bf16_reg_kernel<2>, g, b, 0, st, pdl, x4, w4, y4, eps);
  else if (al && d == 4096) e = launch_kernel(rmsnorm_to_bf16_reg_kernel<4>, g, b, 0, st, pdl, x4, w4, y4, eps);
  else if (al && d == 8192) e = launch_kernel(rmsnorm_to_bf16_reg_kernel<8>, g, b, 0, st, pdl, x4, w4, y4, eps);
  else rmsnorm_to_bf16_kernel<<<rows, 256, (size_t)d * 4, st>>>(x, w, reinterpret_cast<__nv_bfloat16 *>(y), d, eps);
  if (e != cudaSuccess) return fail(AF_ERR_CUDA, "%s: launch: %s", fn, cudaGetErrorString(e));
  return launched(ctx, fn);
}

int launch_rmsnorm_f32(af_ctx *ctx, const float *x, const float *res, const float *w, float *y, float *sum_out,
                       int rows, int d, float eps, cudaStream_t st, const char *fn);

static int gemm(af_ctx *ctx, const void *A, const void *B, int M, int N, int K, bool fp32, void *out, int out_bf16,
                const float *residual, const float *parts, int nparts, float inv_d, float eps, int swiglu,
                cudaStream_t st, const char *fn) {
  GemmEpilogueArgs e;
  e.out = out;
  e.ldo = swiglu ? N / 2 : N;
  e.out_bf16 = out_bf16;
  e.residual = residual;
  e.ldr = N;
  e.row_parts = parts;
  e.nparts = nparts;
  e.inv_d = inv_d;
  e.eps = eps;
  e.swiglu = swiglu;
  return tc_gemm(ctx, A, K, B, K, M, N, K, fp32, e, st, fn);
}

static size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

// Transposed decode projection: W[rows_w][K] as the 128-row operand, the
// activations [batch][K] as one N tile (each weight tile is read by exactly
// one CTA), split-K to fill the SMs.
constexpr int kTransPartials = 4;
static int trans_tile(int batch) {
  int bn = 16;
  while (bn < batch) bn *= 2;
  return bn;
}
static int trans_splits(const af_ctx *ctx, int rows_w, int K, int max_splits) {
  const int mt = (rows_w + 127) / 128;
  int sp = ctx->num_sms / mt;
  const int nk = (K + 63) / 64;
  if (sp > nk / 2) sp = nk / 2;
  if (sp > max_splits) sp = max_splits;
  return sp < 1 ? 1 : sp;
}
static int gemm_t(af_ctx *ctx, const void *W, int rows_w, const void *X, int batch, int K, GemmEpilogueArgs e,
                  int max_splits, cudaStream_t st, const char *fn) {
  e.trans = 1;
  e.force_bn = trans_tile(batch);
  e.force_splits = max_splits > 1 ? trans_splits(ctx, rows_w, K, max_splits) : 1;
  return tc_gemm(ctx, W, K, X, K, rows_w, batch, K, false, e, st, fn);
}

static int check_layer(const af_layer_weights *w, int B, int d, int H, int f, const char *fn) {
  if (!w || !w->w_qkv || !w->w_o || !w->w_gate_up || !w->w_down || !w->norm1 || !w->norm2 || !w->ret_norm)
    return fail(AF_ERR_ARG, "%s: null weight pointer", fn);
  if (B < 0 || d <= 0 || H <= 0 || d % H || f <= 0 || f % 16)
    return fail(AF_ERR_ARG, "%s: bad sizes batch=%d d=%d heads=%d ffn=%d (ffn must be a multiple of 16)", fn, B, d,
                H, f);
  if (d % 8 || f % 8) return fail(AF_ERR_ARG, "%s: d_model and ffn must be multiples of 8", fn);
  return AF_OK;
}
}  // namespace af

extern "C" int af_decoder_layer_decode(af_ctx *ctx, const af_layer_weights *w, int weights_bf16, float *x,
                                       float *state, int64_t state_batch_stride, const float *gamma, float eps,
                                       int B, int d, int H, int f, af_stream_t stream) {
  const char *fn = "af_decoder_layer_decode";
  AF_ENTER(ctx, fn);
  int rc = af::check_layer(w, B, d, H, f, fn);
  if (rc) return rc;
  AF_REQUIRE(x && state && gamma && af::aligned16(x) && af::aligned16(state), "af_decoder_layer_decode",
             "x and state must be non-null and 16-byte aligned");
  const int dh = d / H;
  AF_REQUIRE(dh == 64 || dh == 128 || dh == 256, "af_decoder_layer_decode", "head_dim %d must be 64, 128 or 256",
             dh);
  AF_REQUIRE(state_batch_stride >= (int64_t)H * dh * dh && state_batch_stride % 4 == 0, "af_decoder_layer_decode",
             "bad state_batch_stride");
  if (B == 0) return AF_OK;
  const bool fp32 = !weights_bf16;
  // bf16 weights, up to 256 streams: every projection runs transposed
  const bool tr = !fp32 && B <= 256 && d % 64 == 0 && f % 64 == 0;
  const size_t ab = fp32 ? 4 : 2;  // activation bytes feeding the GEMMs
  const size_t h_b = af::align256((size_t)B * d * ab),
               qkv_b = af::align256((size_t)(tr ? af::kTransPartials : 1) * B * 3 * d * 4),
               o_b = af::align256((size_t)B * d * ab), ss_b = af::align256((size_t)B * H * 4),
               hid_b = af::align256((size_t)B * f * ab);
  void *ws = nullptr;
  rc = af::workspace(ctx, h_b + qkv_b + o_b + ss_b + hid_b, &ws, fn);
  if (rc) return rc;
  uint8_t *p = static_cast<uint8_t *>(ws);
  void *h = p;
  float *qkv = reinterpret_cast<float *>(p + h_b);
  void *o = p + h_b + qkv_b;
  float *ss = reinterpret_cast<float *>(p + h_b + qkv_b + o_b);
  void *hid = p + h_b + qkv_b + o_b + ss_b;
  cudaStream_t st = af::stream_of(stream);
  if (tr) {
    const int tm = ctx->decode_transposed;  // which projections run as W . x^T
    // Every kernel of the chain is a programmatic dependent launch: the
    // weight GEMMs stream their first weight tiles while the kernel before
    // drains.  1. h = bf16(RMSNorm1(x))
    rc = af::rmsnorm_to_bf16(ctx, x, w->norm1, (uint16_t *)h, B, d, eps, st, fn, true);
    if (rc) return rc;
    // 2. qkv (transposed: split-K partial buffers, summed by the state stream)
    int nsp = 1;
    if (tm & 1) {
      af::GemmEpilogueArgs e1;
      e1.out = qkv;
      e1.ldo = 3 * d;
      e1.split_stride = (int64_t)B * 3 * d;
      e1.max_partials = af::kTransPartials;
      e1.pdl = 1;
      e1.pre_operand = 1;
      rc = af::gemm_t(ctx, w->w_qkv, 3 * d, h, B, d, e1, af::kTransPartials, st, fn);
      nsp = af::trans_splits(ctx, 3 * d, d, af::kTransPartials);
    } else {
      rc = af::gemm(ctx, h, w->w_qkv, B, 3 * d, d, false, qkv, 0, nullptr, nullptr, 0, 0.f, 0.f, 0, st, fn);
    }
    if (rc) return rc;
    // 3. state stream
    rc = af::launch_retention_step(ctx, state, state_batch_stride, gamma, qkv, qkv + d, qkv + 2 * d, 3 * (int64_t)d,
                                   (float *)o, d, B, H, dh, w->ret_norm, ss, st, fn, 1, nullptr, 0, 0, 0, nsp,
                                   (int64_t)B * 3 * d, true);
    if (rc) return rc;
    // 4. x += diag(1/rms) (o*w) W_o^T (transposed: atomics over K splits, 1/rms per column)
    if (tm & 2) {
      af::GemmEpilogueArgs e2;
      e2.out = x;
      e2.ldo = d;
      e2.accumulate = 1;
      e2.row_parts = ss;
      e2.nparts = H;
      e2.inv_d = 1.0f / (float)d;
      e2.eps = eps;
      e2.pdl = 1;
      e2.pre_operand = 1;
      rc = af::gemm_t(ctx, w->w_o, d, o, B, d, e2, 8, st, fn);
    } else {
      rc = af::gemm(ctx, o, w->w_o, B, d, d, false, x, 0, x, ss, H, 1.0f / (float)d, eps, 0, st, fn);
    }
    if (rc) return rc;
    // 5. h = bf16(RMSNorm2(x)); 6. hid = silu(g) * u
    rc = af::rmsnorm_to_bf16(ctx, x, w->norm2, (uint16_t *)h, B, d, eps, st, fn, true);
    if (rc) return rc;
    if (tm & 4) {
      af::GemmEpilogueArgs e3;
      e3.out = hid;
      e3.ldo = f;
      e3.out_bf16 = 1;
      e3.swiglu = 1;
      e3.pdl = 1;
      e3.pre_operand = 1;
      rc = af::gemm_t(ctx, w->w_gate_up, 2 * f, h, B, d, e3, 1, st, fn);
    } else {
      rc = af::gemm(ctx, h, w->w_gate_up, B, 2 * f, d, false, hid, 1, nullptr, nullptr, 0, 0.f, 0.f, 1, st, fn);
    }
    if (rc) return rc;
    // 7. x += hid W_down^T
    if (tm & 8) {
      af::GemmEpilogueArgs e4;
      e4.out = x;
      e4.ldo = d;
      e4.accumulate = 1;
      e4.pdl = 1;
      e4.pre_operand = 1;
      return af::gemm_t(ctx, w->w_down, d, hid, B, f, e4, 8, st, fn);
    }
    return af::gemm(ctx, hid, w->w_down, B, d, f, false, x, 0, x, nullptr, 0, 0.f, 0.f, 0, st, fn);
  }
  if (fp32) rc = af::launch_rmsnorm_f32(ctx, x, nullptr, w->norm1, (float *)h, nullptr, B, d, eps, st, fn);
  else rc = af_rmsnorm_to_bf16(ctx, x, w->norm1, (uint16_t *)h, B, d, eps, stream);
  if (rc) return rc;
  rc = af::gemm(ctx, h, w->w_qkv, B, 3 * d, d, fp32, qkv, 0, nullptr, nullptr, 0, 0.f, 0.f, 0, st, fn);
  if (rc) return rc;
  rc = af::launch_retention_step(ctx, state, state_batch_stride, gamma, qkv, qkv + d, qkv + 2 * d, 3 * (int64_t)d,
                                 (float *)o, d, B, H, dh, w->ret_norm, ss, st, fn, fp32 ? 0 : 1);
  if (rc) return rc;
  rc = af::gemm(ctx, o, w->w_o, B, d, d, fp32, x, 0, x, ss, H, 1.0f / (float)d, eps, 0, st, fn);
  if (rc) return rc;
  if (fp32) rc = af::launch_rmsnorm_f32(ctx, x, nullptr, w->norm2, (float *)h, nullptr, B, d, eps, st, fn);
  else rc = af_rmsnorm_to_bf16(ctx, x, w->norm2, (uint16_t *)h, B, d, eps, stream);
  if (rc) return rc;
  rc = af::gemm(ctx, h, w->w_gate_up, B, 2 * f, d, fp32, hid, fp32 ? 0 : 1, nullptr, nullptr, 0, 0.f, 0.f, 1, st, fn);
  if (rc) return rc;
  return af::gemm(ctx, hid, w->w_down, B, d, f, fp32, x, 0, x, nullptr, 0, 0.f, 0.f, 0, st, fn);
}

extern "C" int af_decoder_layer_prefill(af_ctx *ctx, const af_layer_weights *w, float *x, const float *state_in,
                                        float *state_out, const float *gamma, float eps, int B, int T, int d, int H,
                                        int f, af_stream_t stream) {
  const char *fn = "af_decoder_layer_prefill";
  AF_ENTER(ctx, fn);
  int rc = af::check_layer(w, B, d, H, f, fn);
  if (rc) return rc;
  AF_REQUIRE(x && gamma && af::aligned16(x), "af_decoder_layer_prefill", "x must be non-null and 16-byte aligned");
  AF_REQUIRE(d == H * af::chunkwise_head_dim(), "af_decoder_layer_prefill", "head_dim must be %d",
             af::chunkwise_head_dim());
  AF_REQUIRE((int64_t)B * T <= 65535LL * 128, "af_decoder_layer_prefill", "batch*T too large");
  if (B == 0 || T == 0) return AF_OK;
  const int N = B * T;
  const int C = af::chunkwise_default_chunk(ctx);
  const int parts = H * af::chunkwise_parts(C);
  const size_t h_b = af::align256((size_t)N * d * 2), qkv_b = af::align256((size_t)N * 3 * d * 2),
               o_b = af::align256((size_t)N * d * 2), ss_b = af::align256((size_t)N * parts * 4),
               hid_b = af::align256((size_t)N * f * 2);
  const af::ChunkPlan pl = af::chunkwise_plan(ctx->num_sms, B, T, H, ctx->chunk_segments, C);
  const size_t seg_b = af::chunkwise_seg_state_bytes(B, H, pl);
  void *ws = nullptr;
  rc = af::workspace(ctx, h_b + qkv_b + o_b + ss_b + hid_b + seg_b, &ws, fn);
  if (rc) return rc;
  uint8_t *p = static_cast<uint8_t *>(ws);
  uint16_t *h = reinterpret_cast<uint16_t *>(p);
  void *qkv = p + h_b;
  void *o = p + h_b + qkv_b;
  float *ss = reinterpret_cast<float *>(p + h_b + qkv_b + o_b);
  void *hid = p + h_b + qkv_b + o_b + ss_b;
  float *seg = seg_b ? reinterpret_cast<float *>(p + h_b + qkv_b + o_b + ss_b + hid_b) : nullptr;
  cudaStream_t st = af::stream_of(stream);
  rc = af_rmsnorm_to_bf16(ctx, x, w->norm1, h, N, d, eps, stream);
  if (rc) return rc;
  rc = af::gemm(ctx, h, w->w_qkv, N, 3 * d, d, false, qkv, 1, nullptr, nullptr, 0, 0.f, 0.f, 0, st, fn);
  if (rc) return rc;
  rc = af::retention_chunkwise_bf16(ctx, qkv, B, T, H, gamma, state_in, state_out, o, w->ret_norm, ss, pl, seg, st,
                                    fn);
  if (rc) return rc;
  rc = af::gemm(ctx, o, w->w_o, N, d, d, false, x, 0, x, ss, parts, 1.0f / (float)d, eps, 0, st, fn);
  if (rc) return rc;
  rc = af_rmsnorm_to_bf16(ctx, x, w->norm2, h, N, d, eps, stream);
  if (rc) return rc;
  rc = af::gemm(ctx, h, w->w_gate_up, N, 2 * f, d, false, hid, 1, nullptr, nullptr, 0, 0.f, 0.f, 1, st, fn);
  if (rc) return rc;
  return af::gemm(ctx, hid, w->w_down, N, d, f, false, x, 0, x, nullptr, 0, 0.f, 0.f, 0, st, fn);
}

// logits = table . norm(x) (tied LM head, sampler.rs:67-81) then first-max
// argmax.  `final_norm` (may be NULL) is AceEngine's optional final RMSNorm.
extern "C" int af_lm_head_argmax(af_ctx *ctx, const float *x, const float *final_norm, float eps, const void *table,
                                 int table_bf16, int B, int V, int d, float *logits, int32_t *tokens,
                                 af_stream_t stream) {
  const char *fn = "af_lm_head_argmax";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(x && table && logits && tokens && B >= 0 && V > 0 && d > 0 && d % 8 == 0, "af_lm_head_argmax",
             "bad arguments");
  if (B == 0) return AF_OK;
  cudaStream_t st = af::stream_of(stream);
  const bool fp32 = !table_bf16;
  void *ws = nullptr;
  int rc = af::workspace(ctx, af::align256((size_t)B * d * 4), &ws, fn);
  if (rc) return rc;
  if (fp32) {
    if (final_norm) rc = af::launch_rmsnorm_f32(ctx, x, nullptr, final_norm, (float *)ws, nullptr, B, d, eps, st, fn);
    else rc = (cudaMemcpyAsync(ws, x, (size_t)B * d * 4, cudaMemcpyDeviceToDevice, st) == cudaSuccess)
                  ? AF_OK
                  : af::fail(AF_ERR_CUDA, "%s: copy failed", fn);
  } else {
    rc = af_rmsnorm_to_bf16(ctx, x, final_norm, (uint16_t *)ws, B, d, final_norm ? eps : -1.f, stream);
  }
  if (rc) return rc;
  rc = af::gemm(ctx, ws, table, B, V, d, fp32, logits, 0, nullptr, nullptr, 0, 0.f, 0.f, 0, st, fn);
  if (rc) return rc;
  return af_argmax_rows(ctx, logits, B, V, tokens, stream);
}
