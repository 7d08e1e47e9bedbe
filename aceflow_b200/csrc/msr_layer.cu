// Fused MultiScaleRetention layer entry points.
//
// Decode step (one token per stream, fp32, state in HBM):
//   1. qkv = x . W_qkv^T                        (3xTF32 tensor-core GEMM)
//   2. retention step per (b, h), writing o * ret_norm_w and per-head sum o^2
//   3. out = diag(1/rms) (o * w) . W_o^T         (GEMM, norm applied per row)
// This is AceEngine.forward_layer_internal's retention half
// (aceflow-core/src/cpu/mod.rs:651-678) for a batch of streams, with the
// Python module's RMSNorm placement (aceflow/nn/retention.py:64-65).
#include "common.cuh"

namespace af {
int linear_f32(af_ctx *ctx, const float *x, int64_t ldx, const float *w, int64_t ldw, const float *bias, float *y,
               int64_t ldy, int M, int N, int K, const float *parts, int nparts, float inv_d, float eps,
               cudaStream_t st, const char *fn);

// Workspace layout of the decode step, in floats: qkv [B][3d], o [B][d],
// sumsq [B][H].
size_t msr_decode_scratch_floats(int batch, int d, int H) {
  return (size_t)batch * (3 * (size_t)d) + (size_t)batch * d + (size_t)batch * H;
}

int msr_decode_step_impl(af_ctx *ctx, const float *x, float *state, const float *gamma, const float *w_qkv,
                         const float *w_o, const float *ret_norm_w, float eps, int B, int d, int H, float *out,
                         float *scratch, cudaStream_t st, const char *fn) {
  const int dh = d / H;
  float *qkv = scratch;
  float *o = qkv + (size_t)B * 3 * d;
  float *sumsq = o + (size_t)B * d;
  const int64_t sbs = (int64_t)H * dh * dh;
  auto qkv_gemm = [&](int r0, int rows, cudaStream_t s) {
    return linear_f32(ctx, x + (size_t)r0 * d, d, w_qkv, d, nullptr, qkv + (size_t)r0 * 3 * d, 3 * d, rows, 3 * d, d,
                      nullptr, 0, 0.f, 0.f, s, fn);
  };
  auto retention = [&](int r0, int rows, cudaStream_t s) {
    const float *q = qkv + (size_t)r0 * 3 * d;
    return launch_retention_step(ctx, state + (size_t)r0 * sbs, sbs, gamma, q, q + d, q + 2 * d, 3 * (int64_t)d,
                                 o + (size_t)r0 * d, d, rows, H, dh, ret_norm_w, sumsq + (size_t)r0 * H, s, fn, 0);
  };
  auto out_gemm = [&](int r0, int rows, cudaStream_t s) {
    return linear_f32(ctx, o + (size_t)r0 * d, d, w_o, d, nullptr, out + (size_t)r0 * d, d, rows, d, d,
                      sumsq + (size_t)r0 * H, H, 1.0f / (float)d, eps, s, fn);
  };
  const int sr = ctx->decode_slice_rows;
  const int nsl = sr > 0 ? (B + sr - 1) / sr : 1;
  if (nsl < 2 || nsl > af_ctx::kMaxSlices) {
    int rc = qkv_gemm(0, B, st);
    if (rc) return rc;
    rc = retention(0, B, st);
    if (rc) return rc;
    return out_gemm(0, B, st);
  }
  // Overlapped: slice i's projection (tensor cores) runs while slice i-1
  // streams its state (HBM) on a high-priority stream, and slice i-2 runs its
  // output projection; fork/join through events on the caller's stream.
  cudaStream_t s_ret = ctx->side[0], s_out = ctx->side[1];
  AF_CUDA(cudaEventRecord(ctx->ev_fork, st), fn);
  AF_CUDA(cudaStreamWaitEvent(s_ret, ctx->ev_fork, 0), fn);
  AF_CUDA(cudaStreamWaitEvent(s_out, ctx->ev_fork, 0), fn);
  for (int i = 0; i < nsl; ++i) {
    const int r0 = i * sr, rows = B - r0 < sr ? B - r0 : sr;
    int rc = qkv_gemm(r0, rows, st);
    if (rc) return rc;
    AF_CUDA(cudaEventRecord(ctx->ev_a[i], st), fn);
    AF_CUDA(cudaStreamWaitEvent(s_ret, ctx->ev_a[i], 0), fn);
    rc = retention(r0, rows, s_ret);
    if (rc) return rc;
    AF_CUDA(cudaEventRecord(ctx->ev_b[i], s_ret), fn);
    AF_CUDA(cudaStreamWaitEvent(s_out, ctx->ev_b[i], 0), fn);
    rc = out_gemm(r0, rows, s_out);
    if (rc) return rc;
  }
  AF_CUDA(cudaEventRecord(ctx->ev_join, s_out), fn);
  AF_CUDA(cudaStreamWaitEvent(st, ctx->ev_join, 0), fn);
  return AF_OK;
}

// Decode step from weights split beforehand.  The QKV weights are packed
// head-major ([H][q|k|v][dh][d], af_pack_qkv_heads) and split into tf32
// hi + lo (af_split_tf32); W_o is split as it is.  The input is split by a
// small kernel, the state-stream kernel writes its output split, and both
// projections run as pre-split 3xTF32 GEMMs.
//
// With G > 1 head groups the step is a three-stream pipeline: the QKV GEMM
// of group g+1 (tensor cores, caller's stream) runs while group g streams its
// state (HBM, high-priority side stream) and group g-1's W_o product
// (tensor cores, second side stream) accumulates into an fp32 buffer; the
// RMSNorm row scale is applied once at the end.  Head-major packing makes
// every group's weights a contiguous block, so no weight is read twice.
// Workspace floats: x hi/lo 2Bd, qkv 3Bd, o hi/lo 2Bd, partial sums Bd, sumsq BH.
// QKV split-K partial buffers of the transposed projection (kQkvPartials - 1
// beyond the one the sequential layout already holds)
constexpr int kQkvPartials = 4;
size_t msr_decode_split_scratch_floats(int B, int d, int H) {
  return (size_t)B * ((5 + 3 * kQkvPartials) * (size_t)d + H) + 64;
}

// Split count of the transposed QKV projection (weights as the 128-row
// operand, the batch as one 128- or 256-wide tile), or 0 when the batch
// does not fit one tile or is small enough for the direct form.
static int qkv_trans_splits(const af_ctx *ctx, int B, int d) {
  if (B <= 64 || B > 256 || d % 32 != 0) return 0;
  const int mtiles = (3 * d + 127) / 128;
  int sp = ctx->num_sms / mtiles;
  const int nk = d / 32;
  if (sp > nk / 4) sp = nk / 4;
  if (sp > kQkvPartials) sp = kQkvPartials;
  return sp < 1 ? 1 : sp;
}

namespace {
__global__ void rowscale_kernel(const float *__restrict__ P, const float *__restrict__ sumsq, float *__restrict__ out,
                                int d, int H, float inv_d, float eps) {
  const int b = blockIdx.x;
  __shared__ float s_scale;
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int h = 0; h < H; ++h) t += sumsq[(size_t)b * H + h];
    s_scale = 1.0f / sqrtf(t * inv_d + eps);
  }
  __syncthreads();
  const float sc = s_scale;
  const float4 *p4 = reinterpret_cast<const float4 *>(P + (size_t)b * d);
  float4 *o4 = reinterpret_cast<float4 *>(out + (size_t)b * d);
  for (int i = threadIdx.x; i < d / 4; i += blockDim.x) {
    const float4 v = p4[i];
    o4[i] = make_float4(v.x * sc, v.y * sc, v.z * sc, v.w * sc);
  }
}

// dst row (h*3 + part)*dh + i  <-  src row part*d + h*dh + i
__global__ void pack_qkv_heads_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int d, int H,
                                      int row_bytes) {
  const int r = blockIdx.x;  // destination row
  const int dh = d / H;
  const int h = r / (3 * dh), part = (r / dh) % 3, i = r % dh;
  const uint8_t *a = src + ((size_t)part * d + (size_t)h * dh + i) * row_bytes;
  uint8_t *o = dst + (size_t)r * row_bytes;
  for (int c = threadIdx.x * 16; c < row_bytes; c += blockDim.x * 16)
    *reinterpret_cast<uint4 *>(o + c) = *reinterpret_cast<const uint4 *>(a + c);
}
}  // namespace

int msr_decode_step_split_impl(af_ctx *ctx, const float *x, float *state, const float *gamma, const float *wq_hi,
                               const float *wq_lo, const float *wo_hi, const float *wo_lo, const float *ret_norm_w,
                               float eps, int B, int d, int H, float *out, float *scratch, cudaStream_t st,
                               const char *fn) {
  const int dh = d / H;
  float *x_hi = scratch, *x_lo = x_hi + (size_t)B * d;
  float *o_hi = x_lo + (size_t)B * d, *o_lo = o_hi + (size_t)B * d, *P = o_lo + (size_t)B * d;
  float *sumsq = P + (size_t)B * d;
  float *qkv = sumsq + (((size_t)B * H + 63) & ~size_t(63));  // kQkvPartials x [B][3d]
  const int64_t sbs = (int64_t)H * dh * dh;
  int G = ctx->decode_head_groups;
  if (G < 2 || H % G != 0 || G > af_ctx::kMaxSlices) G = 1;
  const int Hg = H / G, Ng = 3 * Hg * dh;
  // the sequential step's W_o GEMM accumulates into out, zeroed here
  int rc = split_tf32(ctx, x, x_hi, x_lo, (int64_t)B * d, st, fn, G == 1 ? out : nullptr, G == 1);
  if (rc) return rc;
  auto qkv_gemm = [&](int g, cudaStream_t s) {
    GemmEpilogueArgs e;
    e.out = qkv + (size_t)g * B * Ng;
    e.ldo = Ng;
    return tc_gemm_presplit(ctx, x_hi, x_lo, d, wq_hi + (size_t)g * Ng * d, wq_lo + (size_t)g * Ng * d, d, B, Ng, d, e,
                            s, fn);
  };
  auto retention = [&](int g, cudaStream_t s) {
    const float *q = qkv + (size_t)g * B * Ng;
    return launch_retention_step(ctx, state, sbs, gamma, q, q + dh, q + 2 * dh, Ng, o_hi, d, B, H, dh, ret_norm_w,
                                 sumsq, s, fn, 0, o_lo, g * Hg, Hg, 3 * (int64_t)dh);
  };
  if (G == 1) {
    const int nsp = qkv_trans_splits(ctx, B, d);
    if (nsp > 0) {
      // qkv^T = W_qkv . x^T: each weight tile is read by one CTA, split-K
      // partials go to separate buffers that the retention kernel sums
      GemmEpilogueArgs e;
      e.out = qkv;
      e.ldo = 3 * d;
      e.trans = 1;
      e.split_stride = (int64_t)B * 3 * d;
      e.max_partials = kQkvPartials;
      e.force_bn = B > 128 ? 256 : 128;
      e.force_splits = nsp;
      e.pdl = 1;  // programmatic dependent launches: weight tiles stream while the split kernel drains
      e.pre_operand = 1;
      e.pair = ctx->decode_pairs;  // CTA pairs: each CTA fetches half of the activation tile
      rc = tc_gemm_presplit(ctx, wq_hi, wq_lo, d, x_hi, x_lo, d, 3 * d, B, d, e, st, fn);
      if (rc) return rc;
      rc = launch_retention_step(ctx, state, sbs, gamma, qkv, qkv + dh, qkv + 2 * dh, 3 * (int64_t)d, o_hi, d, B, H,
                                 dh, ret_norm_w, sumsq, st, fn, 0, o_lo, 0, H, 3 * (int64_t)dh, nsp,
                                 (int64_t)B * 3 * d, true);
    } else {
      rc = qkv_gemm(0, st);
      if (rc) return rc;
      rc = retention(0, st);
    }
    if (rc) return rc;
    GemmEpilogueArgs e2;
    e2.out = out;
    e2.ldo = d;
    e2.accumulate = 1;  // into the zeroed out: split-K needs no memset
    e2.pdl = 1;
    e2.pre_operand = 2;  // W_o (B) does not depend on the state stream
    // (W_o on CTA pairs measured slower: 25.9 vs 24.3 us with per-thread atomics, and with the
    // staged reduce-add epilogue 0.2279 vs 0.2272 ms per step: 16 K slices per split are too few)
    e2.row_parts = sumsq;
    e2.nparts = H;
    e2.inv_d = 1.0f / (float)d;
    e2.eps = eps;
    return tc_gemm_presplit(ctx, o_hi, o_lo, d, wo_hi, wo_lo, d, B, d, d, e2, st, fn);
  }
  cudaStream_t s_ret = ctx->side[0], s_out = ctx->side[1];
  AF_CUDA(cudaEventRecord(ctx->ev_fork, st), fn);
  AF_CUDA(cudaStreamWaitEvent(s_ret, ctx->ev_fork, 0), fn);
  AF_CUDA(cudaStreamWaitEvent(s_out, ctx->ev_fork, 0), fn);
  AF_CUDA(cudaMemsetAsync(P, 0, (size_t)B * d * sizeof(float), s_out), fn);
  for (int g = 0; g < G; ++g) {
    rc = qkv_gemm(g, st);
    if (rc) return rc;
    AF_CUDA(cudaEventRecord(ctx->ev_a[g], st), fn);
    AF_CUDA(cudaStreamWaitEvent(s_ret, ctx->ev_a[g], 0), fn);
    rc = retention(g, s_ret);
    if (rc) return rc;
    AF_CUDA(cudaEventRecord(ctx->ev_b[g], s_ret), fn);
    AF_CUDA(cudaStreamWaitEvent(s_out, ctx->ev_b[g], 0), fn);
    GemmEpilogueArgs e;
    e.out = P;
    e.ldo = d;
    e.accumulate = 1;
    const size_t c0 = (size_t)g * Hg * dh;
    rc = tc_gemm_presplit(ctx, o_hi + c0, o_lo + c0, d, wo_hi + c0, wo_lo + c0, d, B, d, Hg * dh, e, s_out, fn);
    if (rc) return rc;
  }
  rowscale_kernel<<<B, 256, 0, s_out>>>(P, sumsq, out, d, H, 1.0f / (float)d, eps);
  rc = launched(ctx, fn);
  if (rc) return rc;
  AF_CUDA(cudaEventRecord(ctx->ev_join, s_out), fn);
  AF_CUDA(cudaStreamWaitEvent(st, ctx->ev_join, 0), fn);
  return AF_OK;
}

int pack_qkv_heads(af_ctx *ctx, const void *src, void *dst, int d, int H, int elem_bytes, cudaStream_t st,
                   const char *fn) {
  pack_qkv_heads_kernel<<<3 * d, 128, 0, st>>>(static_cast<const uint8_t *>(src), static_cast<uint8_t *>(dst), d, H,
                                                d * elem_bytes);
  return launched(ctx, fn);
}

int check_msr_decode(const char *fn, const float *x, float *state, const float *gamma, const float *w_qkv,
                     const float *w_o, const float *ret_norm_w, int B, int d, int H, const float *out) {
  if (!x || !state || !gamma || !w_qkv || !w_o || !ret_norm_w || !out)
    return fail(AF_ERR_ARG, "%s: null pointer", fn);
  if (B < 0 || d <= 0 || H <= 0 || d % H != 0)
    return fail(AF_ERR_ARG, "%s: d_model (%d) must be divisible by num_heads (%d), batch %d >= 0", fn, d, H, B);
  const int dh = d / H;
  if (dh % 4 != 0 || dh > 1024) return fail(AF_ERR_ARG, "%s: head_dim %d must be a multiple of 4 and <= 1024", fn, dh);
  if (!aligned16(state)) return fail(AF_ERR_ARG, "%s: state must be 16-byte aligned", fn);
  return AF_OK;
}

}  // namespace af

extern "C" int af_msr_decode_step_f32(af_ctx *ctx, const float *x, float *state, const float *gamma,
                                      const float *w_qkv, const float *w_o, const float *ret_norm_w, float eps,
                                      int B, int d, int H, float *out, af_stream_t stream) {
  const char *fn = "af_msr_decode_step_f32";
  AF_ENTER(ctx, fn);
  int rc = af::check_msr_decode(fn, x, state, gamma, w_qkv, w_o, ret_norm_w, B, d, H, out);
  if (rc) return rc;
  if (B == 0) return AF_OK;
  void *ws = nullptr;
  rc = af::workspace(ctx, af::msr_decode_scratch_floats(B, d, H) * sizeof(float), &ws, fn);
  if (rc) return rc;
  return af::msr_decode_step_impl(ctx, x, state, gamma, w_qkv, w_o, ret_norm_w, eps, B, d, H, out,
                                  static_cast<float *>(ws), af::stream_of(stream), fn);
}

extern "C" int af_msr_decode_step_f32_split(af_ctx *ctx, const float *x, float *state, const float *gamma,
                                            const float *w_qkv_hi, const float *w_qkv_lo, const float *w_o_hi,
                                            const float *w_o_lo, const float *ret_norm_w, float eps, int B, int d,
                                            int H, float *out, af_stream_t stream) {
  const char *fn = "af_msr_decode_step_f32_split";
  AF_ENTER(ctx, fn);
  int rc = af::check_msr_decode(fn, x, state, gamma, w_qkv_hi, w_o_hi, ret_norm_w, B, d, H, out);
  if (rc) return rc;
  AF_REQUIRE(w_qkv_lo && w_o_lo, "af_msr_decode_step_f32_split", "null weight pointer");
  const int dh = d / H;
  AF_REQUIRE((dh == 64 || dh == 128 || dh == 256) && d % 4 == 0 && af::aligned16(x) && af::aligned16(out) &&
                 af::aligned16(w_qkv_hi) && af::aligned16(w_qkv_lo) && af::aligned16(w_o_hi) && af::aligned16(w_o_lo),
             "af_msr_decode_step_f32_split", "head_dim must be 64, 128 or 256 and every pointer 16-byte aligned");
  if (B == 0) return AF_OK;
  void *ws = nullptr;
  rc = af::workspace(ctx, af::msr_decode_split_scratch_floats(B, d, H) * sizeof(float), &ws, fn);
  if (rc) return rc;
  return af::msr_decode_step_split_impl(ctx, x, state, gamma, w_qkv_hi, w_qkv_lo, w_o_hi, w_o_lo, ret_norm_w, eps, B,
                                        d, H, out, static_cast<float *>(ws), af::stream_of(stream), fn);
}

// ---------------------------------------------------------------------------
// Prefill on the bf16 tensor cores (chunkwise form):
//   1. qkv = x . W_qkv^T        bf16 GEMM -> bf16 [B*T][3d]
//   2. chunkwise retention      -> bf16 O * ret_norm_w, per-row partial sum O^2, final state
//   3. out = diag(1/rms) (O*w) . W_o^T   bf16 GEMM with the row scale in its epilogue

extern "C" int af_chunkwise_plan(int num_sms, int B, int T, int H, int nseg_req, int chunk, int *nseg,
                                 int *seg_len) {
  AF_REQUIRE(num_sms > 0 && B >= 0 && T >= 0 && H > 0 && nseg_req >= 0 && nseg && seg_len &&
                 (chunk == 0 || chunk == 64 || chunk == 128),
             "af_chunkwise_plan", "bad arguments");
  const af::ChunkPlan pl = af::chunkwise_plan(num_sms, B, T, H, nseg_req, chunk ? chunk : 64);
  *nseg = pl.nseg;
  *seg_len = pl.seg_len;
  return AF_OK;
}

namespace af {
// The chunk length of a call: 0 takes the context's default.
int resolve_chunk(const af_ctx *ctx, int chunk, int *out, const char *fn) {
  if (chunk != 0 && chunk != 64 && chunk != 128) return fail(AF_ERR_ARG, "%s: chunk must be 64 or 128 (or 0)", fn);
  *out = chunk ? chunk : chunkwise_default_chunk(ctx);
  return AF_OK;
}
}  // namespace af

extern "C" int af_retention_chunkwise_bf16(af_ctx *ctx, const uint16_t *qkv, int B, int T, int H, const float *gamma,
                                           const float *state_in, float *state_out, uint16_t *out,
                                           const float *norm_w, float *sumsq, int chunk, af_stream_t stream) {
  const char *fn = "af_retention_chunkwise_bf16";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(qkv && gamma && out, "af_retention_chunkwise_bf16", "null pointer");
  AF_REQUIRE(B >= 0 && T >= 0 && H > 0, "af_retention_chunkwise_bf16", "bad sizes B=%d T=%d H=%d", B, T, H);
  AF_REQUIRE(af::aligned16(qkv) && af::aligned16(out), "af_retention_chunkwise_bf16",
             "qkv and out must be 16-byte aligned");
  int C = 0;
  if (int rc = af::resolve_chunk(ctx, chunk, &C, fn)) return rc;
  if (B == 0 || T == 0) return AF_OK;
  const af::ChunkPlan pl = af::chunkwise_plan(ctx->num_sms, B, T, H, ctx->chunk_segments, C);
  void *ws = nullptr;
  const size_t seg_bytes = af::chunkwise_seg_state_bytes(B, H, pl);
  if (seg_bytes) {
    int rc = af::workspace(ctx, seg_bytes, &ws, fn);
    if (rc) return rc;
  }
  af::mark_begin(ctx, af::stream_of(stream));
  return af::retention_chunkwise_bf16(ctx, qkv, B, T, H, gamma, state_in, state_out, out, norm_w, sumsq, pl,
                                      static_cast<float *>(ws), af::stream_of(stream), fn);
}

extern "C" int af_msr_prefill_bf16(af_ctx *ctx, const uint16_t *x, const uint16_t *w_qkv, const uint16_t *w_o,
                                   const float *ret_norm_w, const float *gamma, float eps, int B, int T, int d, int H,
                                   const float *state_in, float *state_out, void *out, int out_bf16, int chunk,
                                   af_stream_t stream) {
  const char *fn = "af_msr_prefill_bf16";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(x && w_qkv && w_o && ret_norm_w && gamma && out, "af_msr_prefill_bf16", "null pointer");
  AF_REQUIRE(B >= 0 && T >= 0 && H > 0 && d == H * af::chunkwise_head_dim(), "af_msr_prefill_bf16",
             "the tensor-core prefill needs head_dim %d (d_model %d, heads %d)", af::chunkwise_head_dim(), d, H);
  AF_REQUIRE(af::aligned16(x) && af::aligned16(w_qkv) && af::aligned16(w_o), "af_msr_prefill_bf16",
             "x and weights must be 16-byte aligned");
  AF_REQUIRE((int64_t)B * T <= 65535LL * 128, "af_msr_prefill_bf16", "B*T too large");
  int C = 0;
  if (int rc = af::resolve_chunk(ctx, chunk, &C, fn)) return rc;
  if (B == 0 || T == 0) return AF_OK;
  const int64_t N = (int64_t)B * T;
  const int parts = H * af::chunkwise_parts(C);
  const size_t qkv_bytes = ((size_t)N * 3 * d * 2 + 255) & ~size_t(255);
  const size_t o_bytes = ((size_t)N * d * 2 + 255) & ~size_t(255);
  const size_t ss_bytes = ((size_t)N * parts * 4 + 255) & ~size_t(255);
  const af::ChunkPlan pl = af::chunkwise_plan(ctx->num_sms, B, T, H, ctx->chunk_segments, C);
  const size_t seg_bytes = af::chunkwise_seg_state_bytes(B, H, pl);
  void *ws = nullptr;
  int rc = af::workspace(ctx, qkv_bytes + o_bytes + ss_bytes + seg_bytes, &ws, fn);
  if (rc) return rc;
  uint8_t *base = static_cast<uint8_t *>(ws);
  void *qkv = base;
  void *o = base + qkv_bytes;
  float *ss = reinterpret_cast<float *>(base + qkv_bytes + o_bytes);
  float *seg = seg_bytes ? reinterpret_cast<float *>(base + qkv_bytes + o_bytes + ss_bytes) : nullptr;
  cudaStream_t st = af::stream_of(stream);
  af::mark_begin(ctx, st);
  af::GemmEpilogueArgs e1;
  e1.out = qkv;
  e1.ldo = 3 * d;
  e1.out_bf16 = 1;
  rc = af::tc_gemm(ctx, x, d, w_qkv, d, (int)N, 3 * d, d, false, e1, st, fn);
  if (rc) return rc;
  af::mark(ctx, "qkv", st);
  rc = af::retention_chunkwise_bf16(ctx, qkv, B, T, H, gamma, state_in, state_out, o, ret_norm_w, ss, pl, seg, st,
                                    fn);
  if (rc) return rc;
  af::GemmEpilogueArgs e2;
  e2.out = out;
  e2.ldo = d;
  e2.out_bf16 = out_bf16;
  e2.row_parts = ss;
  e2.nparts = parts;
  e2.inv_d = 1.0f / (float)d;
  e2.eps = eps;
  rc = af::tc_gemm(ctx, o, d, w_o, d, (int)N, d, d, false, e2, st, fn);
  af::mark(ctx, "w_o", st);
  return rc;
}

extern "C" int af_pack_qkv_heads(af_ctx *ctx, const void *src, void *dst, int d, int H, int elem_bytes,
                                 af_stream_t stream) {
  const char *fn = "af_pack_qkv_heads";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(src && dst && src != dst, "af_pack_qkv_heads", "src and dst must be distinct buffers");
  AF_REQUIRE(H > 0 && d % H == 0 && (elem_bytes == 2 || elem_bytes == 4) && ((int64_t)d * elem_bytes) % 16 == 0 &&
                 af::aligned16(src) && af::aligned16(dst),
             "af_pack_qkv_heads", "d %% H == 0, rows of 16-byte multiples, aligned buffers");
  return af::pack_qkv_heads(ctx, src, dst, d, H, elem_bytes, af::stream_of(stream), fn);
}
