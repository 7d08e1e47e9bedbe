// Fused MultiScaleRetention layer entry points.
//
// Decode step (one token per stream, fp32, state in HBM):
//   1. qkv = x . W_qkv^T                        (projection GEMM)
//   2. retention step per (b, h), writing o * ret_norm_w and per-head sum o^2
//   3. out = diag(1/rms) (o * w) . W_o^T         (GEMM, norm applied per row)
// This is AceEngine.forward_layer_internal's retention half
// (aceflow-core/src/cpu/mod.rs:651-678) for a batch of streams, with the
// Python module's RMSNorm placement (aceflow/nn/retention.py:64-65).
#include "common.cuh"

namespace af {
int launch_retention_step(af_ctx *ctx, float *state, int64_t state_bs, const float *gamma, const float *q,
                          const float *k, const float *v, int64_t qs, float *out, int64_t out_rs, int batch, int H,
                          int dh, const float *norm_w, float *sumsq, cudaStream_t st, const char *fn);
int launch_sgemm_nt(af_ctx *ctx, const float *x, const float *w, const float *bias, float *y, int M, int N, int K,
                    const float *parts, int nparts, float inv_d, float eps, cudaStream_t st, const char *fn);

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
  int rc = launch_sgemm_nt(ctx, x, w_qkv, nullptr, qkv, B, 3 * d, d, nullptr, 0, 0.f, 0.f, st, fn);
  if (rc) return rc;
  rc = launch_retention_step(ctx, state, (int64_t)H * dh * dh, gamma, qkv, qkv + d, qkv + 2 * d, 3 * (int64_t)d, o,
                             d, B, H, dh, ret_norm_w, sumsq, st, fn);
  if (rc) return rc;
  return launch_sgemm_nt(ctx, o, w_o, nullptr, out, B, d, d, sumsq, H, 1.0f / (float)d, eps, st, fn);
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
