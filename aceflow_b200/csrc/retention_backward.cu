// Backward of the chunkwise retention core (training).
//
// The forward (aceflow/nn/retention.py:51-61, per head, decay gamma):
//     o_t = sum_{s <= t} gamma^(t-s) (q_t . k_s) v_s  (+ gamma^(t+1) q_t S_0)
// Its gradients for an upstream dO are retention forms themselves:
//     dq_t = sum_{s <= t} gamma^(t-s) (do_t . v_s) k_s  (+ gamma^(t+1) do_t S_0^T)
//          = Retention(q' = dO, k' = V, v' = K) with initial state S_0^T
//     dk_s = sum_{t >= s} gamma^(t-s) (v_s . do_t) q_t
//          = the same form over reversed time: Retention(V, dO, Q) on t' = T-1-t
//     dv_s = sum_{t >= s} gamma^(t-s) (k_s . q_t) do_t
//          = Retention(K, Q, dO) over reversed time
//     dS_0 = sum_t gamma^(t+1) q_t^T do_t = gamma * (the final state of the
//            dV pass, whose keys are q and values do)
// so the backward runs the tensor-core chunkwise forward kernel (128-token
// chunks, the state in TMEM) three times, each pass reading its q', k', v'
// through separate tensor maps: the dQ pass straight from dO and qkv, the two
// reversed passes from one time-reversed copy of qkv and dO, writing their
// rows back in forward order through the kernel's reversed output rows.  The reference
// has no backward (its trainers are PyTorch-only); the float64 oracle's closed
// form gradients of the parallel form pin this one.
#include "common.cuh"

namespace {

constexpr int DH = 256;

inline size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

// dst row b*T + t = src row b*T + T-1-t, rows of `w` 16-byte units
// (src rows `lds` units apart, dst rows `w` apart).
__global__ void reverse_rows_kernel(uint4 *__restrict__ dst, const uint4 *__restrict__ src, int64_t lds, int B, int T,
                                    int w) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)B * T * w) return;
  const int u = (int)(idx % w);
  const int64_t r = idx / w;
  const int64_t b = r / T, t = r % T;
  dst[idx] = src[(b * T + (T - 1 - t)) * lds + u];
}

// dst[bh][v][k] = src[bh][k][v] (fp32 [DH][DH] blocks), 32 x 32 tiles.
__global__ void transpose_states_kernel(const float *__restrict__ src, float *__restrict__ dst) {
  __shared__ float tile[32][33];
  const size_t base = (size_t)blockIdx.z * DH * DH;
  const int x = blockIdx.x * 32 + threadIdx.x, y0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) tile[i][threadIdx.x] = src[base + (size_t)(y0 + i) * DH + x];
  __syncthreads();
  const int xo = blockIdx.y * 32 + threadIdx.x, yo0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) dst[base + (size_t)(yo0 + i) * DH + xo] = tile[threadIdx.x][i];
}

// s[b][h][..] *= gamma[h] (fp32 [B][H][DH*DH]).
__global__ void scale_states_kernel(float4 *__restrict__ s, const float *__restrict__ gamma, int H, int64_t n4) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n4) return;
  const float g = gamma[(idx / (DH * DH / 4)) % H];
  float4 v = s[idx];
  s[idx] = make_float4(v.x * g, v.y * g, v.z * g, v.w * g);
}

}  // namespace

extern "C" int af_retention_chunkwise_backward_bf16(af_ctx *ctx, const uint16_t *qkv, const uint16_t *dout, int B,
                                                    int T, int H, const float *gamma, const float *state_in,
                                                    uint16_t *dqkv, float *dstate_in, af_stream_t stream) {
  const char *fn = "af_retention_chunkwise_backward_bf16";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(qkv && dout && gamma && dqkv, "af_retention_chunkwise_backward_bf16", "null pointer");
  AF_REQUIRE(B >= 0 && T >= 0 && H > 0, "af_retention_chunkwise_backward_bf16", "bad sizes B=%d T=%d H=%d", B, T, H);
  AF_REQUIRE(af::aligned16(qkv) && af::aligned16(dout) && af::aligned16(dqkv) && af::aligned16(state_in) &&
                 af::aligned16(dstate_in),
             "af_retention_chunkwise_backward_bf16", "every buffer must be 16-byte aligned");
  AF_REQUIRE((int64_t)B * T <= 65535LL * 128, "af_retention_chunkwise_backward_bf16", "B*T too large");
  if (B == 0 || T == 0) {
    if (dstate_in && B > 0)
      AF_CUDA(cudaMemsetAsync(dstate_in, 0, (size_t)B * H * DH * DH * 4, af::stream_of(stream)), fn);
    return AF_OK;
  }
  const int d = H * DH;
  const int64_t N = (int64_t)B * T;
  const af::ChunkPlan pl = af::chunkwise_plan(ctx->num_sms, B, T, H, ctx->chunk_segments, 128);
  const size_t rq_b = align256((size_t)N * 3 * d * 2), rd_b = align256((size_t)N * d * 2),
               st_b = state_in ? align256((size_t)B * H * DH * DH * 4) : 0,
               seg_b = align256(af::chunkwise_seg_state_bytes(B, H, pl));
  void *ws = nullptr;
  int rc = af::workspace(ctx, rq_b + rd_b + st_b + seg_b, &ws, fn);
  if (rc) return rc;
  uint8_t *base = static_cast<uint8_t *>(ws);
  uint16_t *rqkv = reinterpret_cast<uint16_t *>(base);         // qkv, each stream's rows in reverse
  uint16_t *rdout = reinterpret_cast<uint16_t *>(base + rq_b);  // dout likewise
  float *s0t = state_in ? reinterpret_cast<float *>(base + rq_b + rd_b) : nullptr;
  float *seg = seg_b ? reinterpret_cast<float *>(base + rq_b + rd_b + st_b) : nullptr;
  cudaStream_t st = af::stream_of(stream);
  const uint16_t *K = qkv + d, *V = qkv + 2 * d;
  const int64_t ld = 3 * (int64_t)d;
  af::mark_begin(ctx, st);
  // dQ = Retention(dO, V, K) from S_0^T, written to dqkv[:, 0:d]
  if (state_in) {
    transpose_states_kernel<<<dim3(DH / 32, DH / 32, B * H), dim3(32, 8), 0, st>>>(state_in, s0t);
    if ((rc = af::launched(ctx, fn))) return rc;
  }
  rc = af::retention_chunkwise_bf16(ctx, af::ChunkSrc{dout, V, K, d, ld, ld}, B, T, H, gamma, s0t, nullptr, dqkv,
                                    nullptr, nullptr, pl, seg, st, fn, ld, false);
  if (rc) return rc;
  af::mark(ctx, "dq", st);
  // the time-reversed operands of the other two passes
  for (int part = 0; part < 2; ++part) {
    const int w = (part == 0 ? 3 * d : d) / 8;
    const int64_t n = N * w;
    reverse_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
        reinterpret_cast<uint4 *>(part == 0 ? rqkv : rdout), reinterpret_cast<const uint4 *>(part == 0 ? qkv : dout),
        w, B, T, w);
    if ((rc = af::launched(ctx, fn))) return rc;
  }
  const uint16_t *rQ = rqkv, *rK = rqkv + d, *rV = rqkv + 2 * d;
  // dK = reversed Retention(V, dO, Q), rows written back in forward order to dqkv[:, d:2d]
  rc = af::retention_chunkwise_bf16(ctx, af::ChunkSrc{rV, rdout, rQ, ld, d, ld}, B, T, H, gamma, nullptr, nullptr,
                                    dqkv + d, nullptr, nullptr, pl, seg, st, fn, ld, true);
  if (rc) return rc;
  af::mark(ctx, "dk", st);
  // dV = reversed Retention(K, Q, dO) to dqkv[:, 2d:3d]; its final state * gamma = dS_0
  rc = af::retention_chunkwise_bf16(ctx, af::ChunkSrc{rK, rQ, rdout, ld, ld, d}, B, T, H, gamma, nullptr, dstate_in,
                                    dqkv + 2 * d, nullptr, nullptr, pl, seg, st, fn, ld, true);
  if (rc) return rc;
  if (dstate_in) {
    const int64_t n4 = (int64_t)B * H * DH * DH / 4;
    scale_states_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(reinterpret_cast<float4 *>(dstate_in), gamma,
                                                                       H, n4);
    if ((rc = af::launched(ctx, fn))) return rc;
  }
  af::mark(ctx, "dv", st);
  return AF_OK;
}
