// Recurrent retention step on B200: the HBM-bound fp32 state stream.
//
// Semantics (aceflow-core/src/cpu/recurrence.rs:18-41): for each stream b,
// head h and state row i (the k index),
//     S[i,:] = gamma_h * S[i,:] + k_i * v        (outer-product update)
//     o     += q_i * S[i,:]                       (with the UPDATED row)
//
// Design: one CTA owns one (b, h) state of head_dim^2 fp32 values, streamed
// once from HBM and written back once.  Threads map to float4 column groups
// (16-byte coalesced loads, `ld.global.cs`/`st.global.cs` streaming hints
// since each byte is touched exactly once per step) and to interleaved row
// groups; each thread keeps UNROLL rows of loads in flight.  k and q of the
// head sit in shared memory, v's four columns in registers.  The per-thread
// partial outputs are reduced over row groups through shared memory.
//
// Fusions for the decode layer: the CTA can multiply o by the RMSNorm weight
// on the way out and write the head's sum of o^2, so the following W_o GEMM
// applies 1/rms per row in its epilogue; no separate norm pass touches o.
#include "common.cuh"

namespace {

struct HeadGroup {
  int h0, n;                // first head and number of heads in this launch
  int64_t qkv_head_stride;  // floats between consecutive heads' q (and k, v)
  int nsplit;               // q/k/v are the sum of nsplit partial buffers (split-K GEMM output)
  int64_t split_stride;     // floats between the partial buffers
};

template <int DH, int THREADS>
struct StepShape {
  static constexpr int NCG = DH / 4;            // float4 column groups per row
  static constexpr int RG = THREADS / NCG;      // row groups
  static constexpr int ROWS = DH / RG;          // rows per thread
  static constexpr int UNROLL = ROWS < 8 ? ROWS : 8;
  static_assert(DH % 4 == 0 && THREADS % NCG == 0 && DH % RG == 0 && ROWS % UNROLL == 0, "shape");
};

// One token of one (b, h).  sk/sq hold k and q of the head (DH floats each).
// Returns this thread's partial output for columns 4*cg .. 4*cg+3.
template <int DH, int THREADS>
__device__ __forceinline__ float4 step_rows(float *__restrict__ S, float g, const float *sk,
                                            const float *sq, float4 vv, int cg, int rg) {
  using Sh = StepShape<DH, THREADS>;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 *base = reinterpret_cast<float4 *>(S) + cg;
#pragma unroll 1
  for (int r0 = 0; r0 < Sh::ROWS; r0 += Sh::UNROLL) {
    float4 s[Sh::UNROLL];
#pragma unroll
    for (int u = 0; u < Sh::UNROLL; ++u) {
      const int i = rg + (r0 + u) * Sh::RG;
      s[u] = ld_stream(base + (size_t)i * Sh::NCG);
    }
#pragma unroll
    for (int u = 0; u < Sh::UNROLL; ++u) {
      const int i = rg + (r0 + u) * Sh::RG;
      const float kk = sk[i], qq = sq[i];
      float4 t = s[u];
      t.x = fmaf(g, t.x, kk * vv.x);
      t.y = fmaf(g, t.y, kk * vv.y);
      t.z = fmaf(g, t.z, kk * vv.z);
      t.w = fmaf(g, t.w, kk * vv.w);
      st_stream(base + (size_t)i * Sh::NCG, t);
      acc.x = fmaf(qq, t.x, acc.x);
      acc.y = fmaf(qq, t.y, acc.y);
      acc.z = fmaf(qq, t.z, acc.z);
      acc.w = fmaf(qq, t.w, acc.w);
    }
  }
  return acc;
}

// Reduces the per-row-group partials, writes o (optionally * norm_w) and
// optionally the head's sum of o^2.  `red` holds RG*DH floats.
template <int DH, int THREADS>
__device__ __forceinline__ void finish_head(float4 acc, float4 *red, float *__restrict__ o_out,
                                            const float *__restrict__ norm_w_head,
                                            float *__restrict__ sumsq_out, int cg, int rg, bool out_bf16 = false,
                                            float *__restrict__ o_lo = nullptr) {
  using Sh = StepShape<DH, THREADS>;
  red[rg * Sh::NCG + cg] = acc;
  __syncthreads();
  __shared__ float warp_part[THREADS / 32];
  float ss = 0.f;
  if (threadIdx.x < Sh::NCG) {
    float4 o = red[threadIdx.x];
#pragma unroll 4
    for (int r = 1; r < Sh::RG; ++r) {
      const float4 p = red[r * Sh::NCG + threadIdx.x];
      o.x += p.x;
      o.y += p.y;
      o.z += p.z;
      o.w += p.w;
    }
    ss = o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
    if (norm_w_head) {
      const float4 w = reinterpret_cast<const float4 *>(norm_w_head)[threadIdx.x];
      o.x *= w.x;
      o.y *= w.y;
      o.z *= w.z;
      o.w *= w.w;
    }
    if (o_lo) {  // exact tf32 part + remainder, the operands of the split GEMM
      const float4 h = make_float4(__uint_as_float(__float_as_uint(o.x) & 0xFFFFE000u),
                                   __uint_as_float(__float_as_uint(o.y) & 0xFFFFE000u),
                                   __uint_as_float(__float_as_uint(o.z) & 0xFFFFE000u),
                                   __uint_as_float(__float_as_uint(o.w) & 0xFFFFE000u));
      reinterpret_cast<float4 *>(o_out)[threadIdx.x] = h;
      reinterpret_cast<float4 *>(o_lo)[threadIdx.x] = make_float4(o.x - h.x, o.y - h.y, o.z - h.z, o.w - h.w);
    } else if (out_bf16) {
      __nv_bfloat162 lo = __floats2bfloat162_rn(o.x, o.y), hi = __floats2bfloat162_rn(o.z, o.w);
      reinterpret_cast<uint2 *>(o_out)[threadIdx.x] =
          make_uint2(*reinterpret_cast<uint32_t *>(&lo), *reinterpret_cast<uint32_t *>(&hi));
    } else {
      reinterpret_cast<float4 *>(o_out)[threadIdx.x] = o;
    }
  }
  if (sumsq_out) {
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) warp_part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      constexpr int nw = (Sh::NCG + 31) / 32;
#pragma unroll
      for (int w = 0; w < nw; ++w) t += warp_part[w];
      *sumsq_out = t;
    }
  }
}

template <int DH, int THREADS>
__global__ void __launch_bounds__(THREADS)
    retention_step_kernel(float *__restrict__ state, int64_t state_bs, const float *__restrict__ gamma,
                          const float *__restrict__ q, const float *__restrict__ k,
                          const float *__restrict__ v, int64_t qs, float *__restrict__ out,
                          int64_t out_rs, int H, const float *__restrict__ norm_w,
                          float *__restrict__ sumsq, int out_bf16, float *__restrict__ out_lo, HeadGroup hg) {
  // This launch covers heads [hg.h0, hg.h0 + hg.n) of H; q/k/v of head
  // h0 + j sit j * hg.qkv_head_stride floats after the row's q/k/v pointers.
  using Sh = StepShape<DH, THREADS>;
  __shared__ float sk[DH], sq[DH];
  __shared__ float4 red[Sh::RG * Sh::NCG];
  const int b = blockIdx.x / hg.n, hl = blockIdx.x % hg.n, h = hg.h0 + hl;
  const int cg = threadIdx.x % Sh::NCG, rg = threadIdx.x / Sh::NCG;
  const float *qh = q + (size_t)b * qs + (size_t)hl * hg.qkv_head_stride;
  const float *kh = k + (size_t)b * qs + (size_t)hl * hg.qkv_head_stride;
  const float *vh = v + (size_t)b * qs + (size_t)hl * hg.qkv_head_stride;
  griddep_launch();
  griddep_wait();  // q, k, v come from the kernel before (programmatic launch)
  for (int i = threadIdx.x; i < DH; i += THREADS) {
    float kk = kh[i], qq = qh[i];
    for (int z = 1; z < hg.nsplit; ++z) {
      kk += kh[(size_t)z * hg.split_stride + i];
      qq += qh[(size_t)z * hg.split_stride + i];
    }
    sk[i] = kk;
    sq[i] = qq;
  }
  float4 vv = make_float4(vh[4 * cg], vh[4 * cg + 1], vh[4 * cg + 2], vh[4 * cg + 3]);
  for (int z = 1; z < hg.nsplit; ++z) {
    const float *vz = vh + (size_t)z * hg.split_stride + 4 * cg;
    vv.x += vz[0];
    vv.y += vz[1];
    vv.z += vz[2];
    vv.w += vz[3];
  }
  const float g = gamma[h];
  __syncthreads();
  float *S = state + (size_t)b * state_bs + (size_t)h * DH * DH;
  const float4 acc = step_rows<DH, THREADS>(S, g, sk, sq, vv, cg, rg);
  float *o_out = out_bf16 ? reinterpret_cast<float *>(reinterpret_cast<__nv_bfloat16 *>(out) + (size_t)b * out_rs +
                                                   (size_t)h * DH)
                         : out + (size_t)b * out_rs + (size_t)h * DH;
  finish_head<DH, THREADS>(acc, red, o_out, norm_w ? norm_w + (size_t)h * DH : nullptr,
                           sumsq ? sumsq + (size_t)b * H + h : nullptr, cg, rg, out_bf16 != 0,
                           out_lo ? out_lo + (size_t)b * out_rs + (size_t)h * DH : nullptr);
}

// Token-serial scan: the same per-token work, T tokens in order.
template <int DH, int THREADS>
__global__ void __launch_bounds__(THREADS)
    retention_scan_kernel(float *__restrict__ state, int64_t state_bs, const float *__restrict__ gamma,
                          const float *__restrict__ q, const float *__restrict__ k,
                          const float *__restrict__ v, int64_t qs, float *__restrict__ out, int T,
                          int H) {
  using Sh = StepShape<DH, THREADS>;
  __shared__ float sk[DH], sq[DH];
  __shared__ float4 red[Sh::RG * Sh::NCG];
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  const int cg = threadIdx.x % Sh::NCG, rg = threadIdx.x / Sh::NCG;
  const float g = gamma[h];
  float *S = state + (size_t)b * state_bs + (size_t)h * DH * DH;
  const int d = H * DH;
  for (int t = 0; t < T; ++t) {
    const size_t row = (size_t)b * T + t;
    const float *qh = q + row * qs + (size_t)h * DH;
    const float *kh = k + row * qs + (size_t)h * DH;
    const float *vh = v + row * qs + (size_t)h * DH;
    __syncthreads();  // previous token's readers of sk/sq/red are done
    for (int i = threadIdx.x; i < DH; i += THREADS) {
      sk[i] = kh[i];
      sq[i] = qh[i];
    }
    const float4 vv = make_float4(vh[4 * cg], vh[4 * cg + 1], vh[4 * cg + 2], vh[4 * cg + 3]);
    __syncthreads();
    const float4 acc = step_rows<DH, THREADS>(S, g, sk, sq, vv, cg, rg);
    finish_head<DH, THREADS>(acc, red, out + row * d + (size_t)h * DH, nullptr, nullptr, cg, rg);
  }
}

// Generic head_dim (multiple of 4, <= 1024): runtime loop bounds.
__global__ void __launch_bounds__(256)
    retention_step_generic(float *__restrict__ state, int64_t state_bs, const float *__restrict__ gamma,
                           const float *__restrict__ q, const float *__restrict__ k,
                           const float *__restrict__ v, int64_t qs, float *__restrict__ out,
                           int64_t out_rs, int T, int H, int dh, int rgs, const float *__restrict__ norm_w,
                           float *__restrict__ sumsq) {
  // rgs (row groups) comes from the host, which sized `red` for rgs * ncg
  // entries; blockDim.x may exceed rgs * ncg (rounded up to whole warps).
  extern __shared__ float smem[];
  float *sk = smem, *sq = smem + dh;
  float4 *red = reinterpret_cast<float4 *>(smem + 2 * dh);
  __shared__ float warp_part[8];
  const int ncg = dh / 4;
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  const int cg = threadIdx.x % ncg, rg = threadIdx.x / ncg;
  const bool active = rg < rgs;
  const float g = gamma[h];
  float *S = state + (size_t)b * state_bs + (size_t)h * dh * dh;
  for (int t = 0; t < T; ++t) {
    const size_t row = (size_t)b * T + t;
    const float *qh = q + row * qs + (size_t)h * dh;
    const float *kh = k + row * qs + (size_t)h * dh;
    const float *vh = v + row * qs + (size_t)h * dh;
    __syncthreads();
    for (int i = threadIdx.x; i < dh; i += blockDim.x) {
      sk[i] = kh[i];
      sq[i] = qh[i];
    }
    __syncthreads();
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (active) {
      const float4 vv = make_float4(vh[4 * cg], vh[4 * cg + 1], vh[4 * cg + 2], vh[4 * cg + 3]);
      float4 *base = reinterpret_cast<float4 *>(S) + cg;
      for (int i = rg; i < dh; i += rgs) {
        float4 s = ld_stream(base + (size_t)i * ncg);
        const float kk = sk[i], qq = sq[i];
        s.x = fmaf(g, s.x, kk * vv.x);
        s.y = fmaf(g, s.y, kk * vv.y);
        s.z = fmaf(g, s.z, kk * vv.z);
        s.w = fmaf(g, s.w, kk * vv.w);
        st_stream(base + (size_t)i * ncg, s);
        acc.x = fmaf(qq, s.x, acc.x);
        acc.y = fmaf(qq, s.y, acc.y);
        acc.z = fmaf(qq, s.z, acc.z);
        acc.w = fmaf(qq, s.w, acc.w);
      }
      red[rg * ncg + cg] = acc;
    }
    __syncthreads();
    float ss = 0.f;
    float *o_out = out + (T == 1 ? (size_t)b * out_rs : row * out_rs) + (size_t)h * dh;
    for (int c = threadIdx.x; c < ncg; c += blockDim.x) {
      float4 o = red[c];
      for (int r = 1; r < rgs; ++r) {
        const float4 p = red[r * ncg + c];
        o.x += p.x;
        o.y += p.y;
        o.z += p.z;
        o.w += p.w;
      }
      ss += o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
      if (norm_w) {
        const float *w = norm_w + (size_t)h * dh + 4 * c;
        o.x *= w[0];
        o.y *= w[1];
        o.z *= w[2];
        o.w *= w[3];
      }
      o_out[4 * c] = o.x;
      o_out[4 * c + 1] = o.y;
      o_out[4 * c + 2] = o.z;
      o_out[4 * c + 3] = o.w;
    }
    if (sumsq) {
      ss = warp_sum(ss);
      if ((threadIdx.x & 31) == 0) warp_part[threadIdx.x >> 5] = ss;
      __syncthreads();
      if (threadIdx.x == 0) {
        float tsum = 0.f;
        for (int w = 0; w < (int)(blockDim.x + 31) / 32; ++w) tsum += warp_part[w];
        sumsq[blockIdx.x] = tsum;
      }
    }
  }
}

// Any head_dim (the reference accepts every size): one thread per state
// column, rows in order, so each column's output accumulates like
// recurrence.rs:28-39.  Used when head_dim is not a multiple of 4.
__global__ void __launch_bounds__(256)
    retention_step_scalar(float *__restrict__ state, int64_t state_bs, const float *__restrict__ gamma,
                          const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                          int64_t qs, float *__restrict__ out, int64_t out_rs, int T, int H, int dh) {
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  const float g = gamma[h];
  float *S = state + (size_t)b * state_bs + (size_t)h * dh * dh;
  for (int t = 0; t < T; ++t) {
    const size_t row = (size_t)b * T + t;
    const float *qh = q + row * qs + (size_t)h * dh;
    const float *kh = k + row * qs + (size_t)h * dh;
    const float *vh = v + row * qs + (size_t)h * dh;
    float *o_out = out + (T == 1 ? (size_t)b * out_rs : row * out_rs) + (size_t)h * dh;
    for (int j = threadIdx.x; j < dh; j += blockDim.x) {
      const float vj = vh[j];
      float o = 0.f;
      for (int i = 0; i < dh; ++i) {
        const float s = fmaf(g, S[(size_t)i * dh + j], kh[i] * vj);
        S[(size_t)i * dh + j] = s;
        o = fmaf(qh[i], s, o);
      }
      o_out[j] = o;
    }
  }
}

int check_common(const char *fn, float *state, const float *gamma, const float *q, const float *k,
                 const float *v, float *out, int batch, int H, int dh, int64_t state_bs,
                 int64_t qs) {
  if (!state || !gamma || !q || !k || !v || !out) return af::fail(AF_ERR_ARG, "%s: null pointer", fn);
  if (batch < 0 || H <= 0 || dh <= 0) return af::fail(AF_ERR_ARG, "%s: bad sizes batch=%d heads=%d head_dim=%d", fn, batch, H, dh);
  if (state_bs < (int64_t)H * dh * dh)
    return af::fail(AF_ERR_ARG, "%s: state_batch_stride %lld must be >= H*dh*dh", fn, (long long)state_bs);
  if (qs < 1) return af::fail(AF_ERR_ARG, "%s: qkv_row_stride must be positive", fn);
  return AF_OK;
}

}  // namespace

namespace af {

// Launches one decode step; shared by af_retention_step and the fused layer.
int launch_retention_step(af_ctx *ctx, float *state, int64_t state_bs, const float *gamma, const float *q,
                          const float *k, const float *v, int64_t qs, float *out, int64_t out_rs,
                          int batch, int H, int dh, const float *norm_w, float *sumsq, cudaStream_t st,
                          const char *fn, int out_bf16, float *out_lo, int h0, int hn, int64_t qkv_hs, int nsplit,
                          int64_t split_stride, bool pdl) {
  if (batch == 0) return AF_OK;
  if (nsplit < 1) nsplit = 1;
  if (hn <= 0) {  // all heads, q/k/v head-contiguous
    h0 = 0;
    hn = H;
    qkv_hs = dh;
  }
  const HeadGroup hgp{h0, hn, qkv_hs, nsplit, split_stride};
  const bool all_heads = h0 == 0 && hn == H && qkv_hs == dh;
  const dim3 grid((unsigned)(batch * hn));
  if (out_bf16 && !(dh == 256 || dh == 128 || dh == 64) )
    return fail(AF_ERR_ARG, "%s: bf16 output needs head_dim 64, 128 or 256", fn);
  if (dh % 4 != 0 || dh > 1024 || state_bs % 4 != 0 || !aligned16(state)) {
    if (norm_w || sumsq || !all_heads || nsplit > 1) return fail(AF_ERR_ARG, "%s: fused norm needs head_dim %% 4 == 0 and <= 1024", fn);
    retention_step_scalar<<<grid, 256, 0, st>>>(state, state_bs, gamma, q, k, v, qs, out, out_rs, 1, H, dh);
    return launched(ctx, fn);
  }
  bool fast = (out_rs % 4 == 0) && aligned16(out) && (norm_w == nullptr || aligned16(norm_w));
  if ((out_bf16 || out_lo) && !fast) return fail(AF_ERR_ARG, "%s: bf16/split output needs an aligned output", fn);
  if (out_lo && (!aligned16(out_lo) || !(dh == 256 || dh == 128 || dh == 64)))
    return fail(AF_ERR_ARG, "%s: split output needs head_dim 64, 128 or 256 and an aligned buffer", fn);
  if (fast && dh == 256) {
    const cudaError_t e = launch_kernel(retention_step_kernel<256, 256>, grid, dim3(256), 0, st, pdl && ctx->pdl, state,
                                        state_bs, gamma, q, k, v, qs, out, out_rs, H, norm_w, sumsq, out_bf16, out_lo,
                                        hgp);
    if (e != cudaSuccess) return fail(AF_ERR_CUDA, "%s: launch: %s", fn, cudaGetErrorString(e));
  } else if (fast && dh == 128) {
    retention_step_kernel<128, 256><<<grid, 256, 0, st>>>(state, state_bs, gamma, q, k, v, qs, out, out_rs, H,
                                                          norm_w, sumsq, out_bf16, out_lo, hgp);
  } else if (fast && dh == 64) {
    retention_step_kernel<64, 256><<<grid, 256, 0, st>>>(state, state_bs, gamma, q, k, v, qs, out, out_rs, H,
                                                         norm_w, sumsq, out_bf16, out_lo, hgp);
  } else if (fast && dh == 32) {
    retention_step_kernel<32, 256><<<grid, 256, 0, st>>>(state, state_bs, gamma, q, k, v, qs, out, out_rs, H,
                                                         norm_w, sumsq, out_bf16, out_lo, hgp);
  } else if (fast && dh == 16) {
    retention_step_kernel<16, 64><<<grid, 64, 0, st>>>(state, state_bs, gamma, q, k, v, qs, out, out_rs, H,
                                                       norm_w, sumsq, out_bf16, out_lo, hgp);
  } else {
    if (!all_heads || nsplit > 1)
      return fail(AF_ERR_ARG, "%s: head groups and partial sums need head_dim 16..256 (power of two)", fn);
    const int ncg = dh / 4;
    int rgs = 256 / ncg;
    if (rgs < 1) rgs = 1;
    if (rgs > dh) rgs = dh;
    const int threads = ((ncg * rgs + 31) / 32) * 32;
    const size_t smem = (size_t)2 * dh * sizeof(float) + (size_t)rgs * ncg * sizeof(float4);
    retention_step_generic<<<grid, threads, smem, st>>>(state, state_bs, gamma, q, k, v, qs, out, out_rs, 1, H,
                                                        dh, rgs, norm_w, sumsq);
  }
  return launched(ctx, fn);
}

}  // namespace af

extern "C" int af_retention_step(af_ctx *ctx, float *state, int64_t state_bs, const float *gamma, const float *q,
                                 const float *k, const float *v, int64_t qs, float *out, int batch, int H, int dh,
                                 af_stream_t stream) {
  const char *fn = "af_retention_step";
  AF_ENTER(ctx, fn);
  int rc = check_common(fn, state, gamma, q, k, v, out, batch, H, dh, state_bs, qs);
  if (rc) return rc;
  return af::launch_retention_step(ctx, state, state_bs, gamma, q, k, v, qs, out, (int64_t)H * dh, batch, H, dh,
                                   nullptr, nullptr, af::stream_of(stream), fn, 0, nullptr, 0, 0, 0);
}

extern "C" int af_retention_scan(af_ctx *ctx, float *state, int64_t state_bs, const float *gamma, const float *q,
                                 const float *k, const float *v, int64_t qs, float *out, int batch, int T, int H,
                                 int dh, af_stream_t stream) {
  const char *fn = "af_retention_scan";
  AF_ENTER(ctx, fn);
  int rc = check_common(fn, state, gamma, q, k, v, out, batch, H, dh, state_bs, qs);
  if (rc) return rc;
  if (T < 0) return af::fail(AF_ERR_ARG, "%s: T must be >= 0", fn);
  if (batch == 0 || T == 0) return AF_OK;
  cudaStream_t st = af::stream_of(stream);
  const dim3 grid((unsigned)(batch * H));
  if (dh % 4 != 0 || dh > 1024 || state_bs % 4 != 0 || !af::aligned16(state)) {
    retention_step_scalar<<<grid, 256, 0, st>>>(state, state_bs, gamma, q, k, v, qs, out, (int64_t)H * dh, T, H, dh);
    return af::launched(ctx, fn);
  }
  const bool fast = af::aligned16(out) && ((int64_t)H * dh) % 4 == 0;
  if (fast && dh == 256) {
    retention_scan_kernel<256, 256><<<grid, 256, 0, st>>>(state, state_bs, gamma, q, k, v, qs, out, T, H);
  } else if (fast && dh == 128) {
    retention_scan_kernel<128, 256><<<grid, 256, 0, st>>>(state, state_bs, gamma, q, k, v, qs, out, T, H);
  } else if (fast && dh == 64) {
    retention_scan_kernel<64, 256><<<grid, 256, 0, st>>>(state, state_bs, gamma, q, k, v, qs, out, T, H);
  } else {
    const int ncg = dh / 4;
    int rgs = 256 / ncg;
    if (rgs < 1) rgs = 1;
    if (rgs > dh) rgs = dh;
    const int threads = ((ncg * rgs + 31) / 32) * 32;
    const size_t smem = (size_t)2 * dh * sizeof(float) + (size_t)rgs * ncg * sizeof(float4);
    retention_step_generic<<<grid, threads, smem, st>>>(state, state_bs, gamma, q, k, v, qs, out, (int64_t)H * dh,
                                                        T, H, dh, rgs, nullptr, nullptr);
  }
  return af::launched(ctx, fn);
}
