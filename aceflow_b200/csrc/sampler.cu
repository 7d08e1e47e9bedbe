// Next-token sampling from logits rows: the reference's
// sample_token_from_logits (aceflow-core/src/cpu/sampler.rs:104-180) with its
// repetition penalty (sampler.rs:83-102), one CTA per row.
//
// The reference sorts all candidates by scaled logit, normalises a softmax
// over them, cuts the sorted list where the running sum of probabilities
// first exceeds top_p, and walks it again until the running sum reaches
// u * (kept mass).  Here no list is sorted: every "position in the sorted
// list" question is answered by bisection over an order-preserving 32-bit key
// of the scaled logit, each step a block-wide count or sum over the row held
// in shared memory:
//   top-k threshold   largest key T with  #{key >= T}          >= k
//   top-p cutoff      largest key T with  sum{p : key >= T}    >  top_p
//   sampled token     largest key T with  sum{p : key >= T}    >= u * kept
// Items with equal keys keep the lowest index first (the reference's order
// among equal logits is unspecified: it uses unstable sorts).  The uniform
// variate u comes from the caller (the reference draws it from a per-thread
// generator seeded by the clock, sampler.rs:8-35), so results are
// reproducible.  Sums are fp32 block reductions, not the reference's
// sequential sums: a draw that lands within rounding of a boundary between
// two tokens may pick the neighbour.
#include "common.cuh"

namespace {

constexpr int kThreads = 1024;

__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ bool has(const uint32_t *bm, int i) { return (bm[i >> 5] >> (i & 31)) & 1u; }

// Block-wide sum (every thread gets the total); `red` holds 32 partials.
__device__ float block_sum(float v, float *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
  return t;
}
__device__ unsigned block_count(unsigned v, unsigned *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned t = 0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
  return t;
}

struct SampleParams {
  const float *logits;
  int V;
  const int32_t *ctx_tokens;  // row r: ctx_tokens[r * ctx_stride + 0 .. ctx_len)
  int64_t ctx_stride;
  int ctx_len;
  float temperature, top_p, rep;
  int top_k;
  const float *uniforms;  // [rows]; unused when greedy
  int32_t *out;
};

__global__ void __launch_bounds__(kThreads) sample_rows_kernel(SampleParams p) {
  extern __shared__ float xs[];  // the row's logits, then scaled logits
  const int V = p.V, W = (V + 31) / 32;
  uint32_t *pen = reinterpret_cast<uint32_t *>(xs + V);  // penalised tokens
  uint32_t *cand = pen + W;                               // candidates (top-k)
  uint32_t *kept = cand + W;                              // kept after the top-p cutoff
  __shared__ float redf[32];
  __shared__ unsigned redu[32];
  __shared__ float bestv[32];
  __shared__ int besti[32];
  __shared__ int s_pick;
  const int r = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  const float *l = p.logits + (size_t)r * V;
  for (int i = tid; i < V; i += nt) xs[i] = l[i];
  for (int w = tid; w < W; w += nt) pen[w] = 0u;
  __syncthreads();

  // repetition penalty, once per distinct in-range context token (sampler.rs:83-102)
  if (p.rep != 1.0f && p.ctx_len > 0) {
    const int32_t *ct = p.ctx_tokens + (size_t)r * p.ctx_stride;
    for (int j = tid; j < p.ctx_len; j += nt) {
      const int t = ct[j];
      if (t >= 0 && t < V) {
        const uint32_t bit = 1u << (t & 31);
        if (!(atomicOr(&pen[t >> 5], bit) & bit)) {
          const float v = xs[t];
          xs[t] = v > 0.0f ? v / p.rep : v * p.rep;
        }
      }
    }
  }
  __syncthreads();

  // greedy (sampler.rs:118-128): first maximum; NaN in slot 0 wins
  if (p.temperature <= 1e-4f) {
    float best = xs[0];
    int bi = 0;
    for (int i = tid; i < V; i += nt) {
      const float v = xs[i];
      if (v > best || (v == best && i < bi)) {
        best = v;
        bi = i;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if ((tid & 31) == 0) {
      bestv[tid >> 5] = best;
      besti[tid >> 5] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      float b = bestv[0];
      int bidx = besti[0];
      for (int w = 1; w < nt / 32; ++w)
        if (bestv[w] > b || (bestv[w] == b && besti[w] < bidx)) {
          b = bestv[w];
          bidx = besti[w];
        }
      p.out[r] = (xs[0] != xs[0]) ? 0 : bidx;
    }
    return;
  }

  // temperature (sampler.rs:130-133)
  const float inv_t = 1.0f / fmaxf(p.temperature, 1e-5f);
  for (int i = tid; i < V; i += nt) xs[i] *= inv_t;
  __syncthreads();

  // candidates: the top_k largest, ties by lowest index (sampler.rs:134-141)
  const bool use_k = p.top_k > 0 && p.top_k < V;
  uint32_t Tk = 0;
  if (use_k) {
    for (int bit = 31; bit >= 0; --bit) {
      const uint32_t trial = Tk | (1u << bit);
      unsigned c = 0;
      for (int i = tid; i < V; i += nt) c += order_key(xs[i]) >= trial;
      if (block_count(c, redu) >= (unsigned)p.top_k) Tk = trial;
    }
  }
  unsigned gt = 0, eq = 0;
  if (use_k) {
    for (int i = tid; i < V; i += nt) {
      const uint32_t k = order_key(xs[i]);
      gt += k > Tk;
      eq += k == Tk;
    }
    gt = block_count(gt, redu);
    eq = block_count(eq, redu);
  }
  const bool all_ties = !use_k || gt + eq == (unsigned)p.top_k;
  for (int w = tid; w < W; w += nt) {
    uint32_t m = 0;
    for (int b = 0; b < 32; ++b) {
      const int i = 32 * w + b;
      if (i >= V) break;
      const uint32_t k = order_key(xs[i]);
      if (!use_k || k > Tk || (all_ties && k == Tk)) m |= 1u << b;
    }
    cand[w] = m;
  }
  __syncthreads();
  if (!all_ties && tid == 0) {  // more equal logits than places: lowest indices first
    int need = p.top_k - (int)gt;
    for (int i = 0; i < V && need > 0; ++i)
      if (order_key(xs[i]) == Tk) {
        cand[i >> 5] |= 1u << (i & 31);
        --need;
      }
  }
  __syncthreads();

  // softmax over the candidates (sampler.rs:142-153): p_i = exp(x_i - max) / sum
  uint32_t kmax = 0;
  for (int i = tid; i < V; i += nt)
    if (has(cand, i)) kmax = max(kmax, order_key(xs[i]));
#pragma unroll
  for (int o = 16; o; o >>= 1) kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
  __syncthreads();
  if ((tid & 31) == 0) redu[tid >> 5] = kmax;
  __syncthreads();
  for (int w = 0; w < nt / 32; ++w) kmax = max(kmax, redu[w]);
  const float xmax = __uint_as_float((kmax & 0x80000000u) ? (kmax & 0x7fffffffu) : ~kmax);
  float part = 0.f;
  for (int i = tid; i < V; i += nt)
    if (has(cand, i)) part += expf(xs[i] - xmax);
  const float inv_sum = 1.0f / fmaxf(block_sum(part, redf), 1e-12f);
  auto prob = [&](int i) { return expf(xs[i] - xmax) * inv_sum; };
  // sum of p over set members with key >= T (T = 0: all)
  auto mass_ge = [&](const uint32_t *set, uint32_t T, bool strict) {
    float s = 0.f;
    for (int i = tid; i < V; i += nt)
      if (has(set, i)) {
        const uint32_t k = order_key(xs[i]);
        if (strict ? k > T : k >= T) s += prob(i);
      }
    return block_sum(s, redf);
  };
  // Largest key T with mass_ge(set, T) > target (strict) or >= target.
  auto bisect_mass = [&](const uint32_t *set, float target, bool strict) {
    uint32_t T = 0;
    for (int bit = 31; bit >= 0; --bit) {
      const uint32_t trial = T | (1u << bit);
      const float m = mass_ge(set, trial, false);
      if (strict ? m > target : m >= target) T = trial;
    }
    return T;
  };
  // Among items of `set` with key == T, in index order, the first whose
  // addition to `base` makes the running sum pass `target`; -1 if none.
  auto walk_ties = [&](const uint32_t *set, uint32_t T, float base, float target, bool strict) {
    unsigned c = 0;
    for (int i = tid; i < V; i += nt) c += has(set, i) && order_key(xs[i]) == T;
    if (block_count(c, redu) <= 1) {  // the usual case: one item holds that key, and it is the answer
      if (tid == 0) s_pick = -1;
      __syncthreads();
      for (int i = tid; i < V; i += nt)
        if (has(set, i) && order_key(xs[i]) == T) s_pick = i;
      __syncthreads();
      return s_pick;
    }
    if (tid == 0) {
      int pick = -1, last = -1;
      float c = base;
      for (int i = 0; i < V; ++i)
        if (has(set, i) && order_key(xs[i]) == T) {
          c += prob(i);
          last = i;
          if (strict ? c > target : c >= target) {
            pick = i;
            break;
          }
        }
      s_pick = pick >= 0 ? pick : last;
    }
    __syncthreads();
    return s_pick;
  };

  // top-p cutoff (sampler.rs:155-166): keep the sorted prefix through the
  // first item where the running sum exceeds top_p
  for (int w = tid; w < W; w += nt) kept[w] = cand[w];
  __syncthreads();
  if (p.top_p < 1.0f && mass_ge(cand, 0u, false) > p.top_p) {
    const float target = fmaxf(p.top_p, 0.0f);  // below 0 the first item crosses, as at 0
    const uint32_t Tp = bisect_mass(cand, target, true);
    const float above = mass_ge(cand, Tp, true);
    const int last = walk_ties(cand, Tp, above, target, true);  // the item that crosses top_p
    for (int w = tid; w < W; w += nt) {
      uint32_t m = 0;
      for (int b = 0; b < 32; ++b) {
        const int i = 32 * w + b;
        if (i >= V) break;
        const uint32_t k = order_key(xs[i]);
        if (has(cand, i) && (k > Tp || (k == Tp && i <= last))) m |= 1u << b;
      }
      kept[w] = m;
    }
    __syncthreads();
  }

  // draw (sampler.rs:167-179): the first item, in sorted order, where the
  // running sum reaches u * (kept mass); past the end: the top candidate
  const float total = mass_ge(kept, 0u, false);
  const float s = p.uniforms[r] * total;
  int pick;
  if (mass_ge(kept, kmax, false) >= s) {
    pick = walk_ties(kept, kmax, 0.f, s, false);
  } else {
    const uint32_t Ts = bisect_mass(kept, s, false);
    const float above = mass_ge(kept, Ts, true);
    pick = walk_ties(kept, Ts, above, s, false);
  }
  if (tid == 0) p.out[r] = pick;
}

}  // namespace

extern "C" int af_sample_rows(af_ctx *ctx, const float *logits, int rows, int vocab, const int32_t *context_tokens,
                              int64_t context_stride, int context_len, float temperature, int top_k, float top_p,
                              float repetition_penalty, const float *uniforms, int32_t *out, af_stream_t stream) {
  const char *fn = "af_sample_rows";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(logits && out && rows >= 0 && vocab > 0, "af_sample_rows", "bad arguments");
  AF_REQUIRE(vocab <= AF_SAMPLE_MAX_VOCAB, "af_sample_rows", "vocab %d exceeds the maximum %d", vocab,
             AF_SAMPLE_MAX_VOCAB);
  AF_REQUIRE(top_k >= 0, "af_sample_rows", "top_k must be >= 0");
  AF_REQUIRE(temperature <= 1e-4f || uniforms, "af_sample_rows", "uniforms are required unless greedy");
  AF_REQUIRE(context_len >= 0 && (context_len == 0 || (context_tokens && context_stride >= context_len)),
             "af_sample_rows", "bad context: len %d, stride %lld", context_len, (long long)context_stride);
  if (rows == 0) return AF_OK;
  auto smem_for = [](int v) { return (size_t)v * 4 + (size_t)3 * ((v + 31) / 32) * 4; };
  const size_t smem = smem_for(vocab);
  static std::atomic<unsigned long long> attr_devices{0};  // limit raised once for the largest vocabulary
  if (int arc = af::smem_attr(ctx, reinterpret_cast<const void *>(sample_rows_kernel), smem_for(AF_SAMPLE_MAX_VOCAB),
                              attr_devices, fn))
    return arc;
  SampleParams sp{logits,      vocab,        context_tokens, context_stride, context_len, temperature,
                  top_p,       repetition_penalty, top_k,  uniforms,       out};
  sample_rows_kernel<<<rows, kThreads, smem, af::stream_of(stream)>>>(sp);
  return af::launched(ctx, fn);
}
