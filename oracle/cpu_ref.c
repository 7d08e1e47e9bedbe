/*
 * CPU oracle: a C restatement of AceFlow's Rust SIMD CPU path.
 *
 * TEST INFRASTRUCTURE ONLY.  The aceflow_b200 package never links or loads
 * this library.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline / reference arm call it, as the checker or as the timed CPU
 * baseline ("restatement of the reference CPU path": the reference is Rust
 * and there is no Rust toolchain, so its own binary cannot be built).
 *
 * Each function restates a reference function with the same loop order and,
 * for the GEMV, the same AVX2/FMA 4-row x 8-lane accumulation and horizontal
 * sum, so its fp32 rounding follows the reference:
 *   oref_retention_step_core  aceflow-core/src/cpu/recurrence.rs:3-42
 *   oref_gemv                 aceflow-core/src/cpu/gemv.rs:164-184 (dispatch),
 *                             gemv_avx2 13-77, hsum_avx2 79-90, gemv_scalar 152-161
 *   oref_rmsnorm_core         aceflow-core/src/cpu/norm.rs:6-59
 *   oref_swiglu_forward       aceflow-core/src/cpu/swiglu.rs:4-18
 *   oref_dot_product          aceflow-core/src/cpu/sampler.rs:36-65
 *   oref_forward_layer        aceflow-core/src/cpu/mod.rs:646-706
 *   oref_generate_greedy      aceflow-core/src/cpu/mod.rs:708-769 with
 *                             sampler.rs:67-128 at temperature 0
 * Batched drivers run independent streams on OpenMP threads the way the
 * reference runs rows on rayon (gemv.rs:187-194).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <immintrin.h>
#include <omp.h>

/* ---------------------------------------------------------------- retention */
void oref_retention_step_core(float *states, const float *gamma, size_t layer_idx,
                              size_t num_heads, size_t head_dim, const float *q,
                              const float *k, const float *v, float *out) {
  const size_t d = head_dim, hs = d * d;
  const size_t layer_offset = layer_idx * num_heads * hs;
  for (size_t h = 0; h < num_heads; ++h) {
    const float decay = gamma[h];
    const float *qh = q + h * d, *kh = k + h * d, *vh = v + h * d;
    float *S = states + layer_offset + h * hs;
    float *o = out + h * d;
    for (size_t j = 0; j < d; ++j) o[j] = 0.0f;
    for (size_t i = 0; i < d; ++i) {
      const float kv = kh[i], qv = qh[i];
      float *row = S + i * d;
      for (size_t j = 0; j < d; ++j) {
        /* Rust does not contract a*b+c into an FMA; neither does this file
         * (built with -ffp-contract=off), so each product is rounded. */
        const float updated = decay * row[j] + kv * vh[j];
        row[j] = updated;
        o[j] += qv * updated;
      }
    }
  }
}

/* ---------------------------------------------------------------- gemv */
void oref_gemv_scalar(size_t m, size_t k, const float *w, const float *x, float *y) {
  for (size_t r = 0; r < m; ++r) {
    const float *row = w + r * k;
    float s = 0.0f;
    for (size_t j = 0; j < k; ++j) s += row[j] * x[j];
    y[r] = s;
  }
}

__attribute__((target("avx2,fma"))) static float hsum_avx2(__m256 value) {
  __m128 low = _mm256_castps256_ps128(value);
  __m128 high = _mm256_extractf128_ps(value, 1);
  __m128 sum128 = _mm_add_ps(low, high);
  __m128 shuffled = _mm_movehl_ps(sum128, sum128);
  __m128 sum64 = _mm_add_ps(sum128, shuffled);
  __m128 shuffled2 = _mm_shuffle_ps(sum64, sum64, 1);
  return _mm_cvtss_f32(_mm_add_ss(sum64, shuffled2));
}

__attribute__((target("avx2,fma"))) static void gemv_avx2(size_t m, size_t k, const float *w,
                                                          const float *x, float *y) {
  size_t row = 0;
  const size_t kc = (k / 8) * 8;
  for (; row + 4 <= m; row += 4) {
    __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps();
    __m256 a2 = _mm256_setzero_ps(), a3 = _mm256_setzero_ps();
    const float *r0 = w + row * k, *r1 = r0 + k, *r2 = r1 + k, *r3 = r2 + k;
    size_t j = 0;
    for (; j < kc; j += 8) {
      __m256 xv = _mm256_loadu_ps(x + j);
      a0 = _mm256_fmadd_ps(_mm256_loadu_ps(r0 + j), xv, a0);
      a1 = _mm256_fmadd_ps(_mm256_loadu_ps(r1 + j), xv, a1);
      a2 = _mm256_fmadd_ps(_mm256_loadu_ps(r2 + j), xv, a2);
      a3 = _mm256_fmadd_ps(_mm256_loadu_ps(r3 + j), xv, a3);
    }
    float s0 = hsum_avx2(a0), s1 = hsum_avx2(a1), s2 = hsum_avx2(a2), s3 = hsum_avx2(a3);
    for (; j < k; ++j) {
      const float xj = x[j];
      s0 += r0[j] * xj; s1 += r1[j] * xj; s2 += r2[j] * xj; s3 += r3[j] * xj;
    }
    y[row] = s0; y[row + 1] = s1; y[row + 2] = s2; y[row + 3] = s3;
  }
  for (; row < m; ++row) {
    __m256 acc = _mm256_setzero_ps();
    const float *r = w + row * k;
    size_t j = 0;
    for (; j < kc; j += 8) acc = _mm256_fmadd_ps(_mm256_loadu_ps(r + j), _mm256_loadu_ps(x + j), acc);
    float s = hsum_avx2(acc);
    for (; j < k; ++j) s += r[j] * x[j];
    y[row] = s;
  }
}

static int have_avx2_fma(void) {
  static int cached = -1;
  if (cached < 0) {
    __builtin_cpu_init();
    cached = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
  }
  return cached;
}

void oref_gemv(size_t m, size_t k, const float *w, const float *x, float *y) {
  if (have_avx2_fma() && k >= 8) gemv_avx2(m, k, w, x, y);
  else oref_gemv_scalar(m, k, w, x, y);
}

/* ---------------------------------------------------------------- norms */
void oref_rmsnorm_core(float *x, const float *w, size_t len, float eps) {
  if (len == 0) return;
  float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const size_t body = len - len % 8;
  for (size_t c = 0; c < body; c += 8)
    for (int t = 0; t < 8; ++t) s[t] += x[c + t] * x[c + t];
  float sum_sq = ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
  for (size_t c = body; c < len; ++c) sum_sq += x[c] * x[c];
  const float inv = 1.0f / sqrtf(sum_sq / (float)len + eps);
  for (size_t c = 0; c < len; ++c) x[c] *= inv * w[c];
}

void oref_swiglu_forward(size_t ffn_dim, const float *gate_up, float *hidden) {
  const float *g = gate_up, *u = gate_up + ffn_dim;
  for (size_t i = 0; i < ffn_dim; ++i) hidden[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
}

float oref_dot_product(const float *a, const float *b, size_t n) {
  float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const size_t body = n - n % 8;
  for (size_t c = 0; c < body; c += 8)
    for (int t = 0; t < 8; ++t) s[t] += a[c + t] * b[c + t];
  float total = ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
  for (size_t c = body; c < n; ++c) total += a[c] * b[c];
  return total;
}

/* ---------------------------------------------------------------- MSR step */
/* One recurrent step of one MultiScaleRetention layer for one stream:
 * qkv = W_qkv x (gemv, 3d x d); retention_step_core; RMSNorm(eps) with
 * weight ret_w; out = W_o normed.  Same sequence as AceEngine's retention
 * half (cpu/mod.rs:651-678); scratch must hold 5*d floats. */
static void msr_step_one(size_t d, size_t H, const float *x, float *state, const float *gamma,
                         const float *w_qkv, const float *w_o, const float *ret_w, float eps,
                         float *out, float *scratch) {
  float *qkv = scratch, *o = scratch + 3 * d, *tmp = scratch + 4 * d;
  oref_gemv(3 * d, d, w_qkv, x, qkv);
  oref_retention_step_core(state, gamma, 0, H, d / H, qkv, qkv + d, qkv + 2 * d, o);
  memcpy(tmp, o, d * sizeof(float));
  oref_rmsnorm_core(tmp, ret_w, d, eps);
  oref_gemv(d, d, w_o, tmp, out);
}

/* x [B,d], state [B,H,dh,dh], out [B,d]; streams split over nthreads. */
void oref_msr_decode_step_batched(size_t B, size_t d, size_t H, const float *x, float *state,
                                  const float *gamma, const float *w_qkv, const float *w_o,
                                  const float *ret_w, float eps, float *out, int nthreads) {
  const size_t dh = d / H, ss = H * dh * dh;
#pragma omp parallel num_threads(nthreads)
  {
    float *scratch = (float *)malloc(5 * d * sizeof(float));
#pragma omp for schedule(static)
    for (long b = 0; b < (long)B; ++b)
      msr_step_one(d, H, x + b * d, state + b * ss, gamma, w_qkv, w_o, ret_w, eps, out + b * d, scratch);
    free(scratch);
  }
}

/* Token-serial prefill (the reference's only CPU prefill, cpu/mod.rs:547-587,
 * here returning every token's layer output): x [B,T,d] -> out [B,T,d]. */
void oref_msr_prefill_recurrent_batched(size_t B, size_t T, size_t d, size_t H, const float *x,
                                        float *state, const float *gamma, const float *w_qkv,
                                        const float *w_o, const float *ret_w, float eps,
                                        float *out, int nthreads) {
  const size_t dh = d / H, ss = H * dh * dh;
#pragma omp parallel num_threads(nthreads)
  {
    float *scratch = (float *)malloc(5 * d * sizeof(float));
#pragma omp for schedule(static)
    for (long b = 0; b < (long)B; ++b)
      for (size_t t = 0; t < T; ++t)
        msr_step_one(d, H, x + (b * T + t) * d, state + b * ss, gamma, w_qkv, w_o, ret_w, eps,
                     out + (b * T + t) * d, scratch);
    free(scratch);
  }
}

/* ---------------------------------------------------------------- decoder */
typedef struct {
  const float *w_qkv, *w_o, *w_gate_up, *w_down, *norm1, *norm2, *ret_norm;
} oref_layer;

/* AceEngine.forward_layer_internal (cpu/mod.rs:646-706) for one stream.
 * scratch: 6*d + 3*f floats. */
static void forward_layer_one(size_t d, size_t H, size_t f, size_t layer_idx, const oref_layer *L,
                              float *states, const float *gamma, float eps, float *x,
                              float *scratch) {
  float *norm_buf = scratch, *qkv = scratch + d, *ret_out = scratch + 4 * d,
        *proj = scratch + 5 * d, *gate_up = scratch + 6 * d, *hidden = gate_up + 2 * f;
  memcpy(norm_buf, x, d * sizeof(float));
  oref_rmsnorm_core(norm_buf, L->norm1, d, eps);
  oref_gemv(3 * d, d, L->w_qkv, norm_buf, qkv);
  oref_retention_step_core(states, gamma, layer_idx, H, d / H, qkv, qkv + d, qkv + 2 * d, ret_out);
  oref_rmsnorm_core(ret_out, L->ret_norm, d, eps);
  oref_gemv(d, d, L->w_o, ret_out, proj);
  for (size_t j = 0; j < d; ++j) x[j] += proj[j];
  memcpy(norm_buf, x, d * sizeof(float));
  oref_rmsnorm_core(norm_buf, L->norm2, d, eps);
  oref_gemv(2 * f, d, L->w_gate_up, norm_buf, gate_up);
  oref_swiglu_forward(f, gate_up, hidden);
  oref_gemv(d, f, L->w_down, hidden, proj);
  for (size_t j = 0; j < d; ++j) x[j] += proj[j];
}

/* Greedy generation for B independent streams (generate_stream_internal,
 * cpu/mod.rs:708-769, temperature 0, repetition penalty 1.0, no final norm,
 * tied LM head = embedding table, EOS id 2 stops a stream when stop_at_eos).
 * layers: array of num_layers oref_layer; states [B, L, H, dh, dh] zeroed by
 * the caller; prompts [B, P]; out_tokens [B, n_new] (-1 after a stop);
 * if logits_out is non-NULL it receives [B, n_new, V] logits and teacher
 * tokens (if non-NULL, [B, n_new]) are fed back instead of the argmax. */
void oref_generate_greedy(size_t B, size_t num_layers, size_t d, size_t H, size_t f, size_t V,
                          const oref_layer *layers, const float *embedding, float *states,
                          const float *gamma, float eps, const int32_t *prompts, size_t P,
                          size_t n_new, int stop_at_eos, const int32_t *teacher,
                          int32_t *out_tokens, float *logits_out, float *hidden_out,
                          int nthreads) {
  const size_t dh = d / H, ls = H * dh * dh;
#pragma omp parallel num_threads(nthreads)
  {
    float *scratch = (float *)malloc((6 * d + 3 * f) * sizeof(float));
    float *cur = (float *)malloc(d * sizeof(float));
    float *logits = (float *)malloc(V * sizeof(float));
#pragma omp for schedule(static)
    for (long b = 0; b < (long)B; ++b) {
      float *st = states + (size_t)b * num_layers * ls;
      memset(cur, 0, d * sizeof(float));
      for (size_t p = 0; p < P; ++p) {
        const int32_t tok = prompts[b * P + p];
        if (tok >= 0 && (size_t)tok < V) memcpy(cur, embedding + (size_t)tok * d, d * sizeof(float));
        for (size_t l = 0; l < num_layers; ++l)
          forward_layer_one(d, H, f, l, &layers[l], st, gamma, eps, cur, scratch);
      }
      int stopped = 0;
      for (size_t s = 0; s < n_new; ++s) {
        if (stopped) { out_tokens[b * n_new + s] = -1; continue; }
        if (hidden_out) memcpy(hidden_out + ((size_t)b * n_new + s) * d, cur, d * sizeof(float));
        for (size_t r = 0; r < V; ++r) logits[r] = oref_dot_product(embedding + r * d, cur, d);
        if (logits_out) memcpy(logits_out + ((size_t)b * n_new + s) * V, logits, V * sizeof(float));
        size_t best = 0;
        float bv = logits[0];
        for (size_t r = 1; r < V; ++r)
          if (logits[r] > bv) { bv = logits[r]; best = r; }
        out_tokens[b * n_new + s] = (int32_t)best;
        int32_t next = teacher ? teacher[b * n_new + s] : (int32_t)best;
        if (stop_at_eos && next == 2) { stopped = 1; continue; }
        if (next >= 0 && (size_t)next < V) memcpy(cur, embedding + (size_t)next * d, d * sizeof(float));
        else memset(cur, 0, d * sizeof(float));
        for (size_t l = 0; l < num_layers; ++l)
          forward_layer_one(d, H, f, l, &layers[l], st, gamma, eps, cur, scratch);
      }
    }
    free(scratch);
    free(cur);
    free(logits);
  }
}

/* One decoder layer at one token for B streams (batched forward_layer). */
void oref_forward_layer_batched(size_t B, size_t d, size_t H, size_t f, size_t layer_idx,
                                size_t num_layers, const oref_layer *L, float *states,
                                const float *gamma, float eps, float *x, int nthreads) {
  const size_t dh = d / H, ls = H * dh * dh;
#pragma omp parallel num_threads(nthreads)
  {
    float *scratch = (float *)malloc((6 * d + 3 * f) * sizeof(float));
#pragma omp for schedule(static)
    for (long b = 0; b < (long)B; ++b)
      forward_layer_one(d, H, f, layer_idx, L, states + (size_t)b * num_layers * ls, gamma, eps,
                        x + b * d, scratch);
    free(scratch);
  }
}

int oref_max_threads(void) { return omp_get_max_threads(); }
