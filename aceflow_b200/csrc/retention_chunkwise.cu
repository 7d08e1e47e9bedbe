// Chunkwise-parallel retention (prefill) on the sm_100a bf16 tensor cores.
//
// Reference semantics: the parallel form O = (Q K^T * D) V with
// D[i,j] = gamma^(i-j) (aceflow/nn/retention.py:51-61), equal to the
// recurrence of aceflow-core/src/cpu/recurrence.rs:28-39.  Per chunk of C
// tokens starting at t0, with S the state after token t0-1:
//     O_c = D_c (Q_c S + P' V_c),   D_c = diag(gamma^(i+1)),
//           P'[i,j] = (q_i . k_j) gamma^-(j+1)  for j <= i, else 0
//     S  <- gamma^L S + (K_c^T) (diag(gamma^(L-1-j)) V_c)       (L = chunk length)
// (pulling D_c out of the intra term lets one TMEM accumulator hold both
// terms; gamma^-(j+1) <= gamma^-64 stays small).
//
// One CTA owns one (stream b, head h, 128-wide slice of the value dim) and
// walks the chunks in order; the fp32 state slice lives in TMEM for the whole
// sequence, transposed (S^T: TMEM lane = value index v, column = key index k),
// so every MMA operand is either a TMA tile as stored in global memory or a
// tile the math warps write themselves:
//   scores  Sc  = Q_c K_c^T         M=64  N=64  K=256  A,B K-major (TMA)
//   output  O^T = S^T Q_c^T         M=128 N=64  K=256  A = bf16(S^T) K-major (written)
//              + V_c^T P'^T                       K=64   A = V_c MN-major (TMA), B = P' (written)
//   update  S^T += Vs^T K_c        M=128 N=256 K=64   A = decay-scaled V (written), B = K_c MN-major
// Warp roles (320 threads): warp 0 TMA producer; warp 1 TMEM allocator and
// single-thread tcgen05.mma issuer (the state term of O is issued as soon as
// the bf16 state operand is written, before the decay mask is ready); warps
// 2-9 math (TMEM ld/st, decay masks
// generated in registers, bf16 operand tiles, output + RMSNorm partials):
// two warps per TMEM lane quadrant, each taking half of the columns of every
// step, so the per-chunk chain of TMEM round trips is split in two.
//
// Inputs come straight from the bf16 QKV projection [B*T][3d] through one
// 3-D tensor map (d_model fastest, then T, then B) so the T edge zero-fills.
// Outputs: O * ret_norm_w as bf16 [B*T][d] (the A operand of the W_o GEMM;
// staged in shared memory and written by TMA stores, one per 64 x 64 box),
// per-row partial sums of O^2 (the GEMM applies 1/rms per row), and the
// final state in the decode layout [B][H][k][v] fp32.
//
// Sequence segments.  When B*H*(DH/VS) CTAs cannot fill the GPU (one long
// stream, few heads per GPU), each stream is cut into nseg segments of
// seg_len tokens (a multiple of C) and three launches replace one:
//   1. state pass (STATE_ONLY): per segment, from a zero state,
//        dS_s = sum_t gamma^(end_s-1-t) k_t^T v_t   (V pre-scaled, no TMEM decay)
//   2. seg_scan_kernel: S_in[0] = state_in, S_in[s+1] = gamma^seg_len S_in[s] + dS_s
//   3. full pass: every segment runs the chunk loop from S_in[s]; the last
//      segment writes the final state.
// The result equals the single-pass recurrence (the scan is the same
// recurrence applied at segment granularity).
#include "common.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>

namespace {

using namespace sm100;

constexpr int C = 64;       // chunk length (tokens)
constexpr int DH = 256;     // head dim
constexpr int VS = 128;     // value slice per CTA
constexpr int NSL = DH / VS;

constexpr int Q_OFF = 0, Q_BYTES = C * DH * 2;             // 4 K-slices [64 x 64] bf16, 8 KB each
constexpr int K_OFF = Q_OFF + Q_BYTES, K_BYTES = C * DH * 2;
constexpr int V_OFF = K_OFF + K_BYTES, V_BYTES = C * VS * 2;  // 2 boxes [64 tok x 64 v]
constexpr int SOP_OFF = V_OFF + V_BYTES, SOP_BYTES = VS * DH * 2;  // 4 K-slices [128 v x 64 k], 16 KB each
constexpr int P_OFF = SOP_OFF + SOP_BYTES, P_BYTES = C * C * 2;    // [64 i x 64 j]
constexpr int VT_OFF = P_OFF + P_BYTES, VT_BYTES = V_BYTES;         // decay-scaled V, V's layout
// output staging for the TMA store, two buffers of two [64 tok x 64 v] bf16 halves
constexpr int OST_OFF = VT_OFF + VT_BYTES, OST_HALF = C * 64 * 2, OST_BYTES = 2 * 2 * OST_HALF;
constexpr int TILE_BYTES = OST_OFF + OST_BYTES;                     // 200 KB
// The state-only pass keeps a ring of SO_NS slots (K, V, decay-scaled V) in
// the same space, so its loads run two chunks ahead of its update MMAs.
constexpr int SO_SLOT = K_BYTES + 2 * V_BYTES, SO_NS = 3;
static_assert(SO_NS * SO_SLOT <= TILE_BYTES, "state-pass ring");
// tail: 24 mbarrier words (the TMEM slot in the last), gamma^n (C+1),
// gamma^-(j+1) (C), [4][C] partials
constexpr size_t TAIL_BYTES = 24 * 8 + 4 * ((C + 1) + C + 4 * C);
constexpr size_t SMEM = 1024 + TILE_BYTES + ((TAIL_BYTES + 255) / 256) * 256;
constexpr int BOX = 64 * 64 * 2;  // one TMA box: 64 rows x 128 bytes

constexpr uint32_t TM_S = 0, TM_SC = 256, TM_O = 320, TM_COLS = 512;

struct ChunkParams {
  int B, T, H;
  int nseg, seg_len;      // segments per stream and their length (seg_len % C == 0)
  const float *gamma;
  const float *state_in;  // [B][nseg][H][DH][DH] state before each segment, or null (zeros)
  float *state_out;       // [B][H][DH][DH] final state (STATE_ONLY: [B][nseg][H][DH][DH] segment states), or null
  __nv_bfloat16 *out;     // [B*T][H*DH]
  const float *norm_w;    // [H*DH] or null
  float *sumsq;           // [B*T][H*NSL] or null
  int *err;
  int64_t ldo = 0;        // output row stride in elements (0: H*DH; 128-token kernel only)
  int out_reverse = 0;    // token t of a stream is written to row T-1-t (128-token kernel only)
};

// MN-major SW128 descriptor: 64-element MN blocks `lbo` bytes apart, 8-row
// K groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc_mn_sw128(const void *tile, uint32_t lbo) {
  const uint64_t addr = smem_u32(tile);
  return ((addr >> 4) & 0x3FFFull) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) | ((uint64_t)(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

// Byte offset of 16-byte chunk `c16` of row `r` in a 128B-swizzled tile.
__device__ __forceinline__ uint32_t sw128(int r, int c16) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c16 ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

constexpr int MATH_THREADS = 256;  // warps 2-9

// TMA store of a [64 x 64] bf16 box from shared memory (bulk group).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void math_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Named barrier over the 256 math threads that also ORs a predicate, so every
// participant leaves with the same answer (s_abort may change concurrently).
__device__ __forceinline__ bool math_sync_or(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, 256, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}

template <bool STATE_ONLY>
__global__ void __launch_bounds__(320, 1)
    retention_chunkwise_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                               const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tm_out,
                               ChunkParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + TILE_BYTES);
  uint64_t *bar_load = bars + 0, *bar_sc = bars + 1, *bar_math = bars + 2, *bar_o = bars + 3, *bar_upd = bars + 4,
           *bar_out = bars + 5, *bar_sop = bars + 6;
  // state-only pass: per ring slot, loads landed / scaled V written / update done
  uint64_t *bar_lds = bars + 8, *bar_mts = bars + 11, *bar_ups = bars + 14;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 23);
  float *gpow = reinterpret_cast<float *>(bars + 24);  // gamma^n, n = 0..C
  float *ginv = gpow + (C + 1);                        // gamma^-(j+1), j = 0..C-1
  float *red = ginv + C;                               // [4][C] per-warp partial sums
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slice = blockIdx.x % NSL;
  const int bsh = blockIdx.x / NSL;   // ((b * nseg) + s) * H + h
  const int h = bsh % p.H, bs = bsh / p.H;
  const int b = bs / p.nseg, s = bs % p.nseg;
  const int tb = s * p.seg_len;                      // first token of this segment
  const int te = min(p.T, tb + p.seg_len);           // one past its last token
  const int nch = (te - tb + C - 1) / C;
  const float g = p.gamma[h];
  const float lg = log2f(g);

  if (threadIdx.x == 0) {
    s_abort = 0;
    mbar_init(bar_load, 1);
    mbar_init(bar_sc, 1);
    mbar_init(bar_math, MATH_THREADS);
    mbar_init(bar_o, 1);
    mbar_init(bar_upd, 1);
    mbar_init(bar_out, MATH_THREADS);
    mbar_init(bar_sop, MATH_THREADS);
    for (int i = 0; i < SO_NS; ++i) {
      mbar_init(&bar_lds[i], 1);
      mbar_init(&bar_mts[i], MATH_THREADS);
      mbar_init(&bar_ups[i], 1);
    }
    fence_barrier_init();
    if (!STATE_ONLY) prefetch_tmap(&tmq);
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
    if (!STATE_ONLY) prefetch_tmap(&tm_out);
  }
  if (threadIdx.x >= 64 && threadIdx.x < 64 + C + 1) {
    const int n = threadIdx.x - 64;
    gpow[n] = exp2f((float)n * lg);
    if (n < C) ginv[n] = exp2f(-(float)(n + 1) * lg);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&]() {
    s_abort = 1;
    atomicOr(p.err, 1 << AF_ERR_TIMEOUT);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && STATE_ONLY) {
      // ring of SO_NS slots: slot c % SO_NS is reused once chunk c - SO_NS's update retired
      int issued = 0;
      for (int c = 0; c < nch && !s_abort; ++c) {
        const int sl = c % SO_NS;
        if (c >= SO_NS && !mbar_wait(&bar_ups[sl], ((c / SO_NS) - 1) & 1)) { fail(); break; }
        const int t0 = tb + c * C;
        uint8_t *base = sm + sl * SO_SLOT;
        mbar_arrive_expect_tx(&bar_lds[sl], K_BYTES + V_BYTES);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tma_load_3d(base + kk * BOX, &tmk, &bar_lds[sl], h * DH + kk * 64, t0, b);
#pragma unroll
        for (int vb = 0; vb < 2; ++vb)
          tma_load_3d(base + K_BYTES + vb * BOX, &tmv, &bar_lds[sl], h * DH + slice * VS + vb * 64, t0, b);
        issued = c + 1;
      }
      for (int c = issued - SO_NS < 0 ? 0 : issued - SO_NS; c < issued; ++c)  // loads still in flight
        if (!mbar_wait(&bar_lds[c % SO_NS], (c / SO_NS) & 1)) { fail(); break; }
    } else if (lane == 0) {
      int issued = 0;
      for (int c = 0; c < nch && !s_abort; ++c) {
        if (c > 0 && !mbar_wait(bar_upd, (c - 1) & 1)) { fail(); break; }
        const int t0 = tb + c * C;
        mbar_arrive_expect_tx(bar_load, (STATE_ONLY ? 0 : Q_BYTES) + K_BYTES + V_BYTES);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          if (!STATE_ONLY) tma_load_3d(sm + Q_OFF + kk * BOX, &tmq, bar_load, h * DH + kk * 64, t0, b);
          tma_load_3d(sm + K_OFF + kk * BOX, &tmk, bar_load, h * DH + kk * 64, t0, b);
        }
#pragma unroll
        for (int vb = 0; vb < 2; ++vb)
          tma_load_3d(sm + V_OFF + vb * BOX, &tmv, bar_load, h * DH + slice * VS + vb * 64, t0, b);
        issued = c + 1;
        if (c + 1 < nch) {  // the next chunk's tiles into L2 (its loads wait for this chunk's update)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            if (!STATE_ONLY) tma_prefetch_3d(&tmq, h * DH + kk * 64, t0 + C, b);
            tma_prefetch_3d(&tmk, h * DH + kk * 64, t0 + C, b);
          }
#pragma unroll
          for (int vb = 0; vb < 2; ++vb) tma_prefetch_3d(&tmv, h * DH + slice * VS + vb * 64, t0 + C, b);
        }
      }
      if (issued > 0 && !mbar_wait(bar_load, (issued - 1) & 1)) fail();  // last load landed
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t id_sc = idesc_f32acc(kFmtBF16, 64, 64);
    constexpr uint32_t id_inter = idesc_f32acc(kFmtBF16, 128, 64);
    constexpr uint32_t id_intra = idesc_f32acc(kFmtBF16, 128, 64) | (1u << 15);         // A MN-major
    constexpr uint32_t id_upd = idesc_f32acc(kFmtBF16, 128, 256) | (1u << 15) | (1u << 16);  // A, B MN-major
    if constexpr (STATE_ONLY) {
      // only the update: S^T += Vs^T . K once the math warps wrote Vs
      for (int c = 0; c < nch; ++c) {
        const int sl = c % SO_NS;
        uint8_t *base = sm + sl * SO_SLOT;
        bool ok = mbar_wait(&bar_mts[sl], (c / SO_NS) & 1);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok || __any_sync(0xffffffffu, s_abort != 0)) { if (!ok && lane == 0) fail(); break; }
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t da = sdesc_mn_sw128(base + K_BYTES + V_BYTES + k * 2048, BOX);
            const uint64_t db = sdesc_mn_sw128(base + k * 2048, BOX);
            umma_bf16(tmem + TM_S, da, db, id_upd, 1);
          }
          umma_commit(&bar_ups[sl]);
        }
        __syncwarp();
      }
    } else
    for (int c = 0; c < nch; ++c) {
      bool ok = mbar_wait(bar_load, c & 1);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || __any_sync(0xffffffffu, s_abort != 0)) { if (!ok && lane == 0) fail(); break; }
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t da = sdesc_k_sw128(sm + Q_OFF + kk * BOX) + ((k * 32) >> 4);
            const uint64_t db = sdesc_k_sw128(sm + K_OFF + kk * BOX) + ((k * 32) >> 4);
            umma_bf16(tmem + TM_SC, da, db, id_sc, (kk | k) != 0);
          }
        umma_commit(bar_sc);
      }
      __syncwarp();
      // O^T = bf16(S^T) . Q^T (K = 256 keys) as soon as the state operand is
      // written: it overlaps the math warps' decay mask and scaled V
      ok = mbar_wait(bar_sop, c & 1);
      if (ok && c > 0) ok = mbar_wait(bar_out, (c - 1) & 1);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || __any_sync(0xffffffffu, s_abort != 0)) { if (!ok && lane == 0) fail(); break; }
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t da = sdesc_k_sw128(sm + SOP_OFF + kk * 2 * BOX) + ((k * 32) >> 4);
            const uint64_t db = sdesc_k_sw128(sm + Q_OFF + kk * BOX) + ((k * 32) >> 4);
            umma_bf16(tmem + TM_O, da, db, id_inter, (kk | k) != 0);
          }
      }
      __syncwarp();
      ok = mbar_wait(bar_math, c & 1);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || __any_sync(0xffffffffu, s_abort != 0)) { if (!ok && lane == 0) fail(); break; }
      tc_fence_after();
      if (lane == 0) {
        //     + V^T . P'^T  (K = 64 tokens)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t da = sdesc_mn_sw128(sm + V_OFF + k * 2048, BOX);
          const uint64_t db = sdesc_k_sw128(sm + P_OFF) + ((k * 32) >> 4);
          umma_bf16(tmem + TM_O, da, db, id_intra, 1);
        }
        umma_commit(bar_o);
        // S^T += Vs^T . K  (K = 64 tokens, N = 256 keys)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t da = sdesc_mn_sw128(sm + VT_OFF + k * 2048, BOX);
          const uint64_t db = sdesc_mn_sw128(sm + K_OFF + k * 2048, BOX);
          umma_bf16(tmem + TM_S, da, db, id_upd, 1);
        }
        umma_commit(bar_upd);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ math warps
    const int q = warp & 3;            // TMEM lane quadrant
    const int half = (warp - 2) >> 2;  // which half of the columns this warp takes
    const int mt = threadIdx.x - 64;   // 0..255
    const int v = q * 32 + lane;       // TMEM lane of this thread = value index in the slice
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    // initial state S^T[v][k] = S[k][v]
    {
      const float *sin = (!STATE_ONLY && p.state_in) ? p.state_in + ((size_t)bsh * DH) * DH + slice * VS + v : nullptr;
#pragma unroll 1
      for (int k0 = half * (DH / 2); k0 < (half + 1) * (DH / 2); k0 += 16) {
        float x[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) x[j] = sin ? sin[(size_t)(k0 + j) * DH] : 0.f;
        __syncwarp();
        tmem_st16(tmem + lane_base + TM_S + k0, x);
      }
      tmem_wait_st();
    }
    if constexpr (STATE_ONLY) {
      // Vs = diag(gamma^(te-1-t)) V for the chunk's tokens t: decay to the segment end
      for (int c = 0; c < nch; ++c) {
        const int t0 = tb + c * C;
        const int L = min(C, te - t0);
        const float tail = exp2f((float)(te - t0 - L) * lg);  // gamma^(tokens after this chunk)
        const int sl = c % SO_NS;
        uint8_t *base = sm + sl * SO_SLOT;
        bool ok = mbar_wait(&bar_lds[sl], (c / SO_NS) & 1);
        if (!ok) s_abort = 1;
        if (ok) {
#pragma unroll 2
          for (int i = mt; i < V_BYTES / 16; i += MATH_THREADS) {
            const int off = i * 16;
            const int j = (off % BOX) / 128;
            const float sc = j < L ? gpow[L - 1 - j] * tail : 0.f;
            uint4 raw = *reinterpret_cast<const uint4 *>(base + K_BYTES + off);
            __nv_bfloat162 *e = reinterpret_cast<__nv_bfloat162 *>(&raw);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              float2 f = __bfloat1622float2(e[u]);
              e[u] = __floats2bfloat162_rn(f.x * sc, f.y * sc);
            }
            *reinterpret_cast<uint4 *>(base + K_BYTES + V_BYTES + off) = raw;
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bar_mts[sl]);
        if (math_sync_or(s_abort != 0)) break;
      }
    } else
    for (int c = 0; c < nch; ++c) {
      const int t0 = tb + c * C;
      const int L = min(C, te - t0);
      bool ok = true;
      if (c > 0) ok = mbar_wait(bar_upd, (c - 1) & 1);
      if (!ok) s_abort = 1;
      if (math_sync_or(s_abort != 0)) break;
      tc_fence_after();
      // (a) S_op = bf16(S^T) (K-major [v][k]); S^T *= gamma^L in TMEM
      const float gL = gpow[L];
#pragma unroll 1
      for (int k0 = half * (DH / 2); k0 < (half + 1) * (DH / 2); k0 += 64) {  // 64 columns per TMEM round trip
        float x[64];
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 4; ++u) tmem_ld16(tmem + lane_base + TM_S + k0 + 16 * u, *reinterpret_cast<float(*)[16]>(x + 16 * u));
        tmem_wait_ld();
        uint8_t *slice_base = sm + SOP_OFF + (k0 >> 6) * (2 * BOX);
#pragma unroll
        for (int c16 = 0; c16 < 8; ++c16) {
          const float *y = x + 8 * c16;
          *reinterpret_cast<uint4 *>(slice_base + sw128(v, c16)) =
              make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]), pack_bf16(y[6], y[7]));
        }
#pragma unroll
        for (int j = 0; j < 64; ++j) x[j] *= gL;
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 4; ++u) tmem_st16(tmem + lane_base + TM_S + k0 + 16 * u, *reinterpret_cast<float(*)[16]>(x + 16 * u));
      }
      tmem_wait_st();
      fence_proxy_async_smem();  // S_op (generic stores) before the MMAs that read it
      tc_fence_before();
      mbar_arrive(bar_sop);
      // (b) Vs = diag(gamma^(L-1-j)) V, same swizzled layout as V
      ok = mbar_wait(bar_load, c & 1);
      if (!ok) s_abort = 1;
      if (ok) {
#pragma unroll 2
        for (int i = mt; i < V_BYTES / 16; i += MATH_THREADS) {
          const int off = i * 16;
          const int j = (off % BOX) / 128;  // token row of this 16-byte chunk
          const float sc = j < L ? gpow[L - 1 - j] : 0.f;
          uint4 raw = *reinterpret_cast<const uint4 *>(sm + V_OFF + off);
          __nv_bfloat162 *e = reinterpret_cast<__nv_bfloat162 *>(&raw);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float2 f = __bfloat1622float2(e[u]);
            e[u] = __floats2bfloat162_rn(f.x * sc, f.y * sc);
          }
          *reinterpret_cast<uint4 *>(sm + VT_OFF + off) = raw;
        }
      }
      // (c) P'[i][j] = Sc[i][j] * gamma^-(j+1) for j <= i (rows i = 16q + lane,
      //     lanes < 16; this warp's half of the columns j)
      ok = ok && mbar_wait(bar_sc, c & 1);
      if (!ok) s_abort = 1;
      if (ok) {
        tc_fence_after();
        const int i = q * 16 + lane;
        constexpr int CH = C / 2;
        const int j0 = half * CH;
        float x[CH];
        __syncwarp();
#pragma unroll
        for (int u = 0; u < CH / 16; ++u)
          tmem_ld16(tmem + lane_base + TM_SC + j0 + 16 * u, *reinterpret_cast<float(*)[16]>(x + 16 * u));
        tmem_wait_ld();
        if (lane < 16) {
#pragma unroll
          for (int j = 0; j < CH; ++j) x[j] = (j0 + j <= i) ? x[j] * ginv[j0 + j] : 0.f;
#pragma unroll
          for (int c16 = 0; c16 < CH / 8; ++c16) {
            const float *y = x + 8 * c16;
            *reinterpret_cast<uint4 *>(sm + P_OFF + sw128(i, j0 / 8 + c16)) =
                make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]), pack_bf16(y[6], y[7]));
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar_math);
      if (math_sync_or(s_abort != 0)) break;
      // (d) O = gamma^(i+1) * O^T[v][i]; store bf16 O * w; partial sum of O^2 per token
      ok = mbar_wait(bar_o, c & 1);
      if (!ok) s_abort = 1;
      if (math_sync_or(s_abort != 0)) break;
      tc_fence_after();
      const int col = h * DH + slice * VS + v;
      const float wv = p.norm_w ? p.norm_w[col] : 1.f;
      constexpr int CH = C / 2;  // this warp's half of the chunk's tokens
      const int i0 = half * CH;
      // staging buffer of this chunk: [v / 64][token][v % 64] bf16
      __nv_bfloat16 *ost = reinterpret_cast<__nv_bfloat16 *>(sm + OST_OFF + (c & 1) * 2 * OST_HALF +
                                                             (v >> 6) * OST_HALF) + (v & 63);
      float x[CH];
      __syncwarp();
#pragma unroll
      for (int u = 0; u < CH / 16; ++u)
        tmem_ld16(tmem + lane_base + TM_O + i0 + 16 * u, *reinterpret_cast<float(*)[16]>(x + 16 * u));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(bar_out);  // O^T is in registers: the next chunk's MMAs may overwrite it
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        x[i] *= gpow[i0 + i + 1];
        ost[(i0 + i) * 64] = __float2bfloat16(x[i] * wv);
        x[i] *= x[i];
      }
      // column sums of o^2 over the warp's 32 values of v: recursive halving
      // (lane l ends with token i0 + l), 31 shuffles for 32 tokens
      static_assert(C == 64, "the halving schedule below is written for 2 x 32 tokens");
#pragma unroll
      for (int o = 16, n = 16; o >= 1; o >>= 1, n >>= 1) {
        const bool up = lane & o;
#pragma unroll
        for (int j = 0; j < n; ++j) {
          const float send = up ? x[j] : x[j + n];
          const float keep = up ? x[j + n] : x[j];
          x[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      red[q * C + i0 + lane] = x[0];
      fence_proxy_async_smem();  // staged output before the TMA store reads it
      math_sync();
      if (mt == 0) {
        // the chunk's [64 tok x 128 v] output: two boxes; rows past T are clipped
        const uint8_t *src = sm + OST_OFF + (c & 1) * 2 * OST_HALF;
        tma_store_3d(&tm_out, src, col - v, t0, b);
        tma_store_3d(&tm_out, src + OST_HALF, col - v + 64, t0, b);
        bulk_commit();
        bulk_wait_read<1>();  // the other buffer (chunk c-1's store) is free for chunk c+1
      }
      if (p.sumsq && mt < L) {
        const float s2 = red[mt] + red[C + mt] + red[2 * C + mt] + red[3 * C + mt];
        p.sumsq[((size_t)b * p.T + t0 + mt) * (p.H * NSL) + h * NSL + slice] = s2;
      }
    }
    if (!STATE_ONLY && mt == 0) bulk_wait_all();  // the output stores have completed
    // final state: S[k][v] = S^T[v][k] (segment end states in the state pass,
    // else the last segment's state)
    const bool aborted = math_sync_or(s_abort != 0);
    const bool write_state = p.state_out && (STATE_ONLY || s == p.nseg - 1);
    // the last chunk's update MMAs (in the state pass: on its ring slot's barrier)
    auto wait_last_update = [&]() {
      if constexpr (STATE_ONLY) return mbar_wait(&bar_ups[(nch - 1) % SO_NS], ((nch - 1) / SO_NS) & 1);
      else return mbar_wait(bar_upd, (nch - 1) & 1);
    };
    if (!aborted && write_state) {
      bool ok = wait_last_update();
      if (!ok) s_abort = 1;
      if (!math_sync_or(s_abort != 0)) {
        tc_fence_after();
        const size_t sidx = STATE_ONLY ? (size_t)bsh : (size_t)(b * p.H + h);
        float *so = p.state_out + (sidx * DH) * DH + slice * VS + v;
#pragma unroll 1
        for (int k0 = half * (DH / 2); k0 < (half + 1) * (DH / 2); k0 += 16) {
          float x[16];
          __syncwarp();
          tmem_ld16(tmem + lane_base + TM_S + k0, x);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) so[(size_t)(k0 + j) * DH] = x[j];
        }
      }
    } else if (!aborted && nch > 0) {
      if (!wait_last_update()) s_abort = 1;  // last MMAs retired before TMEM is freed
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
}

// ---------------------------------------------------------------------------
// 128-token chunks.  Same CTA split (stream, segment, head, 128-wide value
// slice) and the same fp32 state S^T in TMEM, with a data flow that fits 128
// tokens into 227 KB of shared memory:
//   * the masked scores P live in TMEM as bf16 and are the A operand of the
//     intra-chunk MMA (tcgen05.mma with A in tensor memory), so P needs no
//     shared memory;
//   * the decay is folded into V' = diag(gamma^-(j+1)) V (j = position in the
//     chunk), scaled in place where V landed, which serves as both
//         O_c = diag(gamma^(i+1)) (Q S + mask(Q K^T) V')          (O: tokens x v)
//         S  <- gamma^L (S + K^T V')     (the gamma^L applied when the next
//                                         chunk reads S, or to the final state)
//     so no second scaled copy of V is kept (gamma^-128 <= 58 at gamma = 1 - 2^-5);
//   * the output is computed non-transposed (TMEM lane = token): each math
//     thread owns one token row and writes its 128 bytes into a swizzled
//     staging box in the bf16(S^T) region (K slices 1 and 3), stored with
//     TMA; rows written back to front (the backward's reversed passes) are
//     stored directly.
// Shared memory: Q, K [128 tok x 256 k], V' [128 tok x 128 v], bf16(S^T)
// [128 v x 256 k] = 224 KB.  TMEM: S^T 256 columns, scores/P 128, O 128.
// Per chunk: 16 MMAs O = Q . S (N=128), 16 scores (N=128), 8 state updates
// (N=256), 8 intra (A from TMEM): 48 MMAs per 128 tokens against 80 for two
// 64-token chunks.
// Schedule.  The state is the serial chain: chunk c's update, then chunk
// c+1's read-back of S (A), then its update again.  So the update is issued
// before the intra MMAs, and the math warps take chunk c+1's read-back
// before chunk c's output: iteration c of the math loop runs (A) of chunk c,
// (D1) of chunk c-1 (O out of TMEM into registers, which frees O for chunk
// c's O = Q S), (B) V' and (C) P of chunk c, then (D2) of chunk c-1 (staging
// and TMA store, once chunk c's O = Q S has read the staging slices).  Each
// operand has its own load barrier and is reloaded as soon as its last
// reader retired, so K and V' of the next chunk load while this chunk's
// output is written.
namespace c128 {
constexpr int C = 128;
constexpr int SLICE = 128 * 64 * 2;          // one [128 rows x 64] bf16 SW128 tile: 16 KB
constexpr int Q_OFF = 0;                     // 4 K-slices [128 tok x 64 k]
constexpr int K_OFF = Q_OFF + 4 * SLICE;     // 4 K-slices [128 tok x 64 k]
constexpr int V_OFF = K_OFF + 4 * SLICE;     // 2 boxes [128 tok x 64 v], scaled in place to V'
constexpr int SOP_OFF = V_OFF + 2 * SLICE;   // bf16(S^T): 4 K-slices [128 v x 64 k]
constexpr int TILE_BYTES = SOP_OFF + 4 * SLICE;  // 224 KB
constexpr int NBAR = 10;
// tail: barriers, TMEM slot (16 bytes), this CTA's 128 norm weights
constexpr size_t TAIL_BYTES = NBAR * 8 + 16 + VS * 4;
constexpr size_t SMEM = 1024 + TILE_BYTES + TAIL_BYTES;
static_assert(SMEM <= 232448, "227 KB of shared memory per CTA");
constexpr uint32_t TM_S = 0, TM_SC = 256, TM_O = 384, TM_COLS = 512;
constexpr int PARTS = NSL * 2;  // sum-of-squares parts per head: value slice x column half
}  // namespace c128

__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__global__ void __launch_bounds__(320, 1)
    retention_chunk128_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                              const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tm_out,
                              ChunkParams p) {
  // this kernel's layout (shadows the 64-token kernel's constants)
  constexpr int C = c128::C, SLICE = c128::SLICE, Q_OFF = c128::Q_OFF, K_OFF = c128::K_OFF, V_OFF = c128::V_OFF,
                SOP_OFF = c128::SOP_OFF, TILE_BYTES = c128::TILE_BYTES, NBAR = c128::NBAR, PARTS = c128::PARTS;
  constexpr uint32_t TM_S = c128::TM_S, TM_SC = c128::TM_SC, TM_O = c128::TM_O, TM_COLS = c128::TM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + TILE_BYTES);
  // loads landed: bar_q, bar_k, bar_v; MMAs retired: bar_sc (O = Q S and the
  // scores), bar_upd (state update), bar_o (intra, the chunk's last); math
  // warps done: bar_sop (bf16 S^T), bar_vs (V'), bar_math (P), bar_ofree (O read)
  uint64_t *bar_q = bars + 0, *bar_k = bars + 1, *bar_sc = bars + 2, *bar_sop = bars + 3, *bar_math = bars + 4,
           *bar_o = bars + 5, *bar_ofree = bars + 6, *bar_upd = bars + 7, *bar_v = bars + 8, *bar_vs = bars + 9;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NBAR);
  float *wsl = reinterpret_cast<float *>(bars + NBAR + 2);  // norm weights of this slice
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slice = blockIdx.x % NSL;
  const int bsh = blockIdx.x / NSL;  // ((b * nseg) + s) * H + h
  const int h = bsh % p.H, bs = bsh / p.H;
  const int b = bs / p.nseg, s = bs % p.nseg;
  const int d = p.H * DH;
  const int tb = s * p.seg_len;
  const int te = min(p.T, tb + p.seg_len);
  const int nch = (te - tb + C - 1) / C;
  const float lg = log2f(p.gamma[h]);

  if (threadIdx.x == 0) {
    s_abort = 0;
    mbar_init(bar_q, 1);
    mbar_init(bar_k, 1);
    mbar_init(bar_v, 1);
    mbar_init(bar_sc, 1);
    mbar_init(bar_upd, 1);
    mbar_init(bar_o, 1);
    mbar_init(bar_sop, MATH_THREADS);
    mbar_init(bar_vs, MATH_THREADS);
    mbar_init(bar_math, MATH_THREADS);
    mbar_init(bar_ofree, MATH_THREADS);
    fence_barrier_init();
    prefetch_tmap(&tmq);
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
    if (!p.out_reverse) prefetch_tmap(&tm_out);
  }
  if (threadIdx.x >= 64 && threadIdx.x < 64 + VS) {
    const int i = threadIdx.x - 64;
    wsl[i] = p.norm_w ? p.norm_w[h * DH + slice * VS + i] : 1.f;
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&]() {
    s_abort = 1;
    atomicOr(p.err, 1 << AF_ERR_TIMEOUT);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Each operand is reloaded as soon as its last reader of the previous
    // chunk retired: Q after the scores (issued after O = Q S), K after the
    // state update, V' after the intra MMAs (the MMAs run in that order).
    if (lane == 0) {
      int q_issued = 0, k_issued = 0, v_issued = 0;
      for (int c = 0; c < nch && !s_abort; ++c) {
        const int t0 = tb + c * C;
        if (c > 0 && !mbar_wait(bar_sc, (c - 1) & 1)) { fail(); break; }
        mbar_arrive_expect_tx(bar_q, 4 * SLICE);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) tma_load_3d(sm + Q_OFF + kk * SLICE, &tmq, bar_q, h * DH + kk * 64, t0, b);
        q_issued = c + 1;
        if (c > 0 && !mbar_wait(bar_upd, (c - 1) & 1)) { fail(); break; }
        mbar_arrive_expect_tx(bar_k, 4 * SLICE);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) tma_load_3d(sm + K_OFF + kk * SLICE, &tmk, bar_k, h * DH + kk * 64, t0, b);
        k_issued = c + 1;
        if (c > 0 && !mbar_wait(bar_o, (c - 1) & 1)) { fail(); break; }
        mbar_arrive_expect_tx(bar_v, 2 * SLICE);
#pragma unroll
        for (int vb = 0; vb < 2; ++vb)
          tma_load_3d(sm + V_OFF + vb * SLICE, &tmv, bar_v, h * DH + slice * VS + vb * 64, t0, b);
        v_issued = c + 1;
      }
      // loads still in flight land before the CTA may exit
      if (q_issued > 0 && !mbar_wait(bar_q, (q_issued - 1) & 1)) fail();
      if (k_issued > 0 && !mbar_wait(bar_k, (k_issued - 1) & 1)) fail();
      if (v_issued > 0 && !mbar_wait(bar_v, (v_issued - 1) & 1)) fail();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Per chunk, in this order: O = Q . S, the scores Q . K^T, the state
    // update S^T += V'^T K, then O += P . V'.  The update goes before the
    // intra MMAs because the next chunk's read-back of S is the longer chain.
    constexpr uint32_t id_nn = idesc_f32acc(kFmtBF16, 128, 128);                       // A, B K-major
    constexpr uint32_t id_intra = idesc_f32acc(kFmtBF16, 128, 128) | (1u << 16);       // A in TMEM, B MN-major
    constexpr uint32_t id_upd = idesc_f32acc(kFmtBF16, 128, 256) | (1u << 15) | (1u << 16);  // A, B MN-major
    for (int c = 0; c < nch; ++c) {
      // O = Q . S  (K = 256 keys) once Q landed, bf16(S) is written and the
      // previous chunk's O has been read out
      bool ok = mbar_wait(bar_q, c & 1) && mbar_wait(bar_sop, c & 1);
      if (ok && c > 0) ok = mbar_wait(bar_ofree, (c - 1) & 1);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || __any_sync(0xffffffffu, s_abort != 0)) { if (!ok && lane == 0) fail(); break; }
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t da = sdesc_k_sw128(sm + Q_OFF + kk * SLICE) + ((k * 32) >> 4);
            const uint64_t db = sdesc_k_sw128(sm + SOP_OFF + kk * SLICE) + ((k * 32) >> 4);
            umma_bf16(tmem + TM_O, da, db, id_nn, (kk | k) != 0);
          }
      }
      __syncwarp();
      // scores Q . K^T (K = 256 keys)
      ok = mbar_wait(bar_k, c & 1);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || __any_sync(0xffffffffu, s_abort != 0)) { if (!ok && lane == 0) fail(); break; }
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t da = sdesc_k_sw128(sm + Q_OFF + kk * SLICE) + ((k * 32) >> 4);
            const uint64_t db = sdesc_k_sw128(sm + K_OFF + kk * SLICE) + ((k * 32) >> 4);
            umma_bf16(tmem + TM_SC, da, db, id_nn, (kk | k) != 0);
          }
        umma_commit(bar_sc);
      }
      __syncwarp();
      // S^T += V'^T . K  (K = 128 tokens, N = 256 keys) once V' is scaled
      ok = mbar_wait(bar_vs, c & 1);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || __any_sync(0xffffffffu, s_abort != 0)) { if (!ok && lane == 0) fail(); break; }
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int kt = 0; kt < 8; ++kt) {
          const uint64_t da = sdesc_mn_sw128(sm + V_OFF + kt * 2048, SLICE);
          const uint64_t db = sdesc_mn_sw128(sm + K_OFF + kt * 2048, SLICE);
          umma_bf16(tmem + TM_S, da, db, id_upd, 1);
        }
        umma_commit(bar_upd);
      }
      __syncwarp();
      // O += P . V'  (K = 128 tokens; P's columns: j < 64 from TM_SC, j >= 64
      // from TM_SC + 64) once P is written
      ok = mbar_wait(bar_math, c & 1);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || __any_sync(0xffffffffu, s_abort != 0)) { if (!ok && lane == 0) fail(); break; }
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int kj = 0; kj < 8; ++kj) {
          const uint32_t pa = tmem + TM_SC + (kj < 4 ? 8 * kj : 64 + 8 * (kj - 4));
          const uint64_t db = sdesc_mn_sw128(sm + V_OFF + kj * 2048, SLICE);
          umma_bf16_ts(tmem + TM_O, pa, db, id_intra, 1);
        }
        umma_commit(bar_o);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ math warps
    // Iteration c does chunk c's (A) read-back of S, the first half of chunk
    // c-1's output (D1: O out of TMEM), chunk c's (B) V' and (C) P, then
    // the second half of chunk c-1's output (D2: staging and TMA store).
    // Chunk c-1's output thus waits behind chunk c's read-back, which is on
    // the state's critical path, and its staging slices are free again once
    // chunk c's O = Q S (which reads them as part of bf16(S^T)) retired.
    const int q = warp & 3;            // TMEM lane quadrant
    const int half = (warp - 2) >> 2;  // which half of the columns this warp takes
    const int mt = threadIdx.x - 64;   // 0..255
    const int row = q * 32 + lane;     // TMEM lane: value index (state) or token (scores, O)
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    // initial state S^T[v][k] = S[k][v]
    {
      const float *sin = p.state_in ? p.state_in + ((size_t)bsh * DH) * DH + slice * VS + row : nullptr;
#pragma unroll 1
      for (int k0 = half * (DH / 2); k0 < (half + 1) * (DH / 2); k0 += 16) {
        float x[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) x[j] = sin ? sin[(size_t)(k0 + j) * DH] : 0.f;
        __syncwarp();
        tmem_st16(tmem + lane_base + TM_S + k0, x);
      }
      tmem_wait_st();
    }
    const float gC = exp2f((float)C * lg);
    const float fo = exp2f((float)(row + 1) * lg);  // the output row's decay gamma^(i+1)
    // (B) scales the 16-byte chunks mt + 256 r of the two V boxes: token row
    // j = mt / 8 + 32 (r % 4), the same rows every chunk
    float vsc[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) vsc[r] = exp2f(-(float)(mt / 8 + 32 * r + 1) * lg);
    uint32_t ob[32];                                // chunk c-1's bf16 output row, (D1) -> (D2)
#pragma unroll 1
    for (int c = 0; c <= nch; ++c) {
      const bool cur = c < nch, prev = c > 0;
      if (cur) {
        // (A) S = gamma^C S_acc (the previous chunk's decay, deferred); bf16(S^T) -> shared memory
        bool ok = true;
        if (c > 0) ok = mbar_wait(bar_upd, (c - 1) & 1);
        if (!ok) s_abort = 1;
        if (math_sync_or(s_abort != 0)) break;
        tc_fence_after();
#pragma unroll 1
        for (int k0 = half * (DH / 2); k0 < (half + 1) * (DH / 2); k0 += 64) {
          float x[64];
          __syncwarp();
#pragma unroll
          for (int u = 0; u < 4; ++u)
            tmem_ld16(tmem + lane_base + TM_S + k0 + 16 * u, *reinterpret_cast<float(*)[16]>(x + 16 * u));
          tmem_wait_ld();
          if (c > 0) {
#pragma unroll
            for (int j = 0; j < 64; ++j) x[j] *= gC;
            __syncwarp();
#pragma unroll
            for (int u = 0; u < 4; ++u)
              tmem_st16(tmem + lane_base + TM_S + k0 + 16 * u, *reinterpret_cast<float(*)[16]>(x + 16 * u));
          }
          // the second K slice of each half holds chunk c-2's staged output:
          // written only once its TMA stores have read it
          if (k0 != half * (DH / 2) && c > 1 && !p.out_reverse) {
            if (mt == 0) bulk_wait_read<0>();
            math_sync();
          }
          uint8_t *slice_base = sm + SOP_OFF + (k0 >> 6) * SLICE;
#pragma unroll
          for (int c16 = 0; c16 < 8; ++c16) {
            const float *y = x + 8 * c16;
            *reinterpret_cast<uint4 *>(slice_base + sw128(row, c16)) =
                make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]), pack_bf16(y[6], y[7]));
          }
        }
        tmem_wait_st();
        fence_proxy_async_smem();  // bf16(S^T) (generic stores) before the MMAs that read it
        tc_fence_before();
        mbar_arrive(bar_sop);
      }
      if (prev) {
        // (D1) chunk c-1, token row i = row: O = gamma^(i+1) O_acc, bf16 O * w
        // into registers, and the partial sum of O^2 of this warp's 64 values
        const int tp = tb + (c - 1) * C;
        const int Lp = min(C, te - tp);
        bool ok = mbar_wait(bar_o, (c - 1) & 1);
        if (!ok) s_abort = 1;
        if (math_sync_or(s_abort != 0)) break;
        tc_fence_after();
        float x[64];
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 4; ++u)
          tmem_ld16(tmem + lane_base + TM_O + half * 64 + 16 * u, *reinterpret_cast<float(*)[16]>(x + 16 * u));
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(bar_ofree);  // O is in registers: chunk c's O = Q S may overwrite it
        const float *w = wsl + half * 64;
        float ss = 0.f;
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const float o0 = x[2 * jj] * fo, o1 = x[2 * jj + 1] * fo;
          ss = fmaf(o0, o0, ss);
          ss = fmaf(o1, o1, ss);
          ob[jj] = pack_bf16(o0 * w[2 * jj], o1 * w[2 * jj + 1]);
        }
        if (p.sumsq && row < Lp)
          p.sumsq[((size_t)b * p.T + tp + row) * (p.H * PARTS) + h * PARTS + slice * 2 + half] = ss;
      }
      if (cur) {
        // (B) V' = diag(gamma^-(j+1)) V in place
        bool ok = mbar_wait(bar_v, c & 1);
        if (!ok) s_abort = 1;
        if (ok) {
          static_assert(2 * SLICE / 16 == 8 * MATH_THREADS, "eight 16-byte chunks per math thread");
          uint4 raw[8];
#pragma unroll
          for (int r = 0; r < 8; ++r) raw[r] = *reinterpret_cast<const uint4 *>(sm + V_OFF + (mt + r * MATH_THREADS) * 16);
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            __nv_bfloat162 *e = reinterpret_cast<__nv_bfloat162 *>(&raw[r]);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              float2 f = __bfloat1622float2(e[u]);
              e[u] = __floats2bfloat162_rn(f.x * vsc[r & 3], f.y * vsc[r & 3]);
            }
            *reinterpret_cast<uint4 *>(sm + V_OFF + (mt + r * MATH_THREADS) * 16) = raw[r];
          }
        }
        fence_proxy_async_smem();  // V' (generic stores) before the MMAs that read it
        mbar_arrive(bar_vs);
        // (C) P = bf16(Q K^T masked to j <= i), written back into the scores'
        //     columns: this warp's 64 columns j become 32 packed columns at
        //     TM_SC + 64 * half, inside the range it read
        ok = ok && mbar_wait(bar_sc, c & 1);
        if (!ok) s_abort = 1;
        if (ok) {
          tc_fence_after();
          const int j0 = half * 64;
          float x[64];
          __syncwarp();
#pragma unroll
          for (int u = 0; u < 4; ++u)
            tmem_ld16(tmem + lane_base + TM_SC + j0 + 16 * u, *reinterpret_cast<float(*)[16]>(x + 16 * u));
          tmem_wait_ld();
          uint32_t pk[32];
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const int j = j0 + 2 * jj;
            pk[jj] = pack_bf16(j <= row ? x[2 * jj] : 0.f, j + 1 <= row ? x[2 * jj + 1] : 0.f);
          }
          __syncwarp();
          tmem_st16u(tmem + lane_base + TM_SC + j0, *reinterpret_cast<uint32_t(*)[16]>(pk));
          tmem_st16u(tmem + lane_base + TM_SC + j0 + 16, *reinterpret_cast<uint32_t(*)[16]>(pk + 16));
          tmem_wait_st();
        }
        tc_fence_before();
        mbar_arrive(bar_math);
        if (math_sync_or(s_abort != 0)) break;
      }
      if (prev) {
        // (D2) chunk c-1's rows (128 bytes each) to a 128-byte-swizzled
        //      staging box in K slices 1 and 3 of the bf16(S^T) region - free
        //      once chunk c's O = Q S retired, which the scores (waited in
        //      (C)) follow - and one thread stores both boxes [128 tok x 64 v]
        //      with TMA (rows past T are clipped by the tensor map); rows
        //      written back to front (the backward's reversed passes) are
        //      stored directly
        const int tp = tb + (c - 1) * C;
        const int Lp = min(C, te - tp);
        if (p.out_reverse) {
          if (row < Lp) {
            uint4 *dst = reinterpret_cast<uint4 *>(p.out + ((size_t)b * p.T + (p.T - 1 - (tp + row))) *
                                                               (p.ldo ? p.ldo : d) +
                                                   h * DH + slice * VS + half * 64);
#pragma unroll
            for (int c16 = 0; c16 < 8; ++c16)
              dst[c16] = make_uint4(ob[4 * c16], ob[4 * c16 + 1], ob[4 * c16 + 2], ob[4 * c16 + 3]);
          }
        } else {
          // after the last chunk no read-back waited for chunk c-2's stores
          if (!cur && c > 1) {
            if (mt == 0) bulk_wait_read<0>();
            math_sync();
          }
          uint8_t *box = sm + SOP_OFF + (2 * half + 1) * SLICE;
#pragma unroll
          for (int c16 = 0; c16 < 8; ++c16)
            *reinterpret_cast<uint4 *>(box + sw128(row, c16)) =
                make_uint4(ob[4 * c16], ob[4 * c16 + 1], ob[4 * c16 + 2], ob[4 * c16 + 3]);
          fence_proxy_async_smem();  // staged rows before the TMA stores read them
          math_sync();
          if (mt == 0) {
            const int col = h * DH + slice * VS;
            tma_store_3d(&tm_out, sm + SOP_OFF + SLICE, col, tp, b);
            tma_store_3d(&tm_out, sm + SOP_OFF + 3 * SLICE, col + 64, tp, b);
            bulk_commit();
          }
        }
      }
    }
    if (mt == 0) bulk_wait_all();  // the output stores have completed
    // final state S[k][v] = gamma^L_last (S_acc^T[v][k]) of the last segment
    const bool aborted = math_sync_or(s_abort != 0);
    const bool write_state = p.state_out && s == p.nseg - 1;
    if (!aborted && nch > 0) {
      bool ok = mbar_wait(bar_upd, (nch - 1) & 1);  // last MMAs retired before TMEM is read or freed
      if (ok) ok = mbar_wait(bar_o, (nch - 1) & 1);
      if (!ok) s_abort = 1;
      if (!math_sync_or(s_abort != 0) && write_state) {
        tc_fence_after();
        const float gl = exp2f((float)(te - (tb + (nch - 1) * C)) * lg);
        float *so = p.state_out + ((size_t)(b * p.H + h) * DH) * DH + slice * VS + row;
#pragma unroll 1
        for (int k0 = half * (DH / 2); k0 < (half + 1) * (DH / 2); k0 += 16) {
          float x[16];
          __syncwarp();
          tmem_ld16(tmem + lane_base + TM_S + k0, x);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) so[(size_t)(k0 + j) * DH] = x[j] * gl;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
}

// Turns segment end states dS_s ([B][nseg][H][DH*DH], zero-start) into the
// state before each segment, in place:  S_in[0] = state_in (or 0),
// S_in[s+1] = gamma^seg_len S_in[s] + dS_s.  One thread per 4 state entries.
__global__ void seg_scan_kernel(float4 *__restrict__ states, const float4 *__restrict__ state_in,
                                const float *__restrict__ gamma, int B, int nseg, int H, int seg_len) {
  constexpr int PER = DH * DH / 4;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)B * H * PER) return;
  const int e = (int)(idx % PER);
  const int bh = (int)(idx / PER);
  const int h = bh % H, b = bh / H;
  const float gl = exp2f((float)seg_len * log2f(gamma[h]));
  float4 run = state_in ? state_in[(size_t)bh * PER + e] : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < nseg; ++s) {
    float4 *q = states + (((size_t)b * nseg + s) * H + h) * PER + e;
    const float4 t = *q;
    *q = run;
    run = make_float4(gl * run.x + t.x, gl * run.y + t.y, gl * run.z + t.z, gl * run.w + t.w);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode3 = nullptr;

template <bool SO>
int launch_chunkwise(af_ctx *ctx, const CUtensorMap (&tms)[3], const CUtensorMap &tm_out, const ChunkParams &p,
                     cudaStream_t st, const char *fn) {
  static std::atomic<unsigned long long> attr_devices{0};
  if (int arc = af::smem_attr(ctx, reinterpret_cast<const void *>(retention_chunkwise_kernel<SO>), SMEM,
                              attr_devices, fn))
    return arc;
  retention_chunkwise_kernel<SO><<<p.B * p.nseg * p.H * NSL, 64 + MATH_THREADS, SMEM, st>>>(tms[0], tms[1], tms[2],
                                                                                            tm_out, p);
  return af::launched(ctx, fn);
}

int launch_chunk128(af_ctx *ctx, const CUtensorMap (&tms)[3], const CUtensorMap &tm_out, const ChunkParams &p,
                    cudaStream_t st, const char *fn) {
  static std::atomic<unsigned long long> attr_devices{0};
  if (int arc = af::smem_attr(ctx, reinterpret_cast<const void *>(retention_chunk128_kernel), c128::SMEM,
                              attr_devices, fn))
    return arc;
  retention_chunk128_kernel<<<p.B * p.nseg * p.H * NSL, 64 + MATH_THREADS, c128::SMEM, st>>>(tms[0], tms[1], tms[2],
                                                                                              tm_out, p);
  return af::launched(ctx, fn);
}

}  // namespace

namespace af {

ChunkPlan chunkwise_plan(int num_sms, int B, int T, int H, int nseg_req, int chunk) {
  const int Cc = chunk == c128::C ? c128::C : C;
  ChunkPlan pl{1, T > 0 ? ((T + Cc - 1) / Cc) * Cc : Cc, Cc};
  if (B <= 0 || T <= 0 || H <= 0) return pl;
  const int chunks = (T + Cc - 1) / Cc;
  const int ctas = B * H * NSL;
  int nseg = nseg_req > 0 ? nseg_req : num_sms / ctas;  // one CTA per SM
  if (nseg < 1) nseg = 1;
  if (nseg > chunks) nseg = chunks;
  const int per = (chunks + nseg - 1) / nseg;
  pl.seg_len = per * Cc;
  pl.nseg = (chunks + per - 1) / per;
  return pl;
}

size_t chunkwise_seg_state_bytes(int B, int H, const ChunkPlan &pl) {
  return pl.nseg > 1 ? (size_t)B * pl.nseg * H * DH * DH * sizeof(float) : 0;
}

// One operand of the chunkwise kernels: `d` columns (every head) of a bf16
// [B][T][ld] buffer starting at `base`, [64 col x rows tok] 128-byte-swizzled
// boxes.
static int encode_operand_map(CUtensorMap *tm, const void *base, int64_t ld, int B, int T, int d, int rows,
                              const char *fn) {
  if (!aligned16(base) || ld % 8 != 0 || ld < d)
    return fail(AF_ERR_ARG, "%s: q/k/v operands need 16-byte aligned bases and row strides (>= d) of 8k elements",
                fn);
  cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)T * ld * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)rows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode3(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AF_ERR_ARG, "%s: tensor map encode failed (%d)", fn, (int)r);
  return AF_OK;
}

static int encode_operand_maps(CUtensorMap (&tms)[3], const ChunkSrc &src, int B, int T, int d, int rows,
                               const char *fn) {
  int rc = encode_operand_map(&tms[0], src.q, src.ldq, B, T, d, rows, fn);
  if (!rc) rc = encode_operand_map(&tms[1], src.k, src.ldk, B, T, d, rows, fn);
  if (!rc) rc = encode_operand_map(&tms[2], src.v, src.ldv, B, T, d, rows, fn);
  return rc;
}

// Chunkwise retention over a bf16 QKV buffer [B*T][3d] (row stride 3d) in
// chunks of pl.chunk (64 or 128) tokens.  seg_states:
// chunkwise_seg_state_bytes() of scratch when pl.nseg > 1.  The segment state
// pass always walks 64-token tiles (it only accumulates K^T V); segment
// boundaries are multiples of pl.chunk.
int retention_chunkwise_bf16(af_ctx *ctx, const void *qkv, int B, int T, int H, const float *gamma,
                             const float *state_in, float *state_out, void *out, const float *norm_w, float *sumsq,
                             const ChunkPlan &pl, float *seg_states, cudaStream_t st, const char *fn, int64_t ldo,
                             bool out_reverse) {
  const int d = H * DH;
  const uint16_t *b16 = static_cast<const uint16_t *>(qkv);
  const ChunkSrc src{b16, b16 + d, b16 + 2 * d, 3 * (int64_t)d, 3 * (int64_t)d, 3 * (int64_t)d};
  return retention_chunkwise_bf16(ctx, src, B, T, H, gamma, state_in, state_out, out, norm_w, sumsq, pl, seg_states,
                                  st, fn, ldo, out_reverse);
}

int retention_chunkwise_bf16(af_ctx *ctx, const ChunkSrc &src, int B, int T, int H, const float *gamma,
                             const float *state_in, float *state_out, void *out, const float *norm_w, float *sumsq,
                             const ChunkPlan &pl, float *seg_states, cudaStream_t st, const char *fn, int64_t ldo,
                             bool out_reverse) {
  if (!g_encode3) {
    void *fp = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fp, cudaEnableDefault, &qr) != cudaSuccess || !fp)
      return fail(AF_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable", fn);
    g_encode3 = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fp);
  }
  if ((pl.chunk != C && pl.chunk != c128::C) || pl.nseg < 1 || pl.seg_len % pl.chunk != 0 ||
      (int64_t)pl.nseg * pl.seg_len < T || (int64_t)(pl.nseg - 1) * pl.seg_len >= T)
    return fail(AF_ERR_ARG, "%s: bad segment plan (%d x %d tokens in chunks of %d for T=%d)", fn, pl.nseg,
                pl.seg_len, pl.chunk, T);
  if (pl.nseg > 1 && !seg_states) return fail(AF_ERR_ARG, "%s: segment states scratch missing", fn);
  if ((int64_t)B * pl.nseg * H * NSL > 0x7fffffff) return fail(AF_ERR_ARG, "%s: grid too large", fn);
  if (!out) return fail(AF_ERR_ARG, "%s: output is NULL", fn);
  const int d = H * DH;
  if ((ldo != 0 || out_reverse) && (pl.chunk != c128::C || (ldo != 0 && (ldo < d || ldo % 8 != 0))))
    return fail(AF_ERR_ARG, "%s: an output stride or reversed rows need chunk 128 and a stride >= d, 8 | stride", fn);
  CUtensorMap tm[3], tm128[3];
  int rc = encode_operand_maps(tm, src, B, T, d, C, fn);
  if (rc) return rc;
  const bool big = pl.chunk == c128::C;
  if (big && (rc = encode_operand_maps(tm128, src, B, T, d, c128::C, fn))) return rc;
  // output [B][T][d] bf16 for the TMA stores: [64 tok x 64 v] plain boxes
  // (64-token kernel) or [128 tok x 64 v] 128-byte-swizzled boxes with row
  // stride ldo (128-token kernel); the T edge is clipped per stream
  CUtensorMap tm_out = tm[0];
  if (big && !out_reverse) {
    const cuuint64_t ld = (cuuint64_t)(ldo ? ldo : d);
    cuuint64_t odims[3] = {(cuuint64_t)d, (cuuint64_t)T, (cuuint64_t)B};
    cuuint64_t ostrides[2] = {ld * 2, (cuuint64_t)T * ld * 2};
    cuuint32_t obox[3] = {64, (cuuint32_t)c128::C, 1};
    cuuint32_t es[3] = {1, 1, 1};
    if (!aligned16(out)) return fail(AF_ERR_ARG, "%s: output must be 16-byte aligned", fn);
    CUresult r = g_encode3(&tm_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, out, odims, ostrides, obox, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(AF_ERR_ARG, "%s: output tensor map encode failed (%d)", fn, (int)r);
  }
  if (!big) {
    cuuint64_t odims[3] = {(cuuint64_t)d, (cuuint64_t)T, (cuuint64_t)B};
    cuuint64_t ostrides[2] = {(cuuint64_t)d * 2, (cuuint64_t)T * d * 2};
    cuuint32_t obox[3] = {64, (cuuint32_t)C, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = g_encode3(&tm_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, out, odims, ostrides, obox, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(AF_ERR_ARG, "%s: output tensor map encode failed (%d)", fn, (int)r);
  }
  ChunkParams p{B,       T,         H,       pl.nseg, pl.seg_len, gamma, state_in, state_out,
                reinterpret_cast<__nv_bfloat16 *>(out), norm_w, sumsq, ctx->dev_err, ldo, out_reverse ? 1 : 0};
  auto full_pass = [&](const ChunkParams &pp) {
    return big ? launch_chunk128(ctx, tm128, tm_out, pp, st, fn) : launch_chunkwise<false>(ctx, tm, tm_out, pp, st, fn);
  };
  if (pl.nseg == 1) {
    rc = full_pass(p);
    mark(ctx, "chunkwise", st);
    return rc;
  }
  // 1. segment end states from zero
  ChunkParams ps = p;
  ps.state_in = nullptr;
  ps.state_out = seg_states;
  ps.out = nullptr;
  ps.norm_w = nullptr;
  ps.sumsq = nullptr;
  rc = launch_chunkwise<true>(ctx, tm, tm[0], ps, st, fn);
  if (rc) return rc;
  mark(ctx, "chunk_state", st);
  // 2. states before each segment
  const int64_t n4 = (int64_t)B * H * (DH * DH / 4);
  seg_scan_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(reinterpret_cast<float4 *>(seg_states),
                                                                reinterpret_cast<const float4 *>(state_in), gamma, B,
                                                                pl.nseg, H, pl.seg_len);
  rc = launched(ctx, fn);
  if (rc) return rc;
  mark(ctx, "chunk_scan", st);
  // 3. the full pass from each segment's state
  p.state_in = seg_states;
  rc = full_pass(p);
  mark(ctx, "chunkwise", st);
  return rc;
}

int chunkwise_head_dim() { return DH; }
int chunkwise_parts(int chunk) { return chunk == c128::C ? c128::PARTS : NSL; }
int chunkwise_default_chunk(const af_ctx *ctx) { return ctx->chunk_len == c128::C ? c128::C : C; }

}  // namespace af
