// Tensor-core GEMM for sm_100a:  C[M][N] = A[M][K] . B[N][K]^T  (+ epilogue)
//
// Both operands K-major (the PyTorch (out, in) weight layout the reference
// uses, aceflow/nn/layers.py:19-20), accumulated in fp32 in TMEM.
//
// CTA = 6 warps, one 128 x BN output tile:
//   warp 0      TMA producer: A and B K-slices (128-byte rows, 128B swizzle)
//               into a STAGES-deep shared-memory ring, mbarrier complete_tx.
//   warp 1      allocates TMEM; lane 0 issues tcgen05.mma (M=128, N=BN) and
//               tcgen05.commit frees each ring slot when its MMAs retire.
//   warps 2-5   TF32x3 mode: split each fp32 slice in place into an exact
//               tf32 hi part and lo = x - hi; then the epilogue: tcgen05.ld of the 128 x BN
//               accumulator (warp w reads TMEM lanes 32*(w%4)..+31), fused
//               row scale / bias / residual / SwiGLU, vector stores.
//
// Modes (MODE template argument):
//   kBF16  : kind::f16 with bf16 operands (prefill projections).
//   kTF32S : fp32 operands split in shared memory: acc += A.B + A.B_lo + A_lo.B
//            with kind::tf32 - the three-term split of Ootomo & Yokota (2022)
//            that restores fp32 accuracy on the tensor cores.
//   kTF32P : the same products from operands split beforehand (hi and lo
//            arrays in global memory, four TMA loads per stage, no converter):
//            weights are split once at load time, activations by the kernel
//            that produces them.  The decode projections.
// Split-K: gridDim.z CTAs share one output tile over disjoint K ranges and
// add their fp32 partials with vector atomics (small-M GEMMs would otherwise
// leave most SMs idle while the weights stream).
//
// Every mbarrier wait is bounded; a timeout sets the context's device error
// word (AF_ERR_TIMEOUT) and the CTA drains and frees its TMEM.
#include "common.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>
#include <cstdlib>

namespace {

using namespace sm100;

struct GemmEpilogue {
  void *out;
  int64_t ldo;
  int out_bf16;
  const float *bias;       // [N] or null
  const float *row_parts;  // [M][nparts] sums of squares, or null
  int nparts;
  float inv_d, eps;
  const float *residual;   // [M][ldr] fp32 added to the result, or null
  int64_t ldr;
  int swiglu;              // columns in groups of 16 gate then 16 up -> N/2 outputs
  int vec_ok;              // out base 16-byte aligned and ldo a whole number of 16-byte units
  int atomic;              // split-K: add into out (bias/residual only from split 0)
  // Operand layout: A may be K-blocked, i.e. K/a_kb blocks [M][a_kb] stored
  // one after another (a_kb == K: plain).  Element (m, k) sits at row
  // (k / a_kb) * M + m, column k % a_kb of a (K/a_kb * M) x a_kb matrix.
  // row_parts likewise: blocks [M][parts_blk], element (m, p) at
  // (p / parts_blk) * M * parts_blk + m * parts_blk + p % parts_blk.
  int a_kb;
  int parts_blk;
  // Transposed store: element (row, n) goes to out[n * ldo + row] (a product
  // computed as W . X^T lands as X . W^T).  Plain fp32 only.
  int trans;
  // Split-K into separate partial buffers: split z stores (no atomics) at
  // out + z * split_stride; the consumer sums them.  0: one output.
  int64_t split_stride;
  int scale_residual;      // the row scale multiplies the residual too: (acc + r) * scale
  int res_vec;             // residual base 16-byte aligned and ldr a whole number of 16-byte units
  int pre_operand;         // 1 = A, 2 = B: loaded for the first ring slots before griddep_wait()
  // Tile written through shared memory by TMA (the ring, free once the
  // accumulator is complete), see store_tile_staged: 0 = no, kStageTrans =
  // transposed plain store [BN][128] (partial buffers: z = split), kStageAdd
  // = row-major reduce-add into out, 128-byte-swizzled 32-column boxes,
  // kStageTransAdd = transposed reduce-add of the [BN][128] box.
  int staged;
};
constexpr int kStageTrans = 1, kStageAdd = 2, kStageTransAdd = 3, kStageSwiGLU = 4, kStagePair = 5,
              kStagePairAdd = 6;  // pair kernel: TMA store / TMA reduce-add into out (in-place residual)

// v[e] += r[e] * rs for the 16 columns n..n+15 of one row (vector loads when
// the row segment is whole and aligned: each thread owns a different row, so
// scalar loads would touch 32 lines per warp instruction 16 times over).
__device__ __forceinline__ void add_residual16(float (&v)[16], const float *r, int n, int N, float rs, bool vec) {
  if (vec && n + 16 <= N) {
#pragma unroll
    for (int e = 0; e < 16; e += 4) {
      const float4 t = *reinterpret_cast<const float4 *>(r + e);
      v[e] += t.x * rs;
      v[e + 1] += t.y * rs;
      v[e + 2] += t.z * rs;
      v[e + 3] += t.w * rs;
    }
  } else {
    for (int e = 0; e < 16; ++e)
      if (n + e < N) v[e] += r[e] * rs;
  }
}

// 1 / rms of one row from its partial sums of squares.
__device__ __forceinline__ float row_scale(const GemmEpilogue &ep, int row, int M) {
  float sum = 0.f;
  const int pb = ep.parts_blk;
  for (int p0 = 0; p0 < ep.nparts; p0 += pb) {
    const float *q = ep.row_parts + (size_t)(p0 / pb) * M * pb + (size_t)row * pb;
    for (int p = 0; p < pb; ++p) sum += q[p];
  }
  return 1.0f / sqrtf(sum * ep.inv_d + ep.eps);
}

constexpr int kBF16 = 0, kTF32S = 1, kTF32P = 2;

// TMA producers.  One thread issuing a K slice's loads and waiting for a
// ring slot sustains about 3.5 M slices per second whatever their size (16 to
// 64 KB; measured on B200), so the GEMMs below may spread the slices over np
// producer threads: lane 0 of warp 0 and of the np - 1 warps after the six
// fixed ones (TMA, MMA, four epilogue warps).  Producer p issues the K slices
// g = p (mod np); every slot is still handed over by its own full / empty
// barriers, so the MMA thread consumes the slices in order.
constexpr int kMaxProducers = 4;
constexpr int kMaxGemmThreads = 32 * (5 + kMaxProducers);
__host__ __device__ __forceinline__ int gemm_threads(int np) { return 32 * (5 + np); }
__device__ __forceinline__ int num_producers() { return (int)(blockDim.x >> 5) - 5; }
__device__ __forceinline__ bool is_producer_warp(int warp) { return warp == 0 || warp >= 6; }
__device__ __forceinline__ int producer_id(int warp) { return warp == 0 ? 0 : warp - 5; }
// At most S producers take part: a producer waits for slot g % S with a
// parity wait, which is exact only while that slot's empty barrier is at most
// one phase behind, i.e. slice g - 2S has been consumed.  The producer's own
// previous slice g - np was issued after slice g - np - S was consumed, which
// covers g - 2S when np <= S.
__device__ __forceinline__ int active_producers(int S) {
  const int n = num_producers();
  return n < S ? n : S;
}
// first g >= from with g = p (mod np)
__device__ __forceinline__ int first_owned(int from, int p, int np) { return from + ((p - from % np) + np) % np; }
// Before the CTA exits, every load a producer issued has landed.  Normal
// end: its own slices among the last S (no later slice reuses their slots,
// so each parity wait is exact).  After an abort with one producer, the last
// S slices it issued; with several, other producers may have refilled those
// slots, so it waits a fixed 100 us for the copies in flight instead.
template <class Fail>
__device__ __forceinline__ void drain_producer(uint64_t *full, int S, int n, int issued, int p, int np, bool aborted,
                                               Fail &&fail) {
  if (!aborted || np == 1) {
    const int end = aborted ? issued : n;
    for (int g = first_owned(end - S < 0 ? 0 : end - S, p, np); g < end; g += np)
      if (!sm100::mbar_wait(&full[g % S], (g / S) & 1)) {
        fail();
        return;
      }
  } else {
    const uint64_t t0 = sm100::globaltimer();
    while (sm100::globaltimer() - t0 < 100000ull) {
    }
  }
}

template <int BN, int MODE, int KS = 1>
struct TileCfg {
  static constexpr bool TF32X3 = MODE != kBF16;
  static constexpr bool PRE = MODE == kTF32P;
  static constexpr int BM = 128;
  static constexpr int ELEM = TF32X3 ? 4 : 2;
  static constexpr int BK = KS * 128 / ELEM;     // K per stage: KS 128-byte swizzle rows (K slices)
  static constexpr int UK = 32 / ELEM;           // K per tcgen05.mma (32 bytes)
  static constexpr int A_SLICE = BM * 128, B_SLICE = BN * 128;
  static constexpr int A_BYTES = KS * A_SLICE;
  static constexpr int B_BYTES = KS * B_SLICE;
  static constexpr int RAW_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGE_BYTES = PRE ? 2 * RAW_BYTES : RAW_BYTES;  // one TMA ring stage
  // kTF32S: two split slots (lo parts) double-buffer the converter -> MMA
  // hand-off, so the TMA ring keeps its full depth for prefetch.
  static constexpr int LO_SLOTS = MODE == kTF32S ? 2 : 0;
  // ring depth: as many stages as the 227 KB opt-in limit holds (1 KB
  // alignment slack, the barrier block and 64 bytes of static shared memory
  // included) - small GEMMs are bound by the bytes in flight per SM
  static constexpr int SMEM_LIMIT = 227 * 1024 - 64;
  static constexpr int STAGES_FIT = (SMEM_LIMIT - 1024 - 256 - LO_SLOTS * RAW_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT < 12 ? STAGES_FIT : 12;
  // TF32x3: the hi.hi products go round-robin over NACC accumulators and the
  // small hi.lo + lo.hi terms into one more, so each fp32 accumulator sees
  // fewer tensor-core accumulation steps (its rounding error grows with them).
  static constexpr int NACC = TF32X3 ? (BN <= 64 ? 4 : BN < 256 ? 2 : 1) : 1;
  static constexpr int ACC_COLS = (NACC + (TF32X3 ? 1 : 0)) * BN;
  static constexpr int TMEM_COLS =
      ACC_COLS <= 32 ? 32 : ACC_COLS <= 64 ? 64 : ACC_COLS <= 128 ? 128 : ACC_COLS <= 256 ? 256 : 512;
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + (size_t)LO_SLOTS * RAW_BYTES + 256;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N");
  static_assert(KS == 1 || MODE == kBF16, "several K slices per stage: bf16 only");
  static_assert(ACC_COLS <= 512, "TMEM columns");
  static_assert(STAGES >= 2, "pipeline depth");
  static_assert(1024 + (size_t)STAGES * STAGE_BYTES + (size_t)LO_SLOTS * RAW_BYTES + 256 <= (size_t)SMEM_LIMIT,
                "shared memory");
};

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// Epilogue of one 128 x BN tile for the calling warp's 32 rows: reads the
// accumulator through load16 (warp-collective TMEM loads; wait_ld() waits for
// the loads issued so far, so up to 64 columns are in flight per round trip),
// applies row scale, bias, residual or SwiGLU, and stores (or atomically adds,
// for split-K).
template <int BN, class Load16, class WaitLd>
__device__ __forceinline__ void store_tile(const GemmEpilogue &ep, Load16 &&load16, WaitLd &&wait_ld, int row,
                                           bool row_ok, int n0, int N, bool ok, float scale, bool first) {
  if (ep.swiglu && !ep.trans) {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 64) {
      float gu[4][16];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c0 + 16 * u < BN) load16(c0 + 16 * u, gu[u]);
      wait_ld();
#pragma unroll
      for (int pr = 0; pr < 2; ++pr) {
        const int c = c0 + 32 * pr;
        if (c >= BN) break;
        const float(&g)[16] = gu[2 * pr];
        const float(&u)[16] = gu[2 * pr + 1];
        const int nout = (n0 + c) / 2;  // first output column of this group
        if (ok && row_ok && n0 + c + 32 <= N) {
          float hh[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float gg = g[e] * scale, uu = u[e] * scale;
            hh[e] = gg / (1.0f + expf(-gg)) * uu;
          }
          if (ep.out_bf16) {
            __nv_bfloat16 *o = reinterpret_cast<__nv_bfloat16 *>(ep.out) + (size_t)row * ep.ldo + nout;
            uint32_t pk[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              __nv_bfloat162 b2 = __floats2bfloat162_rn(hh[2 * e], hh[2 * e + 1]);
              pk[e] = *reinterpret_cast<uint32_t *>(&b2);
            }
            reinterpret_cast<uint4 *>(o)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            reinterpret_cast<uint4 *>(o)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          } else {
            float *o = reinterpret_cast<float *>(ep.out) + (size_t)row * ep.ldo + nout;
#pragma unroll
            for (int e = 0; e < 16; e += 4)
              *reinterpret_cast<float4 *>(o + e) = make_float4(hh[e], hh[e + 1], hh[e + 2], hh[e + 3]);
          }
        }
      }
    }
  } else if (ep.trans) {
    // Transposed tile: `row` is an output column (a weight row), the 16
    // accumulator columns of a chunk are 16 output rows n..n+15 (batch rows).
    // Lanes hold consecutive `row`s, so every store or atomic of one e is one
    // coalesced 128-byte line.
    const int lane = threadIdx.x & 31;
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      float v[16];
      load16(c, v);
      wait_ld();
      const int n = n0 + c;
      if (ep.swiglu) {
        // rows in groups of 16 gate then 16 up: lane l < 16 takes the up value
        // of its hidden unit from lane l + 16
        float u[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) u[e] = __shfl_down_sync(0xffffffffu, v[e], 16);
        if (!ok || !row_ok || n >= N || lane >= 16) continue;
        const int j = ((row - lane) >> 1) + lane;  // hidden unit: 16 per 32-row group
        __nv_bfloat16 *o = reinterpret_cast<__nv_bfloat16 *>(ep.out) + j;
#pragma unroll
        for (int e = 0; e < 16; ++e)
          if (n + e < N) {
            const float gg = v[e];
            o[(size_t)(n + e) * ep.ldo] = __float2bfloat16(gg / (1.0f + expf(-gg)) * u[e]);
          }
        continue;
      }
      // per-column 1/rms (output rows are streams): lane l computes column n + (l & 15)
      float my_scale = 1.f;
      if (ep.row_parts && n + (lane & 15) < N) my_scale = row_scale(ep, n + (lane & 15), N);
      float cs[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) cs[e] = __shfl_sync(0xffffffffu, my_scale, e);
      if (!ok || !row_ok || n >= N) continue;
      float *o = reinterpret_cast<float *>(ep.out) + (size_t)blockIdx.z * ep.split_stride + row;
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (n + e < N) {
          const float val = v[e] * cs[e];
          if (ep.atomic) atomicAdd(o + (size_t)(n + e) * ep.ldo, val);
          else o[(size_t)(n + e) * ep.ldo] = val;
        }
    }
  } else {
    // one 16-column chunk: scale, bias, residual, store / atomic add
    auto emit16 = [&](float(&v)[16], int n) {
      if (!ok || !row_ok || n >= N) return;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        v[e] *= scale;
        if (first && ep.bias && n + e < N) v[e] += ep.bias[n + e];
      }
      if (ep.atomic) {
        if (first && ep.residual) add_residual16(v, ep.residual + (size_t)row * ep.ldr + n, n, N, 1.f, ep.res_vec);
        float *o = reinterpret_cast<float *>(ep.out) + (size_t)row * ep.ldo + n;
        if (n + 16 <= N && ep.vec_ok) {
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            atomicAdd(reinterpret_cast<float4 *>(o + e), make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]));
        } else {
          for (int e = 0; e < 16 && n + e < N; ++e) atomicAdd(o + e, v[e]);
        }
        return;
      }
      if (ep.residual)
        add_residual16(v, ep.residual + (size_t)row * ep.ldr + n, n, N, ep.scale_residual ? scale : 1.f, ep.res_vec);
      if (ep.out_bf16) {
        __nv_bfloat16 *o = reinterpret_cast<__nv_bfloat16 *>(ep.out) + (size_t)row * ep.ldo + n;
        if (n + 16 <= N && ep.vec_ok) {
          uint32_t pk[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
            pk[e] = *reinterpret_cast<uint32_t *>(&b2);
          }
          reinterpret_cast<uint4 *>(o)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          reinterpret_cast<uint4 *>(o)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        } else {
          for (int e = 0; e < 16 && n + e < N; ++e) o[e] = __float2bfloat16(v[e]);
        }
      } else {
        float *o = reinterpret_cast<float *>(ep.out) + (size_t)row * ep.ldo + n;
        if (n + 16 <= N && ep.vec_ok) {
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            *reinterpret_cast<float4 *>(o + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
        } else {
          for (int e = 0; e < 16 && n + e < N; ++e) o[e] = v[e];
        }
      }
    };
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 64) {
      float vv[4][16];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c0 + 16 * u < BN) load16(c0 + 16 * u, vv[u]);
      wait_ld();
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c0 + 16 * u < BN) emit16(vv[u], n0 + c0 + 16 * u);
    }
  }
}

// Bulk tensor stores from shared memory (bulk async-group completion).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
// Element-wise f32 add of a shared-memory box into global memory (performed
// at L2; replaces per-thread atomics of a split-K or accumulating epilogue).
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *map, const void *src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_but_one() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_commit_wait_all() {
  asm volatile("cp.async.bulk.commit_group;\n\tcp.async.bulk.wait_group 0;" ::: "memory");
}
// Barrier over the four epilogue warps (2..5).
__device__ __forceinline__ void epilogue_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Epilogue through shared memory: the calling warp's 32 rows of a 128 x BN
// accumulator tile are written to `stg` (the free TMA ring) and one thread
// stores the tile with TMA.
//   kStageTrans: element (row, n) at stg[n * 128 + row] (lanes: consecutive
//     rows, conflict-free); one 3-D store {row, n, split} of the [BN][128]
//     box: the transposed product, or its split's partial buffer.
//   kStageTransAdd: the same box with the per-column 1/rms (columns are
//     streams) applied, added into out by one 2-D TMA reduce-add {row, n}.
//   kStageSwiGLU: transposed SwiGLU (rows in groups of 16 gate then 16 up):
//     h = silu(gate) * up as bf16 at [n][hidden], hidden = m0/2 + 0..63, one
//     2-D store of the [BN][64] box.
//   kStageAdd: 32-column boxes [128 rows][32 cols] one after another, each
//     128-byte swizzled (16-byte chunk c of row r at chunk c ^ (r & 7), so the
//     lanes' float4 writes spread over the banks); the row scale is applied
//     and each box is added into out by a TMA reduce-add.
// Rows and columns past the output are dropped by the tensor map bounds.
template <int BN, class Load16, class WaitLd>
__device__ __forceinline__ void store_tile_staged(const GemmEpilogue &ep, const CUtensorMap *tmO, Load16 &&load16,
                                                  WaitLd &&wait_ld, float *stg, int r, int m0, int n0, int z,
                                                  int N, bool ok, float scale) {
  if (ep.staged == kStageSwiGLU) {
    const int lane = threadIdx.x & 31;
    __nv_bfloat16 *hb = reinterpret_cast<__nv_bfloat16 *>(stg) + (r - lane) / 2 + lane;  // hidden unit of lane < 16
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      float v[16];
      load16(c, v);
      wait_ld();
      float u[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) u[e] = __shfl_down_sync(0xffffffffu, v[e], 16);
      if (lane < 16) {
#pragma unroll
        for (int e = 0; e < 16; ++e) hb[(c + e) * 64] = __float2bfloat16(v[e] / (1.0f + expf(-v[e])) * u[e]);
      }
    }
  } else if (ep.staged == kStageTrans || ep.staged == kStageTransAdd) {
    const int lane = threadIdx.x & 31;
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      float v[16];
      load16(c, v);
      wait_ld();
      if (ep.staged == kStageTransAdd && ep.row_parts) {
        // per-column 1/rms: lane l computes column n0 + c + (l & 15)
        const int col = n0 + c + (lane & 15);
        const float my_scale = col < N ? row_scale(ep, col, N) : 1.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] *= __shfl_sync(0xffffffffu, my_scale, e);
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) stg[(c + e) * 128 + r] = v[e];
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      float v[16];
      load16(c, v);
      wait_ld();
      uint8_t *box = reinterpret_cast<uint8_t *>(stg) + (c / 32) * (128 * 128) + r * 128;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int chunk = ((c % 32) / 4 + u) ^ (r & 7);
        *reinterpret_cast<float4 *>(box + chunk * 16) =
            make_float4(v[4 * u] * scale, v[4 * u + 1] * scale, v[4 * u + 2] * scale, v[4 * u + 3] * scale);
      }
    }
  }
  fence_proxy_async_smem();  // generic-proxy writes before the bulk copy reads them
  epilogue_sync();
  if (threadIdx.x == 64 && ok) {
    if (ep.staged == kStageTrans) {
      tma_store_3d(tmO, stg, m0, n0, z);
    } else if (ep.staged == kStageTransAdd) {
      tma_reduce_add_2d(tmO, stg, m0, n0);
    } else if (ep.staged == kStageSwiGLU) {
      tma_store_2d(tmO, stg, m0 / 2, n0);
    } else {
#pragma unroll 1
      for (int j = 0; j < BN / 32; ++j)
        tma_reduce_add_2d(tmO, reinterpret_cast<uint8_t *>(stg) + j * (128 * 128), n0 + 32 * j, m0);
    }
    bulk_commit_wait_all();  // shared memory is read (and the writes issued) before the CTA exits
  }
}

template <int BN, int MODE, int KS>
__global__ void __launch_bounds__(kMaxGemmThreads, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                     const __grid_constant__ CUtensorMap tmO, int M, int N, int K, GemmEpilogue ep, int *err) {
  using C = TileCfg<BN, MODE, KS>;
  constexpr bool TF32X3 = C::TF32X3;
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *lo_base = smem + (size_t)S * C::STAGE_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(lo_base + (size_t)C::LO_SLOTS * C::RAW_BYTES);
  uint64_t *full = bars;            // [S]  TMA landed
  uint64_t *empty = bars + S;       // [S]  MMAs reading the stage retired
  uint64_t *conv = bars + 2 * S;    // [2]  split slot written (TF32x3)
  uint64_t *lofree = bars + 2 * S + 2;  // [2]  MMAs reading the split slot retired
  uint64_t *accum = bars + 2 * S + 4;   // accumulators complete
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 5);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * C::BM, n0 = blockIdx.x * BN;
  const int nk_all = (K + C::BK - 1) / C::BK;
  // split-K: this CTA's K slices are [kb_base, kb_base + nk)
  const int kb_base = (int)(((int64_t)blockIdx.z * nk_all) / gridDim.z);
  const int nk = (int)(((int64_t)(blockIdx.z + 1) * nk_all) / gridDim.z) - kb_base;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&conv[j], 128);
      mbar_init(&lofree[j], 1);
    }
    mbar_init(accum, 1);
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if constexpr (C::PRE) {
      prefetch_tmap(&tmA2);
      prefetch_tmap(&tmB2);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_launch();

  auto stage_a = [&](int i) { return smem + (size_t)i * C::STAGE_BYTES; };
  auto stage_b = [&](int i) { return smem + (size_t)i * C::STAGE_BYTES + C::A_BYTES; };
  // lo parts: the stage's second half (kTF32P) or a split slot (kTF32S)
  auto lo_a = [&](int i, int j) {
    return C::PRE ? smem + (size_t)i * C::STAGE_BYTES + C::RAW_BYTES : lo_base + (size_t)j * C::RAW_BYTES;
  };
  auto lo_b = [&](int i, int j) { return lo_a(i, j) + C::A_BYTES; };
  auto fail = [&]() {
    s_abort = 1;
    atomicOr(err, 1 << AF_ERR_TIMEOUT);
  };

  if (is_producer_warp(warp)) {
    if (lane == 0 && producer_id(warp) < active_producers(S)) {
      // producer p issues the K slices kb = p (mod np)
      const int np = active_producers(S), p = producer_id(warp);
      auto load_a = [&](int i, int kx) {
        const int ka = kx % ep.a_kb, ma = m0 + (kx / ep.a_kb) * M;  // K-blocked A
        if constexpr (KS > 1) {  // KS slices in one 3-D copy (K blocks are multiples of BK)
          tma_load_3d(stage_a(i), &tmA, &full[i], 0, ma, ka / 64);
        } else {
          tma_load_2d(stage_a(i), &tmA, &full[i], ka, ma);
          if constexpr (C::PRE) tma_load_2d(lo_a(i, 0), &tmA2, &full[i], ka, ma);
        }
      };
      auto load_b = [&](int i, int kx) {
        if constexpr (KS > 1) {
          tma_load_3d(stage_b(i), &tmB, &full[i], 0, n0, kx / 64);
        } else {
          tma_load_2d(stage_b(i), &tmB, &full[i], kx, n0);
          if constexpr (C::PRE) tma_load_2d(lo_b(i, 0), &tmB2, &full[i], kx, n0);
        }
      };
      // The operand that does not depend on the previous kernel (the
      // weights) fills the free ring slots before the dependency wait; the
      // other one follows it (always issued, so every slot's barrier completes).
      const int pre = ep.pre_operand ? (nk < S ? nk : S) : 0;
      for (int kb = p; kb < pre; kb += np) {
        mbar_arrive_expect_tx(&full[kb], C::STAGE_BYTES);
        if (ep.pre_operand == 1) load_a(kb, (kb_base + kb) * C::BK);
        else load_b(kb, (kb_base + kb) * C::BK);
      }
      griddep_wait();
      for (int kb = p; kb < pre; kb += np) {
        if (ep.pre_operand == 1) load_b(kb, (kb_base + kb) * C::BK);
        else load_a(kb, (kb_base + kb) * C::BK);
      }
      int issued = pre;  // K slices [0, issued) are this producer's share issued so far
      for (int kb = first_owned(pre, p, np); kb < nk && !s_abort; kb += np) {
        const int i = kb % S;
        const uint32_t ph = (kb / S) & 1;
        if (!mbar_wait(&empty[i], ph ^ 1)) { fail(); break; }
        const int kx = (kb_base + kb) * C::BK;
        mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
        load_a(i, kx);
        load_b(i, kx);
        issued = kb + 1;
      }
      drain_producer(full, S, nk, issued, p, np, s_abort != 0, fail);
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = idesc_f32acc(TF32X3 ? kFmtTF32 : kFmtBF16, C::BM, BN);
    for (int kb = 0; kb < nk; ++kb) {
      const int i = kb % S, j = kb & 1;
      const bool ok = __all_sync(0xffffffffu, MODE == kTF32S ? mbar_wait(&conv[j], (kb >> 1) & 1)
                                                             : mbar_wait(&full[i], (kb / S) & 1));
      if (!ok) {
        if (lane == 0) fail();
        break;
      }
      if (__any_sync(0xffffffffu, s_abort != 0)) break;
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int sl = 0; sl < KS; ++sl) {
          const uint64_t da = sdesc_k_sw128(stage_a(i) + sl * C::A_SLICE),
                         db = sdesc_k_sw128(stage_b(i) + sl * C::B_SLICE);
#pragma unroll
          for (int k = 0; k < 128 / 32; ++k) {
            const uint64_t off = (uint64_t)(k * 32) >> 4;  // 32 bytes along K inside the swizzle row
            if constexpr (TF32X3) {
              const uint64_t dal = sdesc_k_sw128(lo_a(i, j)), dbl = sdesc_k_sw128(lo_b(i, j));
              const uint32_t acc = tmem + (uint32_t)((kb % C::NACC) * BN);
              const uint32_t corr = tmem + (uint32_t)(C::NACC * BN);
              umma_tf32(acc, da + off, db + off, idesc, (kb >= C::NACC || k > 0) ? 1u : 0u);
              umma_tf32(corr, da + off, dbl + off, idesc, (kb > 0 || k > 0) ? 1u : 0u);
              umma_tf32(corr, dal + off, db + off, idesc, 1);
            } else {
              umma_bf16(tmem, da + off, db + off, idesc, (kb | sl | k) != 0);
            }
          }
        }
        umma_commit(&empty[i]);
        if constexpr (MODE == kTF32S) umma_commit(&lofree[j]);
      }
      __syncwarp();
    }
    if (lane == 0) umma_commit(accum);
    __syncwarp();
  } else {
    // ---- warps 2..5
    const int t = threadIdx.x - 64;  // 0..127
    if constexpr (MODE == kTF32S) {
      for (int kb = 0; kb < nk; ++kb) {
        const int i = kb % S, j = kb & 1;
        if (!mbar_wait(&full[i], (kb / S) & 1) || !mbar_wait(&lofree[j], ((kb >> 1) & 1) ^ 1)) {
          fail();
          break;
        }
        // x = hi + lo exactly: hi = x with the low 13 mantissa bits cleared
        // (an exact tf32 value, written back in place), lo = x - hi.
        float4 *ra = reinterpret_cast<float4 *>(stage_a(i));
        float4 *la = reinterpret_cast<float4 *>(lo_a(i, j));
#pragma unroll 4
        for (int e = t; e < C::RAW_BYTES / 16; e += 128) {  // A then B, contiguous in both buffers
          const float4 v = ra[e];
          const float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
          ra[e] = h;
          la[e] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
        }
        fence_proxy_async_smem();
        mbar_arrive(&conv[j]);
      }
    }
    const bool ok = mbar_wait(accum, 0);
    if (!ok) fail();
    tc_fence_after();
    griddep_wait();  // the epilogue reads row sums / residual and writes out
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = m0 + q * 32 + lane;
    const bool row_ok = row < M;
    float scale = 1.f;
    if (ep.row_parts && row_ok && !ep.trans) scale = row_scale(ep, row, M);  // transposed: per column
    const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16);
    const int nacc = nk < C::NACC ? nk : C::NACC;  // accumulators that received products
    // Sum of the accumulators for 16 columns starting at `col` (warp-collective).
    auto load16 = [&](int col, float (&v)[16]) {
      __syncwarp();
      tmem_ld16(tbase + col, v);
      if constexpr (TF32X3) {  // sums the accumulators (waits inside)
        float w[16];
        tmem_ld16(tbase + (uint32_t)(C::NACC * BN) + col, w);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] += w[e];
#pragma unroll 1
        for (int a = 1; a < nacc; ++a) {
          __syncwarp();
          tmem_ld16(tbase + (uint32_t)(a * BN) + col, w);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] += w[e];
        }
      }
    };
    auto wait_ld = [&]() {
      if constexpr (!TF32X3) tmem_wait_ld();
    };
    if (ep.staged)
      store_tile_staged<BN>(ep, &tmO, load16, wait_ld, reinterpret_cast<float *>(smem), q * 32 + lane, m0, n0,
                            blockIdx.z, N, ok && !s_abort, scale);
    else
      store_tile<BN>(ep, load16, wait_ld, row, row_ok, n0, N, ok, scale, blockIdx.z == 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// Persistent bf16 GEMM for large M (prefill): one CTA per SM walks the
// output tiles (row-band major, so consecutive CTAs share A rows), with two
// TMEM accumulators so the epilogue of one tile overlaps the MMAs of the
// next.  The TMA ring and its phases run continuously across tiles.
template <int BN>
__global__ void __launch_bounds__(kMaxGemmThreads, 1)
    umma_gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                int M, int N, int K, GemmEpilogue ep, int *err) {
  using C = TileCfg<BN, kBF16>;
  constexpr int S = C::STAGES;
  constexpr uint32_t TM_COLS = 2 * BN;  // two accumulators
  static_assert(2 * BN <= 512 && (BN & (BN - 1)) == 0, "two accumulators must fit TMEM");
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (size_t)S * C::STAGE_BYTES);
  uint64_t *full = bars, *empty = bars + S;
  uint64_t *accf = bars + 2 * S;      // [2] accumulator b holds a finished tile
  uint64_t *acce = bars + 2 * S + 2;  // [2] accumulator b has been read out
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 4);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (N + BN - 1) / BN, m_tiles = (M + C::BM - 1) / C::BM;
  const int total = n_tiles * m_tiles;
  const int nk = (K + C::BK - 1) / C::BK;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 128);
    }
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto stage_a = [&](int i) { return smem + (size_t)i * C::STAGE_BYTES; };
  auto stage_b = [&](int i) { return smem + (size_t)i * C::STAGE_BYTES + C::A_BYTES; };
  auto fail = [&]() {
    s_abort = 1;
    atomicOr(err, 1 << AF_ERR_TIMEOUT);
  };

  if (is_producer_warp(warp)) {
    if (lane == 0 && producer_id(warp) < active_producers(S)) {
      const int np = active_producers(S), p = producer_id(warp);  // producer p: slices g = p (mod np)
      const int my_tiles = blockIdx.x < total ? (total - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
      const int g_end = my_tiles * nk;  // K slices of this CTA over all its tiles
      int issued = 0;
      for (int g = p; g < g_end && !s_abort; g += np) {
        const int t = (int)blockIdx.x + (g / nk) * (int)gridDim.x, kb = g % nk;
        const int m0 = (t / n_tiles) * C::BM, n0 = (t % n_tiles) * BN;
        const int i = g % S;
        if (!mbar_wait(&empty[i], ((g / S) & 1) ^ 1)) { fail(); break; }
        mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
        const int kx = kb * C::BK;
        tma_load_2d(stage_a(i), &tmA, &full[i], kx % ep.a_kb, m0 + (kx / ep.a_kb) * M);
        tma_load_2d(stage_b(i), &tmB, &full[i], kb * C::BK, n0);
        issued = g + 1;
      }
      drain_producer(full, S, g_end, issued, p, np, s_abort != 0, fail);
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = idesc_f32acc(kFmtBF16, C::BM, BN);
    int g = 0, it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
      const int b = it & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&acce[b], ((it >> 1) & 1) ^ 1));
      if (!ok) break;
      tc_fence_after();
      const uint32_t acc = tmem + (uint32_t)(b * BN);
      for (int kb = 0; kb < nk; ++kb, ++g) {
        const int i = g % S;
        ok = __all_sync(0xffffffffu, mbar_wait(&full[i], (g / S) & 1));
        if (!ok || __any_sync(0xffffffffu, s_abort != 0)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint64_t da = sdesc_k_sw128(stage_a(i)), db = sdesc_k_sw128(stage_b(i));
#pragma unroll
          for (int k = 0; k < C::BK / C::UK; ++k) {
            const uint64_t off = (uint64_t)(k * 32) >> 4;
            umma_bf16(acc, da + off, db + off, idesc, (kb | k) != 0);
          }
          umma_commit(&empty[i]);
        }
        __syncwarp();
      }
      if (lane == 0 && ok) umma_commit(&accf[b]);
      __syncwarp();
    }
    if (!ok && lane == 0) fail();
  } else {
    const int q = warp & 3;
    int it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
      const int b = it & 1;
      const bool ok = mbar_wait(&accf[b], (it >> 1) & 1);
      if (!ok) {
        fail();
        break;
      }
      tc_fence_after();
      const int m0 = (t / n_tiles) * C::BM, n0 = (t % n_tiles) * BN;
      const int row = m0 + q * 32 + lane;
      const bool row_ok = row < M;
      float scale = 1.f;
      if (ep.row_parts && row_ok && !ep.trans) scale = row_scale(ep, row, M);  // transposed: per column
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN);
      auto load16 = [&](int col, float (&v)[16]) {
        __syncwarp();
        tmem_ld16(tbase + col, v);
      };
      auto wait_ld = [&]() { tmem_wait_ld(); };
      store_tile<BN>(ep, load16, wait_ld, row, row_ok, n0, N, true, scale, true);
      tc_fence_before();
      mbar_arrive(&acce[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
}

// Persistent bf16 GEMM on CTA pairs (cta_group::2): a cluster of two CTAs
// on the two SMs of a TPC computes 256 x 256 tiles.  Each CTA loads its own
// 128 rows of A and 128 rows of B per K slice (32 KB per stage, so a stage
// carries a third fewer bytes per MMA flop than a 128 x 256 tile on one SM);
// the rank-0 CTA issues the MMAs, whose accumulator rows land in each CTA's
// own TMEM (two 256-column buffers: one tile's epilogue overlaps the next
// tile's MMAs).  Barriers:
//   full[i]  (rank 0)  both CTAs' TMA bytes of stage i landed
//   empty[i] (each)    the MMAs reading stage i retired (commit to both CTAs)
//   accf[b]  (each)    accumulator b holds a finished tile (commit to both)
//   acce[b]  (rank 0)  both CTAs' epilogues (256 threads) read accumulator b
//
// A ring stage holds KS consecutive 64-element K slices (KS = 2 when K allows:
// one 3-D TMA copy per operand and stage).  Each stage costs the MMA thread a
// barrier wait and a commit per CTA, about 200 ns measured on B200 against
// 70 ns per 256 x 256 x 16 MMA, so two slices per stage (8 MMAs) amortise
// them twice as well as one.
template <int KS>
struct PairCfg {
  static constexpr int BM = 256, BN = 256, HALF = 128, BK = 64 * KS;  // K elements per stage
  static constexpr int SLICE = HALF * 128;                            // one K slice of 128 rows
  static constexpr int A_BYTES = KS * SLICE, B_BYTES = KS * SLICE, STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SMEM_LIMIT = 227 * 1024 - 64;
  static constexpr int STAGES = (SMEM_LIMIT - 1024 - 256) / STAGE_BYTES;
  // Epilogue staging (output through TMA stores), when it fits beside the
  // ring: 8 KB per epilogue warp.
  static constexpr int STG_WARP = 8192;
  static constexpr int STG_BYTES =
      1024 + STAGES * STAGE_BYTES + 1024 + 4 * STG_WARP <= SMEM_LIMIT ? 4 * STG_WARP : 0;
  static constexpr size_t STG_OFF = (size_t)STAGES * STAGE_BYTES + 1024;  // after the barrier block
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + (STG_BYTES ? 1024 + STG_BYTES : 256);
  static_assert(STAGES >= 2 && 2 * STAGES + 5 <= 32, "ring depth / barrier block");
};

template <int KS>
__global__ void __launch_bounds__(kMaxGemmThreads, 1)
    umma_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmO, int M, int N, int K, GemmEpilogue ep, int *err) {
  using C = PairCfg<KS>;
  constexpr int S = C::STAGES;
  constexpr uint32_t TM_COLS = 512;  // two 256-column accumulators
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (size_t)S * C::STAGE_BYTES);
  uint64_t *full = bars, *empty = bars + S;
  uint64_t *accf = bars + 2 * S, *acce = bars + 2 * S + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 4);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  const int n_tiles = (N + C::BN - 1) / C::BN, m_tiles = (M + C::BM - 1) / C::BM;
  const int total = n_tiles * m_tiles;
  const int nk = (K + C::BK - 1) / C::BK;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 256);
    }
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist and their TMEM is allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto stage_a = [&](int i) { return smem + (size_t)i * C::STAGE_BYTES; };
  auto stage_b = [&](int i) { return smem + (size_t)i * C::STAGE_BYTES + C::A_BYTES; };
  auto fail = [&]() {
    s_abort = 1;
    atomicOr(err, 1 << AF_ERR_TIMEOUT);
  };

  if (is_producer_warp(warp)) {
    if (lane == 0 && producer_id(warp) < active_producers(S)) {
      const int np = active_producers(S), p = producer_id(warp);  // producer p: slices g = p (mod np)
      const int my_tiles = cid < total ? (total - 1 - cid) / ncl + 1 : 0;
      const int g_end = my_tiles * nk;  // K slices of this pair over all its tiles
      int issued = 0;
      for (int g = p; g < g_end && !s_abort; g += np) {
        const int t = cid + (g / nk) * ncl, kb = g % nk;
        const int m0 = (t / n_tiles) * C::BM + (int)rank * C::HALF, n0 = (t % n_tiles) * C::BN + (int)rank * C::HALF;
        const int i = g % S;
        if (!mbar_wait(&empty[i], ((g / S) & 1) ^ 1)) { fail(); break; }
        if (rank == 0) mbar_arrive_expect_tx(&full[i], 2 * C::STAGE_BYTES);
        const uint32_t fb = mapa_shared(&full[i], 0);
        const int kx = kb * C::BK;
        if constexpr (KS == 1) {
          tma_load_2d_pair(stage_a(i), &tmA, fb, kx % ep.a_kb, m0 + (kx / ep.a_kb) * M);
          tma_load_2d_pair(stage_b(i), &tmB, fb, kx, n0);
        } else {  // KS slices per copy: K blocks of A are multiples of BK (host check)
          tma_load_3d_pair(stage_a(i), &tmA, fb, 0, m0 + (kx / ep.a_kb) * M, (kx % ep.a_kb) / 64);
          tma_load_3d_pair(stage_b(i), &tmB, fb, 0, n0, kx / 64);
        }
        issued = g + 1;
      }
      if (rank == 0) {
        drain_producer(full, S, g_end, issued, p, np, s_abort != 0, fail);  // both CTAs' loads
      } else if (s_abort) {
        // this CTA's loads complete the other CTA's barriers: give them time to land
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 100000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      constexpr uint32_t idesc = idesc_f32acc(kFmtBF16, C::BM, C::BN);
      int g = 0, it = 0;
      bool ok = true;
      for (int t = cid; t < total && ok; t += ncl, ++it) {
        const int b = it & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&acce[b], ((it >> 1) & 1) ^ 1));
        if (!ok) break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * C::BN);
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int i = g % S;
          ok = __all_sync(0xffffffffu, mbar_wait(&full[i], (g / S) & 1));
          if (!ok || __any_sync(0xffffffffu, s_abort != 0)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
#pragma unroll
            for (int sl = 0; sl < KS; ++sl) {
              const uint64_t da = sdesc_k_sw128(stage_a(i) + sl * C::SLICE), db = sdesc_k_sw128(stage_b(i) + sl * C::SLICE);
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const uint64_t off = (uint64_t)(k * 32) >> 4;
                umma_bf16_pair(acc, da + off, db + off, idesc, (kb | sl | k) != 0);
              }
            }
            umma_commit_pair(mapa_shared(&empty[i], 0));
            umma_commit_pair(mapa_shared(&empty[i], 1));
          }
          __syncwarp();
        }
        if (lane == 0 && ok) {
          umma_commit_pair(mapa_shared(&accf[b], 0));
          umma_commit_pair(mapa_shared(&accf[b], 1));
        }
        __syncwarp();
      }
      if (!ok && lane == 0) fail();
    }
  } else {
    const int q = warp & 3;
    int it = 0;
    for (int t = cid; t < total; t += ncl, ++it) {
      const int b = it & 1;
      const bool ok = mbar_wait(&accf[b], (it >> 1) & 1);
      if (!ok) {
        fail();
        break;
      }
      tc_fence_after();
      const int m0 = (t / n_tiles) * C::BM, n0 = (t % n_tiles) * C::BN;
      const int row = m0 + (int)rank * C::HALF + q * 32 + lane;
      const bool row_ok = row < M;
      float scale = 1.f;
      if (ep.row_parts && row_ok) scale = row_scale(ep, row, M);
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * C::BN);
      auto load16 = [&](int col, float (&v)[16]) {
        __syncwarp();
        tmem_ld16(tbase + col, v);
      };
      auto wait_ld = [&]() { tmem_wait_ld(); };
      if (C::STG_BYTES && (ep.staged == kStagePair || ep.staged == kStagePairAdd)) {
        // The tile through this warp's 8 KB staging buffer and TMA stores, per
        // 64 columns: fp32 as two 128-byte-swizzled [32 rows x 32 cols] boxes
        // (the whole buffer), bf16 as one [32 x 64] box (alternating halves).
        // Chunk c of row r sits at chunk c ^ (r & 7), so the lanes' 16-byte
        // writes spread over the banks.
        uint8_t *buf = smem + C::STG_OFF + q * C::STG_WARP;
        const int row0 = m0 + (int)rank * C::HALF + q * 32;
#pragma unroll 1
        for (int c0 = 0; c0 < C::BN; c0 += 64) {
          float vv[4][16];
#pragma unroll
          for (int u = 0; u < 4; ++u) load16(c0 + 16 * u, vv[u]);
          wait_ld();
          if (ep.out_bf16) {
            uint8_t *box = buf + ((c0 >> 6) & 1) * 4096;
            if (lane == 0) bulk_wait_read_but_one();  // the store that last read this half is done
            __syncwarp();
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int n = n0 + c0 + 16 * u;
              uint32_t pk[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                float x0 = vv[u][2 * e] * scale, x1 = vv[u][2 * e + 1] * scale;
                if (ep.bias) {
                  x0 += n + 2 * e < N ? ep.bias[n + 2 * e] : 0.f;
                  x1 += n + 2 * e + 1 < N ? ep.bias[n + 2 * e + 1] : 0.f;
                }
                __nv_bfloat162 b2 = __floats2bfloat162_rn(x0, x1);
                pk[e] = *reinterpret_cast<uint32_t *>(&b2);
              }
              uint8_t *line = box + lane * 128;
              *reinterpret_cast<uint4 *>(line + (((2 * u) ^ (lane & 7)) * 16)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              *reinterpret_cast<uint4 *>(line + (((2 * u + 1) ^ (lane & 7)) * 16)) =
                  make_uint4(pk[4], pk[5], pk[6], pk[7]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmO, box, n0 + c0, row0);
              bulk_commit();
            }
            continue;
          }
          if (lane == 0) bulk_wait_read_all();  // the buffer's previous stores have read it
          __syncwarp();
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int n = n0 + c0 + 16 * u;
            uint8_t *box = buf + (u >> 1) * 4096 + lane * 128;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              float4 f;
              f.x = vv[u][4 * k] * scale;
              f.y = vv[u][4 * k + 1] * scale;
              f.z = vv[u][4 * k + 2] * scale;
              f.w = vv[u][4 * k + 3] * scale;
              if (ep.bias) {
                const int c = n + 4 * k;
                f.x += c < N ? ep.bias[c] : 0.f;
                f.y += c + 1 < N ? ep.bias[c + 1] : 0.f;
                f.z += c + 2 < N ? ep.bias[c + 2] : 0.f;
                f.w += c + 3 < N ? ep.bias[c + 3] : 0.f;
              }
              *reinterpret_cast<float4 *>(box + ((((u & 1) * 4 + k) ^ (lane & 7)) * 16)) = f;
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (ep.staged == kStagePairAdd) {  // out holds the residual: add the tile into it
              tma_reduce_add_2d(&tmO, buf, n0 + c0, row0);
              tma_reduce_add_2d(&tmO, buf + 4096, n0 + c0 + 32, row0);
            } else {
              tma_store_2d(&tmO, buf, n0 + c0, row0);
              tma_store_2d(&tmO, buf + 4096, n0 + c0 + 32, row0);
            }
            bulk_commit();
          }
        }
      } else {
        store_tile<C::BN>(ep, load16, wait_ld, row, row_ok, n0, N, true, scale, true);
      }
      tc_fence_before();
      if (rank == 0) mbar_arrive(&acce[b]);
      else mbar_arrive_cluster(mapa_shared(&acce[b], 0));
    }
    if (C::STG_BYTES && ep.staged && lane == 0) bulk_wait_all();  // stores done before exit
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA frees TMEM or exits while the pair's MMAs may touch it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, TM_COLS);
  }
}

// One 256 x BN output tile per CTA pair (cta_group::2), split-K over
// gridDim.z: the decode-sized bf16 and pre-split 3xTF32 products.  Each CTA
// loads its own 128 rows of A and BN/2 rows of B per K slice, so the operand
// that every tile shares (the activations of a transposed projection, or the
// weights of a direct one) is fetched half per CTA: fewer bytes per SM per
// MMA flop than a 128 x BN tile on one SM.  Barriers as in the persistent
// pair kernel, one tile: full[i] on rank 0, empty[i] and accf on both CTAs.
template <int BN, int MODE>
struct PairSplitCfg {
  static constexpr bool TF32X3 = MODE != kBF16;
  static constexpr int HALF = 128, BNH = BN / 2;
  static constexpr int ELEM = TF32X3 ? 4 : 2, BK = 128 / ELEM, UK = 32 / ELEM;
  static constexpr int A_BYTES = HALF * 128, B_BYTES = BNH * 128, RAW = A_BYTES + B_BYTES;
  static constexpr int STAGE_BYTES = TF32X3 ? 2 * RAW : RAW;  // hi and lo parts for 3xTF32
  static constexpr int SMEM_LIMIT = 227 * 1024 - 64;
  static constexpr int STAGES_FIT = (SMEM_LIMIT - 1024 - 256) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT < 12 ? STAGES_FIT : 12;
  static constexpr int ACC_COLS = (TF32X3 ? 2 : 1) * BN;  // accumulator (+ correction terms)
  static constexpr int TMEM_COLS =
      ACC_COLS <= 32 ? 32 : ACC_COLS <= 64 ? 64 : ACC_COLS <= 128 ? 128 : ACC_COLS <= 256 ? 256 : 512;
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
  static_assert(MODE == kBF16 || MODE == kTF32P, "bf16 or pre-split tf32");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "pair N");
  static_assert(ACC_COLS <= 512 && STAGES >= 2 && 2 * STAGES + 2 <= 32, "TMEM / ring / barrier block");
};

template <int BN, int MODE>
__global__ void __launch_bounds__(kMaxGemmThreads, 1)
    umma_gemm_pair_split_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                                const __grid_constant__ CUtensorMap tmO, int M, int N, int K, GemmEpilogue ep,
                                int *err) {
  using C = PairSplitCfg<BN, MODE>;
  constexpr bool TF32X3 = C::TF32X3;
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (size_t)S * C::STAGE_BYTES);
  uint64_t *full = bars, *empty = bars + S, *accf = bars + 2 * S;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * S + 1);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int m0 = (int)(blockIdx.x >> 1) * 256 + (int)rank * C::HALF;  // this CTA's A rows
  const int n0 = blockIdx.y * BN, nb0 = n0 + (int)rank * C::BNH;       // the tile's N, this CTA's B rows
  const int nk_all = (K + C::BK - 1) / C::BK;
  const int kb_base = (int)(((int64_t)blockIdx.z * nk_all) / gridDim.z);
  const int nk = (int)(((int64_t)(blockIdx.z + 1) * nk_all) / gridDim.z) - kb_base;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(accf, 1);
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if constexpr (TF32X3) {
      prefetch_tmap(&tmA2);
      prefetch_tmap(&tmB2);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist and their TMEM is allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto stage = [&](int i) { return smem + (size_t)i * C::STAGE_BYTES; };
  auto fail = [&]() {
    s_abort = 1;
    atomicOr(err, 1 << AF_ERR_TIMEOUT);
  };

  if (is_producer_warp(warp)) {
    if (lane == 0 && producer_id(warp) < active_producers(S)) {
      const int np = active_producers(S), p = producer_id(warp);  // producer p: K slices kb = p (mod np)
      auto load_a = [&](int i, int kx) {
        const uint32_t fb = mapa_shared(&full[i], 0);
        const int ka = kx % ep.a_kb, ma = m0 + (kx / ep.a_kb) * M;
        tma_load_2d_pair(stage(i), &tmA, fb, ka, ma);
        if constexpr (TF32X3) tma_load_2d_pair(stage(i) + C::RAW, &tmA2, fb, ka, ma);
      };
      auto load_b = [&](int i, int kx) {
        const uint32_t fb = mapa_shared(&full[i], 0);
        tma_load_2d_pair(stage(i) + C::A_BYTES, &tmB, fb, kx, nb0);
        if constexpr (TF32X3) tma_load_2d_pair(stage(i) + C::RAW + C::A_BYTES, &tmB2, fb, kx, nb0);
      };
      // operand independent of the previous kernel first (programmatic launch)
      const int pre = ep.pre_operand ? (nk < S ? nk : S) : 0;
      for (int kb = p; kb < pre; kb += np) {
        if (rank == 0) mbar_arrive_expect_tx(&full[kb], 2 * C::STAGE_BYTES);
        if (ep.pre_operand == 1) load_a(kb, (kb_base + kb) * C::BK);
        else load_b(kb, (kb_base + kb) * C::BK);
      }
      griddep_wait();
      for (int kb = p; kb < pre; kb += np) {
        if (ep.pre_operand == 1) load_b(kb, (kb_base + kb) * C::BK);
        else load_a(kb, (kb_base + kb) * C::BK);
      }
      int issued = pre;
      for (int kb = first_owned(pre, p, np); kb < nk && !s_abort; kb += np) {
        const int i = kb % S;
        if (!mbar_wait(&empty[i], ((kb / S) & 1) ^ 1)) { fail(); break; }
        if (rank == 0) mbar_arrive_expect_tx(&full[i], 2 * C::STAGE_BYTES);
        const int kx = (kb_base + kb) * C::BK;
        load_a(i, kx);
        load_b(i, kx);
        issued = kb + 1;
      }
      if (rank == 0) {
        drain_producer(full, S, nk, issued, p, np, s_abort != 0, fail);  // both CTAs' loads
      } else if (s_abort) {
        const uint64_t t0 = globaltimer();  // this CTA's loads complete the other CTA's barriers
        while (globaltimer() - t0 < 100000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      constexpr uint32_t idesc = idesc_f32acc(TF32X3 ? kFmtTF32 : kFmtBF16, 256, BN);
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        const int i = kb % S;
        ok = __all_sync(0xffffffffu, mbar_wait(&full[i], (kb / S) & 1));
        if (!ok || __any_sync(0xffffffffu, s_abort != 0)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint64_t da = sdesc_k_sw128(stage(i)), db = sdesc_k_sw128(stage(i) + C::A_BYTES);
#pragma unroll
          for (int k = 0; k < C::BK / C::UK; ++k) {
            const uint64_t off = (uint64_t)(k * 32) >> 4;
            if constexpr (TF32X3) {
              const uint64_t dal = sdesc_k_sw128(stage(i) + C::RAW), dbl = sdesc_k_sw128(stage(i) + C::RAW + C::A_BYTES);
              umma_tf32_pair(tmem, da + off, db + off, idesc, (kb | k) != 0);
              umma_tf32_pair(tmem + BN, da + off, dbl + off, idesc, (kb | k) != 0);
              umma_tf32_pair(tmem + BN, dal + off, db + off, idesc, 1);
            } else {
              umma_bf16_pair(tmem, da + off, db + off, idesc, (kb | k) != 0);
            }
          }
          umma_commit_pair(mapa_shared(&empty[i], 0));
          umma_commit_pair(mapa_shared(&empty[i], 1));
        }
        __syncwarp();
      }
      if (lane == 0) {
        if (!ok) fail();
        umma_commit_pair(mapa_shared(accf, 0));  // also on failure, so the epilogues do not wait out
        umma_commit_pair(mapa_shared(accf, 1));
      }
      __syncwarp();
    }
  } else {
    const bool ok = mbar_wait(accf, 0);
    if (!ok) fail();
    tc_fence_after();
    griddep_wait();  // the epilogue reads row sums / residual and writes out
    const int q = warp & 3;
    const int row = m0 + q * 32 + lane;
    const bool row_ok = row < M;
    float scale = 1.f;
    if (ep.row_parts && row_ok && !ep.trans) scale = row_scale(ep, row, M);
    const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16);
    auto load16 = [&](int col, float (&v)[16]) {
      __syncwarp();
      tmem_ld16(tbase + col, v);
      if constexpr (TF32X3) {  // accumulator + correction terms
        float w[16];
        tmem_ld16(tbase + (uint32_t)BN + col, w);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] += w[e];
      }
    };
    auto wait_ld = [&]() {
      if constexpr (!TF32X3) tmem_wait_ld();
    };
    if (ep.staged)
      store_tile_staged<BN>(ep, &tmO, load16, wait_ld, reinterpret_cast<float *>(smem), q * 32 + lane, m0, n0,
                            blockIdx.z, N, ok && !s_abort, scale);
    else
      store_tile<BN>(ep, load16, wait_ld, row, row_ok, n0, N, ok && !s_abort, scale, blockIdx.z == 0);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA frees TMEM or exits while the pair's MMAs may touch it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host
// Threads of a GEMM CTA: the six fixed warps and one more warp per extra
// TMA producer (the option, capped at the ring depth).
int block_threads(const af_ctx *ctx, int stages) {
  return gemm_threads(ctx->gemm_producers < stages ? ctx->gemm_producers : stages);
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int get_encoder(const char *fn) {
  if (g_encode) return AF_OK;
  void *p = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
    return af::fail(AF_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable", fn);
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  return AF_OK;
}

// K-major 2-D tensor map: rows x K elements, row stride ld elements; box =
// (128 bytes of K) x box_rows, 128-byte swizzle, zero fill out of bounds.
int make_kmajor_map(CUtensorMap *map, const void *base, bool fp32, int rows, int K, int64_t ld, int box_rows,
                    const char *fn) {
  const int elem = fp32 ? 4 : 2;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * elem};
  cuuint32_t box[2] = {(cuuint32_t)(128 / elem), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                        const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return af::fail(AF_ERR_ARG, "%s: cuTensorMapEncodeTiled failed (%d)", fn, (int)r);
  return AF_OK;
}

// Tensor map of the output for a staged epilogue (store_tile_staged).
int make_staged_out_map(CUtensorMap *map, const GemmEpilogue &ep, int M, int N, int splits, int BN, const char *fn) {
  CUresult r;
  if (ep.staged == kStageTrans) {
    const int64_t zs = ep.split_stride ? ep.split_stride : ep.ldo * (int64_t)N;
    cuuint64_t dims[3] = {(cuuint64_t)M, (cuuint64_t)N, (cuuint64_t)(ep.split_stride ? splits : 1)};
    cuuint64_t strides[2] = {(cuuint64_t)ep.ldo * 4, (cuuint64_t)zs * 4};
    cuuint32_t box[3] = {128, (cuuint32_t)BN, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, ep.out, dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else if (ep.staged == kStageSwiGLU) {
    cuuint64_t dims[2] = {(cuuint64_t)(M / 2), (cuuint64_t)N};
    cuuint64_t strides[1] = {(cuuint64_t)ep.ldo * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)BN};
    cuuint32_t estr[2] = {1, 1};
    r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ep.out, dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else if (ep.staged == kStageTransAdd) {
    cuuint64_t dims[2] = {(cuuint64_t)M, (cuuint64_t)N};
    cuuint64_t strides[1] = {(cuuint64_t)ep.ldo * 4};
    cuuint32_t box[2] = {128, (cuuint32_t)BN};
    cuuint32_t estr[2] = {1, 1};
    r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ep.out, dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)ep.ldo * 4};
    cuuint32_t box[2] = {32, 128};
    cuuint32_t estr[2] = {1, 1};
    r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ep.out, dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return af::fail(AF_ERR_ARG, "%s: output tensor map failed (%d)", fn, (int)r);
  return AF_OK;
}

// Bytes of shared memory a staged epilogue of a 128 x BN tile needs.
constexpr size_t staged_bytes(int BN) { return (size_t)128 * BN * 4; }

template <int BN>
int launch_persistent(af_ctx *ctx, const void *A, int64_t lda, const void *B, int64_t ldb, int M, int N, int K,
                      const GemmEpilogue &ep, cudaStream_t st, const char *fn, int ep_max_ctas) {
  using C = TileCfg<BN, kBF16>;
  CUtensorMap ta, tb;
  int rc = make_kmajor_map(&ta, A, false, (K / ep.a_kb) * M, ep.a_kb, lda, C::BM, fn);
  if (rc) return rc;
  rc = make_kmajor_map(&tb, B, false, N, K, ldb, BN, fn);
  if (rc) return rc;
  static std::atomic<unsigned long long> attr_devices{0};
  if (int arc = af::smem_attr(ctx, reinterpret_cast<const void *>(umma_gemm_persistent_kernel<BN>), C::SMEM,
                              attr_devices, fn))
    return arc;
  const int64_t total = (int64_t)((N + BN - 1) / BN) * ((M + C::BM - 1) / C::BM);
  const int cap = ep_max_ctas > 0 && ep_max_ctas < ctx->num_sms ? ep_max_ctas : ctx->num_sms;
  const int grid = (int)(total < cap ? total : cap);
  umma_gemm_persistent_kernel<BN><<<grid, block_threads(ctx, C::STAGES), C::SMEM, st>>>(ta, tb, M, N, K, ep,
                                                                                       ctx->dev_err);
  return af::launched(ctx, fn);
}

template <int BN, int MODE>
int launch_pair_split(af_ctx *ctx, const void *A, const void *A2, int64_t lda, const void *B, const void *B2,
                      int64_t ldb, int M, int N, int K, int splits, const GemmEpilogue &ep, cudaStream_t st,
                      const char *fn, bool pdl) {
  using C = PairSplitCfg<BN, MODE>;
  const bool fp32 = MODE != kBF16;
  CUtensorMap ta, tb, ta2, tb2;
  int rc = make_kmajor_map(&ta, A, fp32, (K / ep.a_kb) * M, ep.a_kb, lda, C::HALF, fn);
  if (rc) return rc;
  rc = make_kmajor_map(&tb, B, fp32, N, K, ldb, C::BNH, fn);
  if (rc) return rc;
  ta2 = ta;
  tb2 = tb;
  if (MODE == kTF32P) {
    rc = make_kmajor_map(&ta2, A2, true, (K / ep.a_kb) * M, ep.a_kb, lda, C::HALF, fn);
    if (rc) return rc;
    rc = make_kmajor_map(&tb2, B2, true, N, K, ldb, C::BNH, fn);
    if (rc) return rc;
  }
  static std::atomic<unsigned long long> attr_devices{0};
  if (int arc = af::smem_attr(ctx, reinterpret_cast<const void *>(umma_gemm_pair_split_kernel<BN, MODE>), C::SMEM,
                              attr_devices, fn))
    return arc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * ((M + 255) / 256), (N + BN - 1) / BN, splits);
  cfg.blockDim = dim3(block_threads(ctx, C::STAGES));
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  CUtensorMap to = ta;
  GemmEpilogue epx = ep;
  // the ring must hold the staged tile; reduce-adds go in 32-column boxes
  if ((size_t)C::STAGES * C::STAGE_BYTES < staged_bytes(BN) || (epx.staged == kStageAdd && BN % 32 != 0))
    epx.staged = 0;
  if (epx.staged) {
    rc = make_staged_out_map(&to, epx, M, N, splits, BN, fn);
    if (rc) return rc;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, umma_gemm_pair_split_kernel<BN, MODE>, ta, tb, ta2, tb2, to, M, N, K,
                                           epx, ctx->dev_err);
  if (e != cudaSuccess) return af::fail(AF_ERR_CUDA, "%s: pair launch: %s", fn, cudaGetErrorString(e));
  return af::launched(ctx, fn);
}

// K-major 3-D view of a bf16 matrix for stages of KS K slices: {64 elements,
// rows, K / 64 slices}, strides {row pitch, 128 bytes}; box {64, box_rows, KS}.
int make_kslices_map(CUtensorMap *map, const void *base, int rows, int K, int64_t ld, int box_rows, int ks,
                     const char *fn) {
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(K / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, 128};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)ks};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return af::fail(AF_ERR_ARG, "%s: cuTensorMapEncodeTiled (3-D) failed (%d)", fn, (int)r);
  return AF_OK;
}

template <int KS>
int launch_pair_ks(af_ctx *ctx, const void *A, int64_t lda, const void *B, int64_t ldb, int M, int N, int K,
                   const GemmEpilogue &ep, cudaStream_t st, const char *fn) {
  using C = PairCfg<KS>;
  CUtensorMap ta, tb;
  int rc;
  if constexpr (KS == 1) {
    rc = make_kmajor_map(&ta, A, false, (K / ep.a_kb) * M, ep.a_kb, lda, C::HALF, fn);
    if (rc) return rc;
    rc = make_kmajor_map(&tb, B, false, N, K, ldb, C::HALF, fn);
  } else {
    rc = make_kslices_map(&ta, A, (K / ep.a_kb) * M, ep.a_kb, lda, C::HALF, KS, fn);
    if (rc) return rc;
    rc = make_kslices_map(&tb, B, N, K, ldb, C::HALF, KS, fn);
  }
  if (rc) return rc;
  static std::atomic<unsigned long long> attr_devices{0};
  if (int arc = af::smem_attr(ctx, reinterpret_cast<const void *>(umma_gemm_pair_kernel<KS>), C::SMEM, attr_devices,
                              fn))
    return arc;
  const int64_t total = (int64_t)((N + C::BN - 1) / C::BN) * ((M + C::BM - 1) / C::BM);
  const int pairs = (int)(total < ctx->num_sms / 2 ? total : ctx->num_sms / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(block_threads(ctx, C::STAGES));
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // fp32 or bf16 output without residual: epilogue through shared memory
  // and TMA stores (AF_GEMM_NO_STAGE=1 turns it off)
  CUtensorMap to = ta;
  GemmEpilogue epx = ep;
  epx.staged = 0;
  const int ob = ep.out_bf16 ? 2 : 4;
  // a residual that is the output itself (x += ...) becomes a TMA reduce-add
  const bool in_place = ep.residual && (const void *)ep.residual == ep.out && ep.ldr == ep.ldo && !ep.out_bf16 &&
                        !ep.scale_residual;
  if (C::STG_BYTES && !ep.trans && !ep.atomic && !ep.swiglu && (!ep.residual || in_place) && af::aligned16(ep.out) &&
      (ep.ldo * ob) % 16 == 0 && !getenv("AF_GEMM_NO_STAGE")) {
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)ep.ldo * ob};
    cuuint32_t box[2] = {(cuuint32_t)(128 / ob), 32};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r =
        g_encode(&to, ep.out_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ep.out,
                 dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return af::fail(AF_ERR_ARG, "%s: output tensor map failed (%d)", fn, (int)r);
    epx.staged = in_place ? kStagePairAdd : kStagePair;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, umma_gemm_pair_kernel<KS>, ta, tb, to, M, N, K, epx, ctx->dev_err);
  if (e != cudaSuccess) return af::fail(AF_ERR_CUDA, "%s: pair launch: %s", fn, cudaGetErrorString(e));
  return af::launched(ctx, fn);
}

// Two K slices per stage when every stage's slices lie in one K block of A
// (K a multiple of 64; K blocks, if any, multiples of 128); AF_GEMM_KS=1
// forces one.
int launch_pair(af_ctx *ctx, const void *A, int64_t lda, const void *B, int64_t ldb, int M, int N, int K,
                const GemmEpilogue &ep, cudaStream_t st, const char *fn) {
  bool two = K % 64 == 0 && (ep.a_kb == K || ep.a_kb % 128 == 0);
  if (const char *e = getenv("AF_GEMM_KS")) two = two && atoi(e) != 1;
  if (two) return launch_pair_ks<2>(ctx, A, lda, B, ldb, M, N, K, ep, st, fn);
  return launch_pair_ks<1>(ctx, A, lda, B, ldb, M, N, K, ep, st, fn);
}

template <int BN, int MODE, int KS>
int launch_tc_ks(af_ctx *ctx, const void *A, const void *A2, int64_t lda, const void *B, const void *B2, int64_t ldb,
                 int M, int N, int K, int splits, const GemmEpilogue &ep, cudaStream_t st, const char *fn, bool pdl) {
  using C = TileCfg<BN, MODE, KS>;
  CUtensorMap ta, tb, ta2, tb2;
  const bool fp32 = MODE != kBF16;
  int rc;
  if constexpr (KS > 1) {
    rc = make_kslices_map(&ta, A, (K / ep.a_kb) * M, ep.a_kb, lda, C::BM, KS, fn);
    if (rc) return rc;
    rc = make_kslices_map(&tb, B, N, K, ldb, BN, KS, fn);
  } else {
    rc = make_kmajor_map(&ta, A, fp32, (K / ep.a_kb) * M, ep.a_kb, lda, C::BM, fn);
    if (rc) return rc;
    rc = make_kmajor_map(&tb, B, fp32, N, K, ldb, BN, fn);
  }
  if (rc) return rc;
  ta2 = ta;
  tb2 = tb;
  if (MODE == kTF32P) {
    rc = make_kmajor_map(&ta2, A2, true, (K / ep.a_kb) * M, ep.a_kb, lda, C::BM, fn);
    if (rc) return rc;
    rc = make_kmajor_map(&tb2, B2, true, N, K, ldb, BN, fn);
    if (rc) return rc;
  }
  CUtensorMap to = ta;
  GemmEpilogue epx = ep;
  // the ring must hold the staged tile; reduce-adds go in 32-column boxes
  if ((size_t)C::STAGES * C::STAGE_BYTES < staged_bytes(BN) || (epx.staged == kStageAdd && BN % 32 != 0))
    epx.staged = 0;
  if (epx.staged) {
    rc = make_staged_out_map(&to, epx, M, N, splits, BN, fn);
    if (rc) return rc;
  }
  static std::atomic<unsigned long long> attr_devices{0};
  if (int arc = af::smem_attr(ctx, reinterpret_cast<const void *>(umma_gemm_kernel<BN, MODE, KS>), C::SMEM,
                              attr_devices, fn))
    return arc;
  const dim3 grid((N + BN - 1) / BN, (M + C::BM - 1) / C::BM, splits);
  const cudaError_t e =
      af::launch_kernel(umma_gemm_kernel<BN, MODE, KS>, grid, dim3(block_threads(ctx, C::STAGES)), C::SMEM, st, pdl,
                        ta, tb, ta2, tb2, to, M, N, K, epx, ctx->dev_err);
  if (e != cudaSuccess) return af::fail(AF_ERR_CUDA, "%s: launch: %s", fn, cudaGetErrorString(e));
  return af::launched(ctx, fn);
}

// bf16 tiles up to 128 wide take two K slices per stage (half the MMA
// thread's barrier waits and commits per MMA) when K is a multiple of 64, K
// blocks of A are multiples of 128 and every split keeps at least one stage;
// AF_GEMM_KS=1 forces one slice.
template <int BN, int MODE>
int launch_tc(af_ctx *ctx, const void *A, const void *A2, int64_t lda, const void *B, const void *B2, int64_t ldb,
              int M, int N, int K, int splits, const GemmEpilogue &ep, cudaStream_t st, const char *fn, bool pdl) {
  if constexpr (MODE == kBF16 && BN <= 128) {
    bool two = K % 64 == 0 && (ep.a_kb == K || ep.a_kb % 128 == 0) && splits <= (K + 127) / 128;
    if (const char *e = getenv("AF_GEMM_KS")) two = two && atoi(e) != 1;
    if (two) return launch_tc_ks<BN, MODE, 2>(ctx, A, A2, lda, B, B2, ldb, M, N, K, splits, ep, st, fn, pdl);
  }
  return launch_tc_ks<BN, MODE, 1>(ctx, A, A2, lda, B, B2, ldb, M, N, K, splits, ep, st, fn, pdl);
}

// Splits the fp32 array src into an exact tf32 part and the remainder.
__global__ void split_tf32_kernel(const float *__restrict__ src, float *__restrict__ hi, float *__restrict__ lo,
                                  int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float x = src[i];
    const float h = tf32_hi(x);
    hi[i] = h;
    lo[i] = x - h;
  }
}

// The same over float4s (16-byte aligned arrays, n % 4 == 0); optionally
// zeroes `zero` (n floats) on the way - the output that a later split-K GEMM
// of the same step accumulates into.
__global__ void split_tf32_vec_kernel(const float4 *__restrict__ src, float4 *__restrict__ hi, float4 *__restrict__ lo,
                                      float4 *__restrict__ zero, int64_t n4) {
  griddep_wait();  // programmatic launch: the previous kernel may still read `zero`
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 x = src[i];
    const float4 h = make_float4(tf32_hi(x.x), tf32_hi(x.y), tf32_hi(x.z), tf32_hi(x.w));
    hi[i] = h;
    lo[i] = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
    if (zero) zero[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// Tile width, split count and launch for one GEMM.  Narrow tiles and split-K
// put a CTA on every SM for decode-sized M; split-K needs an fp32, non-SwiGLU
// epilogue (it accumulates with atomics).
template <int MODE>
int dispatch(af_ctx *ctx, const void *A, const void *A2, int64_t lda, const void *B, const void *B2, int64_t ldb,
             int M, int N, int K, const af::GemmEpilogueArgs &a, cudaStream_t st, const char *fn) {
  int rc = get_encoder(fn);
  if (rc) return rc;
  if (M == 0 || N == 0) return AF_OK;
  const bool vec = af::aligned16(a.out) && (a.ldo * (a.out_bf16 ? 2 : 4)) % 16 == 0;
  if (a.swiglu && !a.trans && (!vec || N % 32 != 0))
    return af::fail(AF_ERR_ARG, "%s: SwiGLU epilogue needs an aligned output and N %% 32 == 0", fn);
  constexpr int bk_elems = MODE == kBF16 ? 64 : 32;
  if (a.a_kblock && (a.a_kblock % bk_elems != 0 || K % a.a_kblock != 0 || lda < a.a_kblock))
    return af::fail(AF_ERR_ARG, "%s: K block %d must divide K=%d and be a multiple of %d", fn, a.a_kblock, K, bk_elems);
  if (a.parts_block && (a.parts_block < 1 || a.nparts % a.parts_block != 0))
    return af::fail(AF_ERR_ARG, "%s: parts block %d must divide nparts=%d", fn, a.parts_block, a.nparts);
  GemmEpilogue ep{a.out, a.ldo,      a.out_bf16, a.bias,   a.row_parts, a.nparts,   a.inv_d,
                  a.eps, a.residual, a.ldr,      a.swiglu, vec ? 1 : 0, 0,
                  a.a_kblock ? a.a_kblock : K, a.parts_block ? a.parts_block : (a.nparts > 0 ? a.nparts : 1),
                  a.trans, a.split_stride, a.scale_residual,
                  a.residual && af::aligned16(a.residual) && (a.ldr * 4) % 16 == 0 ? 1 : 0, 0};
  // programmatic dependent launch (non-persistent kernels only; split-K with a
  // memset before it is launched normally)
  bool pdl = a.pdl && ctx->pdl;
  ep.pre_operand = pdl ? a.pre_operand : 0;
  if (a.split_stride && (!a.trans || a.swiglu || a.out_bf16 || a.bias || a.residual || a.row_parts || a.accumulate ||
                         a.a_kblock))
    return af::fail(AF_ERR_ARG, "%s: partial buffers: transposed plain fp32 output only", fn);
  if (a.trans && (a.bias || a.residual || a.a_kblock || a.scale_residual || (a.out_bf16 && !a.swiglu) ||
                  (a.swiglu && (a.accumulate || !a.out_bf16 || M % 32 != 0))))
    return af::fail(AF_ERR_ARG, "%s: unsupported transposed epilogue", fn);
  const int64_t mt = (M + 127) / 128;
  auto tiles = [&](int bn) { return mt * ((N + bn - 1) / bn); };
  const int64_t sms = ctx->num_sms;
  constexpr int bk = MODE == kBF16 ? 64 : 32;
  const int nk = (K + bk - 1) / bk;
  const bool can_split = !a.swiglu && !a.out_bf16 && ctx->allow_split_k && !a.scale_residual;
  // Widest tile first (each A slice then feeds the most MMA work and is
  // re-read by the fewest CTAs; measured on B200: a 256x6144x2048 3xTF32
  // GEMM takes 54 us at BN=128 vs 92 us at BN=64).  Small-M GEMMs then fill
  // the SMs with split-K, but only up to one wave (one CTA per SM: a second
  // partial wave costs more than it saves).  Without split-K (SwiGLU or bf16
  // output) the widest tile that still keeps ~60% of the SMs busy is used.
  const int widest = MODE == kBF16 ? 256 : 128;
  int bn = widest;
  if (!can_split) {
    while (bn > (MODE == kBF16 ? 16 : 32) && tiles(bn) * 10 < sms * 6 && !(a.swiglu && bn == 32)) bn /= 2;
  }
  int splits = 1;
  if (can_split && tiles(bn) < sms) {
    int max_split = nk / 4 > 1 ? nk / 4 : 1;  // keep >= 4 K slices per split
    if (max_split > 8) max_split = 8;
    while (bn > 64 && tiles(bn) * max_split * 10 < sms * 6) bn /= 2;  // too few tiles even when split
    splits = (int)(sms / tiles(bn));
    if (splits > max_split) splits = max_split;
    if (splits < 1) splits = 1;
  }
  // Pre-split decode GEMMs (one wave or less): pick width and split by a
  // cost model, waves x tile width x K slices per CTA, which also weighs the
  // 96-wide tile (a 256 x 6144 QKV projection: 128 CTAs of 96 columns beat
  // 96 CTAs of 128 on 148 SMs).
  if (MODE == kTF32P && tiles(widest) < sms) {
    auto cost = [&](int w, int sp) {
      const int64_t ctas = tiles(w) * sp;
      return ((ctas + sms - 1) / sms) * (int64_t)w * ((nk + sp - 1) / sp);
    };
    int64_t best = cost(bn, splits);
    const int widths[4] = {128, 96, 64, 32};
    for (int w : widths) {
      const int max_sp = can_split ? (nk / 4 > 1 ? (nk / 4 > 8 ? 8 : nk / 4) : 1) : 1;
      for (int sp = 1; sp <= max_sp; ++sp) {
        if (tiles(w) * sp > sms) break;
        const int64_t c = cost(w, sp);
        if (c < best) {
          best = c;
          bn = w;
          splits = sp;
        }
      }
    }
  }
  if (a.force_bn) bn = a.force_bn;
  if (a.force_splits) splits = a.force_splits < nk ? a.force_splits : nk;
  // tuning overrides (tile-width / split-K sweeps): AF_GEMM_BN, AF_GEMM_SPLITS
  if (const char *e = getenv("AF_GEMM_BN")) {
    const int v = atoi(e);
    if (v == 16 || v == 32 || v == 64 || v == 128 || v == 256 || (v == 96 && MODE == kTF32P)) bn = v;
  }
  if (const char *e = getenv("AF_GEMM_SPLITS")) {
    const int v = atoi(e);
    if (v >= 1 && v <= 16 && (v == 1 || can_split) && v <= nk) splits = v;
  }
  if (a.split_stride) {
    if (a.split_stride < (int64_t)(a.trans ? N : M) * a.ldo || splits > a.max_partials)
      return af::fail(AF_ERR_ARG, "%s: partial buffers too small or too few", fn);
  } else if (a.accumulate) {
    if (a.swiglu || a.out_bf16) return af::fail(AF_ERR_ARG, "%s: accumulation needs an fp32 linear epilogue", fn);
    ep.atomic = 1;  // partial products added into out as it is
  } else if (splits > 1) {
    ep.atomic = 1;
    if (a.residual == a.out) {
      ep.residual = nullptr;  // out already holds the residual: every split adds its partial into it
    } else {
      pdl = false;
      ep.pre_operand = 0;
      cudaError_t e = cudaMemsetAsync(a.out, 0, (size_t)M * a.ldo * 4, st);
      if (e != cudaSuccess) return af::fail(AF_ERR_CUDA, "%s: zeroing the split-K output: %s", fn, cudaGetErrorString(e));
    }
  }
  // Epilogue through shared memory and TMA (umma_gemm_kernel and the pair
  // split kernel): transposed plain stores (partial buffers) and row-major
  // accumulation without bias or residual.  AF_GEMM_NO_STAGE=1 turns it off.
  const bool out_ok = af::aligned16(a.out) && (a.ldo * 4) % 16 == 0 && (a.split_stride * 4) % 16 == 0;
  if (af::aligned16(a.out) && (a.ldo * 2) % 16 == 0 && a.trans && a.swiglu && a.out_bf16 && !a.row_parts &&
      !ep.atomic && M % 128 == 0 && !getenv("AF_GEMM_NO_STAGE"))
    ep.staged = kStageSwiGLU;
  if (out_ok && !a.out_bf16 && !a.swiglu && !getenv("AF_GEMM_NO_STAGE")) {
    if (a.trans && !ep.atomic && !a.row_parts) ep.staged = kStageTrans;
    else if (a.trans && ep.atomic) ep.staged = kStageTransAdd;
    else if (!a.trans && ep.atomic && !ep.residual && !a.bias) ep.staged = kStageAdd;
  }
  // large bf16 GEMMs (two or more waves of tiles), or a CTA cap (SMs left to
  // a concurrent kernel): persistent kernel
  if (MODE == kBF16 && splits == 1 && !a.trans && !a.pair && (bn == 256 || bn == 128) &&
      (tiles(bn) >= 2 * sms || a.max_ctas > 0) && !getenv("AF_GEMM_NO_PERSIST")) {
    if (bn == 256 && ctx->gemm_pair && !a.max_ctas && M >= 256 && N >= 256)
      return launch_pair(ctx, A, lda, B, ldb, M, N, K, ep, st, fn);
    if (bn == 256) return launch_persistent<256>(ctx, A, lda, B, ldb, M, N, K, ep, st, fn, a.max_ctas);
    return launch_persistent<128>(ctx, A, lda, B, ldb, M, N, K, ep, st, fn, a.max_ctas);
  }
  if (a.pair && (MODE == kBF16 || MODE == kTF32P) && M > 128) {
    // CTA pairs: 256-row tiles (the caller chose width and splits)
    if constexpr (MODE == kBF16 || MODE == kTF32P) {
      switch (bn) {
        case 256:
          return launch_pair_split<256, MODE>(ctx, A, A2, lda, B, B2, ldb, M, N, K, splits, ep, st, fn, pdl);
        case 128:
          return launch_pair_split<128, MODE>(ctx, A, A2, lda, B, B2, ldb, M, N, K, splits, ep, st, fn, pdl);
        case 64:
          return launch_pair_split<64, MODE>(ctx, A, A2, lda, B, B2, ldb, M, N, K, splits, ep, st, fn, pdl);
        default:
          break;
      }
    }
  }
#define AF_LAUNCH(BNV) \
  return launch_tc<BNV, MODE>(ctx, A, A2, lda, B, B2, ldb, M, N, K, splits, ep, st, fn, pdl)
  switch (bn) {
    case 256:
      if constexpr (MODE != kTF32S) AF_LAUNCH(256);
      break;
    case 128:
      AF_LAUNCH(128);
    case 96:
      if constexpr (MODE == kTF32P) AF_LAUNCH(96);
      break;
    case 64:
      AF_LAUNCH(64);
    case 32:
      AF_LAUNCH(32);
    case 16:
      if constexpr (MODE == kBF16) AF_LAUNCH(16);
      break;
  }
#undef AF_LAUNCH
  return af::fail(AF_ERR_ARG, "%s: no tile for N=%d", fn, N);
}

}  // namespace

namespace af {

// Dispatches a tensor-core GEMM.  Operands must be K-major with 16-byte
// aligned bases and row strides; callers fall back to the SIMT GEMM
// otherwise (check tc_gemm_ok first).
bool tc_gemm_ok(const void *A, int64_t lda, const void *B, int64_t ldb, int K, bool fp32) {
  const int elem = fp32 ? 4 : 2;
  return aligned16(A) && aligned16(B) && (lda * elem) % 16 == 0 && (ldb * elem) % 16 == 0 && K > 0 &&
         ((int64_t)K * elem) % 16 == 0;
}

int tc_gemm(af_ctx *ctx, const void *A, int64_t lda, const void *B, int64_t ldb, int M, int N, int K, bool fp32,
            const GemmEpilogueArgs &a, cudaStream_t st, const char *fn) {
  if (fp32) return dispatch<kTF32S>(ctx, A, nullptr, lda, B, nullptr, ldb, M, N, K, a, st, fn);
  return dispatch<kBF16>(ctx, A, nullptr, lda, B, nullptr, ldb, M, N, K, a, st, fn);
}

// fp32 GEMM from operands split beforehand into (hi, lo) pairs.
int tc_gemm_presplit(af_ctx *ctx, const float *A_hi, const float *A_lo, int64_t lda, const float *B_hi,
                     const float *B_lo, int64_t ldb, int M, int N, int K, const GemmEpilogueArgs &a, cudaStream_t st,
                     const char *fn) {
  if (!tc_gemm_ok(A_lo, lda, B_lo, ldb, K, true) || !tc_gemm_ok(A_hi, lda, B_hi, ldb, K, true))
    return fail(AF_ERR_ARG, "%s: split operands must be 16-byte aligned with K %% 4 == 0", fn);
  return dispatch<kTF32P>(ctx, A_hi, A_lo, lda, B_hi, B_lo, ldb, M, N, K, a, st, fn);
}

int split_tf32(af_ctx *ctx, const float *src, float *hi, float *lo, int64_t n, cudaStream_t st, const char *fn,
               float *zero, bool pdl) {
  if (n == 0) return AF_OK;
  if (n % 4 == 0 && aligned16(src) && aligned16(hi) && aligned16(lo) && (!zero || aligned16(zero))) {
    const int64_t n4 = n / 4;
    int64_t blocks = (n4 + 255) / 256;
    if (blocks > (int64_t)ctx->num_sms * 8) blocks = (int64_t)ctx->num_sms * 8;
    const cudaError_t e = launch_kernel(split_tf32_vec_kernel, dim3((unsigned)blocks), dim3(256), 0, st, pdl && ctx->pdl,
                                        reinterpret_cast<const float4 *>(src), reinterpret_cast<float4 *>(hi),
                                        reinterpret_cast<float4 *>(lo), reinterpret_cast<float4 *>(zero), n4);
    if (e != cudaSuccess) return fail(AF_ERR_CUDA, "%s: launch: %s", fn, cudaGetErrorString(e));
    return launched(ctx, fn);
  }
  if (zero) AF_CUDA(cudaMemsetAsync(zero, 0, (size_t)n * sizeof(float), st), fn);
  int64_t blocks = (n + 255) / 256;
  if (blocks > (int64_t)ctx->num_sms * 16) blocks = (int64_t)ctx->num_sms * 16;
  split_tf32_kernel<<<(unsigned)blocks, 256, 0, st>>>(src, hi, lo, n);
  return launched(ctx, fn);
}

}  // namespace af

extern "C" int af_split_tf32(af_ctx *ctx, const float *src, float *hi, float *lo, int64_t n, af_stream_t stream) {
  const char *fn = "af_split_tf32";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(src && hi && lo && n >= 0, "af_split_tf32", "bad arguments");
  return af::split_tf32(ctx, src, hi, lo, n, af::stream_of(stream), fn);
}

extern "C" int af_linear_f32_split(af_ctx *ctx, const float *x_hi, const float *x_lo, const float *w_hi,
                                   const float *w_lo, const float *bias, float *y, int M, int N, int K,
                                   af_stream_t stream) {
  const char *fn = "af_linear_f32_split";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(x_hi && x_lo && w_hi && w_lo && y, "af_linear_f32_split", "null pointer");
  AF_REQUIRE(M >= 0 && N >= 0 && K > 0 && M <= 65535 * 128, "af_linear_f32_split", "bad sizes M=%d N=%d K=%d", M,
             N, K);
  af::GemmEpilogueArgs ep;
  ep.out = y;
  ep.ldo = N;
  ep.bias = bias;
  return af::tc_gemm_presplit(ctx, x_hi, x_lo, K, w_hi, w_lo, K, M, N, K, ep, af::stream_of(stream), fn);
}

extern "C" int af_gemm_bf16(af_ctx *ctx, const uint16_t *A, int64_t lda, int a_kblock, const uint16_t *B,
                            int64_t ldb, int M, int N, int K, void *out, int64_t ldo, int out_bf16, const float *bias,
                            const float *residual, int64_t ldr, const float *row_sumsq, int nparts, int parts_block,
                            float inv_d, float eps, int accumulate, af_stream_t stream) {
  const char *fn = "af_gemm_bf16";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(A && B && out, "af_gemm_bf16", "null pointer");
  AF_REQUIRE(M >= 0 && N >= 0 && K > 0 && M <= 65535 * 128, "af_gemm_bf16", "bad sizes M=%d N=%d K=%d", M, N, K);
  AF_REQUIRE(lda >= (a_kblock ? a_kblock : K) && ldb >= K && ldo >= N && af::tc_gemm_ok(A, lda, B, ldb, K, false),
             "af_gemm_bf16", "operands must be K-major with 16-byte aligned rows (K %% 8 == 0)");
  AF_REQUIRE(!accumulate || !out_bf16, "af_gemm_bf16", "accumulation needs an fp32 output");
  af::GemmEpilogueArgs ep;
  ep.out = out;
  ep.ldo = ldo;
  ep.out_bf16 = out_bf16;
  ep.bias = bias;
  ep.residual = residual;
  ep.ldr = ldr;
  ep.row_parts = row_sumsq;
  ep.nparts = nparts;
  ep.parts_block = parts_block;
  ep.a_kblock = a_kblock;
  ep.inv_d = inv_d;
  ep.eps = eps;
  ep.accumulate = accumulate;
  return af::tc_gemm(ctx, A, lda, B, ldb, M, N, K, false, ep, af::stream_of(stream), fn);
}
