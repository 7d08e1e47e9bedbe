// Head-sharded long-context prefill across the GPUs of one node (one process
// per GPU), the multi-GPU form of af_msr_prefill_bf16.
//
// Rank r of g owns heads [r*H/g, (r+1)*H/g) (dl = d/g columns of every
// projection):
//   1. qkv_r = x . W_qkv[rows of its heads]^T       bf16 GEMM over all tokens
//   2. chunkwise retention of its heads (sequence segments fill the SMs),
//      written straight into slot r of the gather buffer: O_r * ret_norm_w
//      bf16 [N][dl] and per-row partial sums of O_r^2 [N][H/g * 2]
//   3. ncclAllGather of both (in place): every rank holds all head outputs,
//      stacked by rank [g][N][dl] - a K-blocked operand
//   4. out_r = diag(1/rms) O . W_o[r*dl:(r+1)*dl]^T   one GEMM reading the
//      K-blocked gather buffer and the blocked partial sums directly; the
//      output stays column-sharded [N][dl].
// The reference computes this layer on one CPU (aceflow/nn/retention.py:
// 44-66: parallel form, RMSNorm, W_o); the result is the same, split by
// output columns.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2: the copy a PyTorch
// process has already loaded, else the system one), so the library itself
// does not depend on it.
#include "common.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

namespace {

struct NcclApi {
  bool loaded = false;
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclCommAbort) comm_abort = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclSend) send = nullptr;
  decltype(&ncclRecv) recv = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
};

NcclApi g_nccl;
std::mutex g_nccl_mu;

int load_nccl(const char *fn) {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (g_nccl.loaded) return AF_OK;
  void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return af::fail(AF_ERR_NCCL, "%s: cannot load libnccl.so.2: %s", fn, dlerror());
  NcclApi a;
#define AF_SYM(field, name)                                                            \
  a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, name));                       \
  if (!a.field) return af::fail(AF_ERR_NCCL, "%s: libnccl.so.2 lacks %s", fn, name);
  AF_SYM(get_unique_id, "ncclGetUniqueId");
  AF_SYM(comm_init_rank, "ncclCommInitRank");
  AF_SYM(comm_destroy, "ncclCommDestroy");
  AF_SYM(comm_abort, "ncclCommAbort");
  AF_SYM(all_gather, "ncclAllGather");
  AF_SYM(send, "ncclSend");
  AF_SYM(recv, "ncclRecv");
  AF_SYM(group_start, "ncclGroupStart");
  AF_SYM(group_end, "ncclGroupEnd");
  AF_SYM(error_string, "ncclGetErrorString");
#undef AF_SYM
  a.loaded = true;
  g_nccl = a;
  return AF_OK;
}

int nccl_fail(ncclResult_t r, const char *fn, const char *what) {
  return af::fail(AF_ERR_NCCL, "%s: %s: %s", fn, what, g_nccl.error_string ? g_nccl.error_string(r) : "?");
}

inline size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

// dst[n][(i * g + r) * dlg + c] = src[n][r * dl + i * dlg + c] in 16-byte
// units (dlg8 = dlg / 8 bf16 per unit): W_o rows with their columns in the
// K order of the gather buffers [G][g][N][dlg] (head group i, rank r).
__global__ void gather_wo_cols_kernel(const uint4 *__restrict__ src, uint4 *__restrict__ dst, int G, int dl, int g,
                                      int dlg8, int ld8, int dl8) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)dl * G * g * dlg8;
  if (idx >= total) return;
  const int c = (int)(idx % dlg8);
  int64_t t = idx / dlg8;
  const int rr = (int)(t % g);
  t /= g;
  const int i = (int)(t % G);
  const int n = (int)(t / G);
  dst[idx] = src[(size_t)n * ld8 + (size_t)rr * dl8 + (size_t)i * dlg8 + c];
}

}  // namespace

namespace af {

void comm_release(af_ctx *ctx) {
  if (ctx->comm && g_nccl.loaded) g_nccl.comm_destroy(static_cast<ncclComm_t>(ctx->comm));
  ctx->comm = nullptr;
  ctx->comm_nranks = ctx->comm_rank = 0;
}

}  // namespace af

extern "C" {

int af_comm_unique_id(void *id_out) {
  const char *fn = "af_comm_unique_id";
  if (!id_out) return af::fail(AF_ERR_ARG, "%s: id_out is NULL", fn);
  int rc = load_nccl(fn);
  if (rc) return rc;
  ncclUniqueId id;
  ncclResult_t r = g_nccl.get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(r, fn, "ncclGetUniqueId");
  static_assert(sizeof(ncclUniqueId) == AF_COMM_ID_BYTES, "unique id size");
  memcpy(id_out, &id, sizeof(id));
  return AF_OK;
}

int af_comm_init(af_ctx *ctx, int nranks, int rank, const void *unique_id) {
  const char *fn = "af_comm_init";
  AF_ENTER(ctx, fn);
  AF_REQUIRE(unique_id && nranks >= 1 && rank >= 0 && rank < nranks, "af_comm_init", "bad rank %d of %d", rank,
             nranks);
  int rc = load_nccl(fn);
  if (rc) return rc;
  af::comm_release(ctx);
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  ncclComm_t comm = nullptr;
  ncclResult_t r = g_nccl.comm_init_rank(&comm, nranks, id, rank);
  if (r != ncclSuccess) return nccl_fail(r, fn, "ncclCommInitRank");
  ctx->comm = comm;
  ctx->comm_nranks = nranks;
  ctx->comm_rank = rank;
  return AF_OK;
}

int af_comm_destroy(af_ctx *ctx) {
  AF_ENTER(ctx, "af_comm_destroy");
  af::comm_release(ctx);
  return AF_OK;
}

int af_prefill_head_sharded(af_ctx *ctx, const uint16_t *x, const uint16_t *w_qkv_local, const uint16_t *w_o_rows,
                            const float *ret_norm_w, const float *gamma, float eps, int B, int T, int d, int H,
                            const float *state_in, float *state_out, void *out, int out_bf16, int chunk,
                            af_stream_t stream) {
  const char *fn = "af_prefill_head_sharded";
  AF_ENTER(ctx, fn);
  int C = 0;
  if (int rc0 = af::resolve_chunk(ctx, chunk, &C, fn)) return rc0;
  AF_REQUIRE(ctx->comm, "af_prefill_head_sharded", "no communicator: call af_comm_init first");
  const int g = ctx->comm_nranks, r = ctx->comm_rank;
  const int dh = af::chunkwise_head_dim();
  AF_REQUIRE(x && w_qkv_local && w_o_rows && ret_norm_w && gamma && out, "af_prefill_head_sharded", "null pointer");
  AF_REQUIRE(B >= 0 && T >= 0 && H > 0 && d == H * dh && H % g == 0, "af_prefill_head_sharded",
             "needs head_dim %d and heads divisible by ranks (d=%d H=%d ranks=%d)", dh, d, H, g);
  AF_REQUIRE(af::aligned16(x) && af::aligned16(w_qkv_local) && af::aligned16(w_o_rows) && af::aligned16(out),
             "af_prefill_head_sharded", "x, weights and out must be 16-byte aligned");
  AF_REQUIRE((int64_t)B * T * g <= 0x7fffffffLL && (int64_t)B * T <= 65535LL * 128, "af_prefill_head_sharded",
             "B*T too large");
  if (B == 0 || T == 0) return AF_OK;
  const int Hl = H / g, dl = Hl * dh;
  const int64_t N = (int64_t)B * T;
  // Head groups: the all-gather of group i runs on a side stream while group
  // i+1 is projected and retained (the last group's gather stays exposed);
  // one W_o GEMM then reads every group's gather buffer.  Needs per-group
  // state views (one stream, or no state).  sharded_head_groups 0 = auto = 1:
  // measured on B200 at T=65536, d=4096, the overlap did not pay (8 GPUs
  // 2.151 vs 2.165 ms, 4 GPUs 3.267 vs 3.175 ms with 2 groups).
  int G = ctx->sharded_head_groups > 0 ? ctx->sharded_head_groups : 1;
  if (B > 1 && (state_in || state_out)) G = 1;
  while (G > 1 && Hl % G != 0) --G;
  if (G > af_ctx::kMaxSlices) G = af_ctx::kMaxSlices;
  const int hg = Hl / G, dlg = hg * dh, P = hg * af::chunkwise_parts(C);
  const int reserve = G > 1 && g > 1 ? ctx->comm_reserve_sms : 0;  // SMs left to the concurrent all-gather
  const af::ChunkPlan pl = af::chunkwise_plan(ctx->num_sms - reserve, B, T, hg, ctx->chunk_segments, C);
  const size_t qkv_b = align256((size_t)N * 3 * dlg * 2), o_b = align256((size_t)G * g * N * dlg * 2),
               ss_b = align256((size_t)G * g * N * P * 4), seg_b = align256(af::chunkwise_seg_state_bytes(B, hg, pl)),
               wo_b = G > 1 ? align256((size_t)dl * d * 2) : 0;
  void *ws = nullptr;
  int rc = af::workspace(ctx, qkv_b + o_b + ss_b + seg_b + wo_b, &ws, fn);
  if (rc) return rc;
  uint8_t *base = static_cast<uint8_t *>(ws);
  uint16_t *qkv = reinterpret_cast<uint16_t *>(base);
  uint16_t *o_all = reinterpret_cast<uint16_t *>(base + qkv_b);             // [G][g][N][dlg]
  float *ss_all = reinterpret_cast<float *>(base + qkv_b + o_b);            // [G][g][N][P]
  float *seg = seg_b ? reinterpret_cast<float *>(base + qkv_b + o_b + ss_b) : nullptr;
  uint16_t *wo_perm = G > 1 ? reinterpret_cast<uint16_t *>(base + qkv_b + o_b + ss_b + seg_b) : nullptr;
  cudaStream_t st = af::stream_of(stream), cs = ctx->side[0];
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->comm);
  af::mark_begin(ctx, st);
  if (G > 1) {
    // W_o rows with their columns in the gather buffers' K order
    const int64_t vec = (int64_t)G * dl * g * (dlg / 8);
    gather_wo_cols_kernel<<<(unsigned)((vec + 255) / 256), 256, 0, st>>>(
        reinterpret_cast<const uint4 *>(w_o_rows), reinterpret_cast<uint4 *>(wo_perm), G, dl, g, dlg / 8, d / 8,
        dl / 8);
    rc = af::launched(ctx, fn);
    if (rc) return rc;
  }
  for (int i = 0; i < G; ++i) {
    // 1. projections of group i's heads: q, k, v column blocks of qkv [N][3*dlg]
    for (int part = 0; part < 3; ++part) {
      af::GemmEpilogueArgs e;
      e.out = qkv + (size_t)part * dlg;
      e.ldo = 3 * dlg;
      e.out_bf16 = 1;
      e.max_ctas = i > 0 ? ctx->num_sms - reserve : 0;
      const uint16_t *wrows = w_qkv_local + ((size_t)part * dl + (size_t)i * dlg) * d;
      rc = af::tc_gemm(ctx, x, d, wrows, d, (int)N, dlg, d, false, e, st, fn);
      if (rc) return rc;
    }
    if (G == 1) af::mark(ctx, "qkv", st);
    // 2. retention of group i into its slot of the gather buffer
    uint16_t *o_grp = o_all + (size_t)i * g * N * dlg;
    float *ss_grp = ss_all + (size_t)i * g * N * P;
    const size_t st_off = (size_t)i * hg * dh * dh;  // one stream, or no state
    rc = af::retention_chunkwise_bf16(ctx, qkv, B, T, hg, gamma + (size_t)r * Hl + (size_t)i * hg,
                                      state_in ? state_in + st_off : nullptr, state_out ? state_out + st_off : nullptr,
                                      o_grp + (size_t)r * N * dlg, ret_norm_w + (size_t)r * dl + (size_t)i * dlg,
                                      ss_grp + (size_t)r * N * P, pl, seg, st, fn);
    if (rc) return rc;
    // 3. all-gather (in place) of group i's outputs and partial sums of squares
    if (g > 1) {
      cudaStream_t as = G > 1 ? cs : st;
      if (G > 1) {
        AF_CUDA(cudaEventRecord(ctx->ev_a[i], st), fn);
        AF_CUDA(cudaStreamWaitEvent(cs, ctx->ev_a[i], 0), fn);
      }
      ncclResult_t nr = g_nccl.group_start();
      if (nr == ncclSuccess)
        nr = g_nccl.all_gather(o_grp + (size_t)r * N * dlg, o_grp, (size_t)N * dlg, ncclBfloat16, comm, as);
      if (nr == ncclSuccess)
        nr = g_nccl.all_gather(ss_grp + (size_t)r * N * P, ss_grp, (size_t)N * P, ncclFloat32, comm, as);
      const ncclResult_t ne = g_nccl.group_end();
      if (nr == ncclSuccess) nr = ne;
      if (nr != ncclSuccess) return nccl_fail(nr, fn, "ncclAllGather");
      if (G > 1) AF_CUDA(cudaEventRecord(ctx->ev_b[i], cs), fn);
    }
  }
  if (G == 1) af::mark(ctx, "allgather", st);
  const bool waits = G > 1 && g > 1;  // gathers ran on the side stream
  // 4. this rank's output columns: the gather buffers [G][g][N][dlg] as one
  //    K-blocked operand . W_o rows (columns in the same K order)^T, 1/rms
  //    per row in the epilogue
  if (waits)
    for (int i = 0; i < G; ++i) AF_CUDA(cudaStreamWaitEvent(st, ctx->ev_b[i], 0), fn);
  af::GemmEpilogueArgs e;
  e.out = out;
  e.ldo = dl;
  e.out_bf16 = out_bf16;
  e.a_kblock = dlg;
  e.row_parts = ss_all;
  e.nparts = G * g * P;
  e.parts_block = P;
  e.inv_d = 1.0f / (float)d;
  e.eps = eps;
  rc = af::tc_gemm(ctx, o_all, dlg, G > 1 ? wo_perm : w_o_rows, d, (int)N, dl, d, false, e, st, fn);
  if (rc) return rc;
  af::mark(ctx, "w_o", st);
  return AF_OK;
}

// Row-sharded variant: the exchange is an all-to-all instead of an
// all-gather.  Rank r still projects and retains its heads over all N rows,
// then sends rows [s*c, s*c + n_s) of its head outputs (and their partial
// sums of squares) to rank s and receives the other ranks' heads for its own
// rows [r*c, r*c + n_r), c = ceil(N/g): (g-1)/g^2 of the layer's bf16 output
// crosses NVLink per rank instead of the all-gather's (g-1)/g.  Its rows are
// then complete (every head), so the RMSNorm and the FULL W_o run locally:
// out [n_r][d], the layer output's rows of this rank.  The receive buffer
// [g][n_r][dl] is the K-blocked operand of the W_o GEMM (block p = rank p's
// heads = columns p*dl.. of O, W_o's natural K order).
int af_prefill_head_sharded_rows(af_ctx *ctx, const uint16_t *x, const uint16_t *w_qkv_local, const uint16_t *w_o,
                                 const float *ret_norm_w, const float *gamma, float eps, int B, int T, int d, int H,
                                 const float *state_in, float *state_out, void *out, int out_bf16, int chunk,
                                 af_stream_t stream) {
  const char *fn = "af_prefill_head_sharded_rows";
  AF_ENTER(ctx, fn);
  int C = 0;
  if (int rc0 = af::resolve_chunk(ctx, chunk, &C, fn)) return rc0;
  AF_REQUIRE(ctx->comm, "af_prefill_head_sharded_rows", "no communicator: call af_comm_init first");
  const int g = ctx->comm_nranks, r = ctx->comm_rank;
  const int dh = af::chunkwise_head_dim();
  AF_REQUIRE(x && w_qkv_local && w_o && ret_norm_w && gamma && out, "af_prefill_head_sharded_rows", "null pointer");
  AF_REQUIRE(B >= 0 && T >= 0 && H > 0 && d == H * dh && H % g == 0, "af_prefill_head_sharded_rows",
             "needs head_dim %d and heads divisible by ranks (d=%d H=%d ranks=%d)", dh, d, H, g);
  AF_REQUIRE(af::aligned16(x) && af::aligned16(w_qkv_local) && af::aligned16(w_o) && af::aligned16(out),
             "af_prefill_head_sharded_rows", "x, weights and out must be 16-byte aligned");
  AF_REQUIRE((int64_t)B * T <= 65535LL * 128, "af_prefill_head_sharded_rows", "B*T too large");
  if (B == 0 || T == 0) return AF_OK;
  const int Hl = H / g, dl = Hl * dh, P = Hl * af::chunkwise_parts(C);
  const int64_t N = (int64_t)B * T;
  const int64_t c = (N + g - 1) / g;  // rows per rank (the last ranks may hold fewer)
  auto rows_of = [&](int s) -> int64_t {
    const int64_t lo = (int64_t)s * c;
    return lo >= N ? 0 : (N - lo < c ? N - lo : c);
  };
  const int64_t nr = rows_of(r);
  // Row slabs: each rank's row block is exchanged in S slabs of cs rows; the
  // W_o GEMM of slab j runs while slab j+1 crosses NVLink on a side stream
  // (the GEMM leaves comm_reserve_sms SMs to NCCL).  0 = auto = 1: measured on
  // B200 at T=65536, d=4096, 2 GPUs, 3.79 ms per pass with one exchange
  // against 3.84 with 2 slabs and 3.89 with 4 (the exchange and the GEMM
  // slow each other more than the overlap saves).
  int S = ctx->sharded_row_slabs > 0 ? ctx->sharded_row_slabs : 1;
  if (g == 1) S = 1;
  if (S > af_ctx::kMaxSlices) S = af_ctx::kMaxSlices;
  const int64_t cs = (c + S - 1) / S;
  auto slab_rows = [&](int s, int j) -> int64_t {  // rows of slab j of rank s's block
    const int64_t ns = rows_of(s), lo = (int64_t)j * cs;
    return lo >= ns ? 0 : (ns - lo < cs ? ns - lo : cs);
  };
  const af::ChunkPlan pl = af::chunkwise_plan(ctx->num_sms, B, T, Hl, ctx->chunk_segments, C);
  const size_t qkv_b = align256((size_t)N * 3 * dl * 2), o_b = align256((size_t)N * dl * 2),
               ss_b = align256((size_t)N * P * 4), ro_b = align256((size_t)S * g * cs * dl * 2),
               rss_b = align256((size_t)S * g * cs * P * 4), seg_b = align256(af::chunkwise_seg_state_bytes(B, Hl, pl));
  void *ws = nullptr;
  int rc = af::workspace(ctx, qkv_b + o_b + ss_b + ro_b + rss_b + seg_b, &ws, fn);
  if (rc) return rc;
  uint8_t *base = static_cast<uint8_t *>(ws);
  uint16_t *qkv = reinterpret_cast<uint16_t *>(base);
  uint16_t *o_loc = reinterpret_cast<uint16_t *>(base + qkv_b);                      // [N][dl]
  float *ss_loc = reinterpret_cast<float *>(base + qkv_b + o_b);                     // [N][P]
  uint16_t *o_rows = reinterpret_cast<uint16_t *>(base + qkv_b + o_b + ss_b);        // [S][g][slab rows][dl]
  float *ss_rows = reinterpret_cast<float *>(base + qkv_b + o_b + ss_b + ro_b);      // [S][g][slab rows][P]
  float *seg = seg_b ? reinterpret_cast<float *>(base + qkv_b + o_b + ss_b + ro_b + rss_b) : nullptr;
  cudaStream_t st = af::stream_of(stream), xs = S > 1 ? ctx->side[0] : st;
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->comm);
  af::mark_begin(ctx, st);
  // 1. projections of this rank's heads
  for (int part = 0; part < 3; ++part) {
    af::GemmEpilogueArgs e;
    e.out = qkv + (size_t)part * dl;
    e.ldo = 3 * dl;
    e.out_bf16 = 1;
    rc = af::tc_gemm(ctx, x, d, w_qkv_local + (size_t)part * dl * d, d, (int)N, dl, d, false, e, st, fn);
    if (rc) return rc;
  }
  af::mark(ctx, "qkv", st);
  // 2. retention of its heads over all rows
  rc = af::retention_chunkwise_bf16(ctx, qkv, B, T, Hl, gamma + (size_t)r * Hl, state_in, state_out, o_loc,
                                    ret_norm_w + (size_t)r * dl, ss_loc, pl, seg, st, fn);
  if (rc) return rc;
  if (S > 1) {
    AF_CUDA(cudaEventRecord(ctx->ev_fork, st), fn);
    AF_CUDA(cudaStreamWaitEvent(xs, ctx->ev_fork, 0), fn);
  }
  // 3. all-to-all, slab by slab: slab j of rank s's rows goes to rank s;
  //    rank p's heads land in block p of the slab's buffer [g][slab rows]
  for (int j = 0; j < S; ++j) {
    const int64_t nrj = slab_rows(r, j);
    uint16_t *o_slab = o_rows + (size_t)j * g * cs * dl;
    float *ss_slab = ss_rows + (size_t)j * g * cs * P;
    if (g > 1) {
      ncclResult_t nr_ = g_nccl.group_start();
      for (int s2 = 0; s2 < g && nr_ == ncclSuccess; ++s2) {
        const int64_t ns = slab_rows(s2, j), row0 = (int64_t)s2 * c + (int64_t)j * cs;
        if (ns > 0) {
          nr_ = g_nccl.send(o_loc + (size_t)row0 * dl, (size_t)ns * dl, ncclBfloat16, s2, comm, xs);
          if (nr_ == ncclSuccess) nr_ = g_nccl.send(ss_loc + (size_t)row0 * P, (size_t)ns * P, ncclFloat32, s2, comm, xs);
        }
        if (nrj > 0 && nr_ == ncclSuccess) {
          nr_ = g_nccl.recv(o_slab + (size_t)s2 * nrj * dl, (size_t)nrj * dl, ncclBfloat16, s2, comm, xs);
          if (nr_ == ncclSuccess)
            nr_ = g_nccl.recv(ss_slab + (size_t)s2 * nrj * P, (size_t)nrj * P, ncclFloat32, s2, comm, xs);
        }
      }
      const ncclResult_t ne = g_nccl.group_end();
      if (nr_ == ncclSuccess) nr_ = ne;
      if (nr_ != ncclSuccess) return nccl_fail(nr_, fn, "ncclSend/ncclRecv");
      if (S > 1) AF_CUDA(cudaEventRecord(ctx->ev_a[j], xs), fn);
    } else {
      AF_CUDA(cudaMemcpyAsync(o_slab, o_loc, (size_t)N * dl * 2, cudaMemcpyDeviceToDevice, st), fn);
      AF_CUDA(cudaMemcpyAsync(ss_slab, ss_loc, (size_t)N * P * 4, cudaMemcpyDeviceToDevice, st), fn);
    }
  }
  if (S == 1) af::mark(ctx, "alltoall", st);
  // 4. this rank's rows of the output, slab by slab: RMSNorm row scale from
  //    all heads' partial sums, then the full W_o
  for (int j = 0; j < S; ++j) {
    const int64_t nrj = slab_rows(r, j);
    if (S > 1) AF_CUDA(cudaStreamWaitEvent(st, ctx->ev_a[j], 0), fn);  // every slab, so st joins the side stream
    if (nrj == 0) continue;
    af::GemmEpilogueArgs e;
    e.out = static_cast<uint8_t *>(out) + (size_t)j * cs * d * (out_bf16 ? 2 : 4);
    e.ldo = d;
    e.out_bf16 = out_bf16;
    e.a_kblock = dl;
    e.row_parts = ss_rows + (size_t)j * g * cs * P;
    e.nparts = g * P;
    e.parts_block = P;
    e.inv_d = 1.0f / (float)d;
    e.eps = eps;
    e.max_ctas = j + 1 < S ? ctx->num_sms - ctx->comm_reserve_sms : 0;  // SMs left to the next slab's exchange
    rc = af::tc_gemm(ctx, o_rows + (size_t)j * g * cs * dl, dl, w_o, d, (int)nrj, d, d, false, e, st, fn);
    if (rc) return rc;
  }
  af::mark(ctx, S > 1 ? "alltoall_w_o" : "w_o", st);
  return AF_OK;
}

}  // extern "C"
