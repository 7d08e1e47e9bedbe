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
                            const float *state_in, float *state_out, void *out, int out_bf16, af_stream_t stream) {
  const char *fn = "af_prefill_head_sharded";
  AF_ENTER(ctx, fn);
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
  const int parts = Hl * af::chunkwise_parts();
  const af::ChunkPlan pl = af::chunkwise_plan(ctx->num_sms, B, T, Hl, ctx->chunk_segments);
  const size_t qkv_b = align256((size_t)N * 3 * dl * 2), o_b = align256((size_t)g * N * dl * 2),
               ss_b = align256((size_t)g * N * parts * 4), seg_b = af::chunkwise_seg_state_bytes(B, Hl, pl);
  void *ws = nullptr;
  int rc = af::workspace(ctx, qkv_b + o_b + ss_b + seg_b, &ws, fn);
  if (rc) return rc;
  uint8_t *base = static_cast<uint8_t *>(ws);
  uint16_t *qkv = reinterpret_cast<uint16_t *>(base);
  uint16_t *o_all = reinterpret_cast<uint16_t *>(base + qkv_b);
  float *ss_all = reinterpret_cast<float *>(base + qkv_b + o_b);
  float *seg = seg_b ? reinterpret_cast<float *>(base + qkv_b + o_b + ss_b) : nullptr;
  uint16_t *o_mine = o_all + (size_t)r * N * dl;
  float *ss_mine = ss_all + (size_t)r * N * parts;
  cudaStream_t st = af::stream_of(stream);
  // 1. projection of this rank's heads
  af::GemmEpilogueArgs e1;
  e1.out = qkv;
  e1.ldo = 3 * dl;
  e1.out_bf16 = 1;
  rc = af::tc_gemm(ctx, x, d, w_qkv_local, d, (int)N, 3 * dl, d, false, e1, st, fn);
  if (rc) return rc;
  // 2. retention of this rank's heads into its slot of the gather buffer
  rc = af::retention_chunkwise_bf16(ctx, qkv, B, T, Hl, gamma + (size_t)r * Hl, state_in, state_out, o_mine,
                                    ret_norm_w + (size_t)r * dl, ss_mine, pl, seg, st, fn);
  if (rc) return rc;
  // 3. all-gather (in place) of head outputs and partial sums of squares
  if (g > 1) {
    ncclComm_t comm = static_cast<ncclComm_t>(ctx->comm);
    ncclResult_t nr = g_nccl.group_start();
    if (nr == ncclSuccess) nr = g_nccl.all_gather(o_mine, o_all, (size_t)N * dl, ncclBfloat16, comm, st);
    if (nr == ncclSuccess) nr = g_nccl.all_gather(ss_mine, ss_all, (size_t)N * parts, ncclFloat32, comm, st);
    const ncclResult_t ne = g_nccl.group_end();
    if (nr == ncclSuccess) nr = ne;
    if (nr != ncclSuccess) return nccl_fail(nr, fn, "ncclAllGather");
  }
  // 4. this rank's output columns: K-blocked gather buffer . W_o rows^T
  af::GemmEpilogueArgs e2;
  e2.out = out;
  e2.ldo = dl;
  e2.out_bf16 = out_bf16;
  e2.row_parts = ss_all;
  e2.nparts = g * parts;
  e2.parts_block = parts;
  e2.a_kblock = dl;
  e2.inv_d = 1.0f / (float)d;
  e2.eps = eps;
  return af::tc_gemm(ctx, o_all, dl, w_o_rows, d, (int)N, dl, d, false, e2, st, fn);
}

}  // extern "C"
