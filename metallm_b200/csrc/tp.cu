// tp.cu -- tensor parallelism over NCCL: one process (one mlm_ctx) per GPU,
// a communicator over the ranks, and the two collectives the sharded runner
// needs (sum all-reduce of fp32 partials, all-gather of equal slices).
//
// The reference is single-GPU Metal and has no counterpart.  NCCL is bound at
// run time (dlopen of libnccl.so.2): a process that has already loaded NCCL
// (PyTorch's build, say) keeps its copy, so the library never brings a second
// NCCL of a different version into the process; otherwise the system's
// libnccl.so.2 is loaded.  Every collective is enqueued on ctx->stream, so it
// is stream-ordered with this library's kernels and can be captured into the
// runner's CUDA graph.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "mlm_internal.h"

namespace mlm {
namespace {

struct NcclApi {
  bool loaded = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
  ncclResult_t (*GetVersion)(int *) = nullptr;
};

NcclApi g_nccl;
std::mutex g_nccl_lock;

template <class F>
bool bind(void *h, const char *name, F &fn) {
  fn = reinterpret_cast<F>(dlsym(h, name));
  return fn != nullptr;
}

int nccl_load(mlm_ctx *ctx) {
  std::lock_guard<std::mutex> g(g_nccl_lock);
  if (g_nccl.loaded) return MLM_OK;
  void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return set_error(ctx, MLM_ERR_NCCL, "mlm_tp: cannot load libnccl.so.2 (%s)", dlerror());
  NcclApi a;
  if (!bind(h, "ncclGetUniqueId", a.GetUniqueId) || !bind(h, "ncclCommInitRank", a.CommInitRank) ||
      !bind(h, "ncclAllReduce", a.AllReduce) || !bind(h, "ncclAllGather", a.AllGather) ||
      !bind(h, "ncclCommDestroy", a.CommDestroy) ||
      !bind(h, "ncclGetErrorString", a.GetErrorString) || !bind(h, "ncclGetVersion", a.GetVersion))
    return set_error(ctx, MLM_ERR_NCCL, "mlm_tp: libnccl.so.2 lacks an entry point");
  a.loaded = true;
  g_nccl = a;
  return MLM_OK;
}

int nccl_check(mlm_ctx *ctx, ncclResult_t r, const char *what) {
  if (r == ncclSuccess) return MLM_OK;
  return set_error(ctx, MLM_ERR_NCCL, "%s: %s", what, g_nccl.GetErrorString(r));
}

}  // namespace

int tp_allreduce_sum(mlm_ctx *ctx, const float *send, float *recv, size_t count,
                     cudaStream_t stream) {
  return nccl_check(ctx,
                    g_nccl.AllReduce(send, recv, count, ncclFloat32, ncclSum,
                                     reinterpret_cast<ncclComm_t>(ctx->tp_comm), stream),
                    "ncclAllReduce");
}

int tp_allgather_bytes(mlm_ctx *ctx, const void *send, void *recv, size_t bytes,
                       cudaStream_t stream) {
  return nccl_check(ctx,
                    g_nccl.AllGather(send, recv, bytes, ncclUint8,
                                     reinterpret_cast<ncclComm_t>(ctx->tp_comm), stream),
                    "ncclAllGather");
}

void tp_destroy(mlm_ctx *ctx) {
  if (ctx->tp_comm && g_nccl.loaded) g_nccl.CommDestroy(reinterpret_cast<ncclComm_t>(ctx->tp_comm));
  ctx->tp_comm = nullptr;
  ctx->tp_rank = 0;
  ctx->tp_size = 1;
}

}  // namespace mlm

using namespace mlm;

extern "C" int mlm_tp_unique_id(mlm_ctx *ctx, void *out, size_t bytes) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, out && bytes >= sizeof(ncclUniqueId), MLM_ERR_ARG,
              "mlm_tp_unique_id: need %zu bytes", sizeof(ncclUniqueId));
  int st = nccl_load(ctx);
  if (st != MLM_OK) return st;
  ncclUniqueId id;
  st = nccl_check(ctx, g_nccl.GetUniqueId(&id), "ncclGetUniqueId");
  if (st != MLM_OK) return st;
  std::memcpy(out, &id, sizeof(id));
  return MLM_OK;
}

extern "C" int mlm_tp_init(mlm_ctx *ctx, int nranks, int rank, const void *unique_id) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, unique_id && nranks >= 1 && rank >= 0 && rank < nranks, MLM_ERR_ARG,
              "mlm_tp_init: rank %d of %d", rank, nranks);
  MLM_REQUIRE(ctx, !ctx->tp_comm, MLM_ERR_STATE, "mlm_tp_init: context already has a group");
  int st = nccl_load(ctx);
  if (st != MLM_OK) return st;
  MLM_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  ncclComm_t comm = nullptr;
  st = nccl_check(ctx, g_nccl.CommInitRank(&comm, nranks, id, rank), "ncclCommInitRank");
  if (st != MLM_OK) return st;
  ctx->tp_comm = comm;
  ctx->tp_rank = rank;
  ctx->tp_size = nranks;
  return MLM_OK;
}

extern "C" int mlm_tp_info(const mlm_ctx *ctx, int *rank, int *size) {
  if (!ctx) return MLM_ERR_ARG;
  if (rank) *rank = ctx->tp_rank;
  if (size) *size = ctx->tp_comm ? ctx->tp_size : 0;
  return MLM_OK;
}

extern "C" int mlm_tp_allreduce_f32(mlm_ctx *ctx, const float *send, float *recv, size_t count) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, ctx->tp_comm, MLM_ERR_STATE, "mlm_tp_allreduce_f32: no group (mlm_tp_init)");
  MLM_REQUIRE(ctx, send && recv, MLM_ERR_ARG, "mlm_tp_allreduce_f32: null buffer");
  return tp_allreduce_sum(ctx, send, recv, count, ctx->stream);
}

extern "C" int mlm_tp_allgather(mlm_ctx *ctx, const void *send, void *recv, size_t bytes) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, ctx->tp_comm, MLM_ERR_STATE, "mlm_tp_allgather: no group (mlm_tp_init)");
  MLM_REQUIRE(ctx, send && recv, MLM_ERR_ARG, "mlm_tp_allgather: null buffer");
  return tp_allgather_bytes(ctx, send, recv, bytes, ctx->stream);
}
