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
//
// Small sum all-reduces (a decode step's hidden state, 32 KB on the 70B
// shape, 160 of them per token) are latency-bound in NCCL; they run instead
// as one kernel over NVLink peer memory ("one-shot"): every rank has a
// receive area with one slot per source rank, mapped into the other ranks'
// address spaces through CUDA IPC when the group forms.  CTA c of each rank
// stores its slice of the partial into slot [rank] of every rank's area as
// 8-byte words (value, epoch) -- the epoch is CTA c's device counter, which
// advances with every call, so a captured graph replays correctly -- then
// polls (bounded) its own area until every rank's words of its slice carry
// the epoch, and adds them in rank order, so every rank computes the same
// sum bit for bit.  Two areas alternate by epoch parity: a rank can only
// start call e+2 after every rank's part of call e+1 arrived, which each
// rank sends only after it finished reading call e.  Larger reductions (the
// prompt pass) go to NCCL.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "mlm_internal.h"
#include "q4k_gemv_common.cuh"

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

// ---- one-shot all-reduce ----------------------------------------------------

constexpr int kArMaxRanks = 8;
constexpr int kArMaxFloats = 64 * 1024;  // per call: 256 KB of fp32
constexpr int kArCtas = 64;  // CTAs storing to the peers: a batch's 256 KB needs the store rate
constexpr int kArThreads = 256;
// receive area: [2 parities][ranks][kArMaxFloats] 8-byte words, each the
// value's bits and the epoch that wrote it
constexpr size_t kArWords = (size_t)2 * kArMaxRanks * kArMaxFloats;
constexpr size_t kArBytes = kArWords * sizeof(uint2);

struct ArPeers {
  uint2 *area[kArMaxRanks];
};

// Each word carries its own epoch: an aligned 8-byte store is single-copy
// atomic, so a receiver that sees epoch e in a word sees the value stored
// with it, and no fence or separate flag is needed.
__global__ void __launch_bounds__(kArThreads) ar_oneshot_kernel(const float *__restrict__ send,
                                                               float *__restrict__ recv, int count,
                                                               ArPeers peers, int rank, int nranks,
                                                               int *epoch, int *status) {
  __shared__ int s_e;
  const int c = blockIdx.x;
  // launched as a programmatic dependent of the kernel that wrote `send`: the
  // epoch was last written two launches back, which that kernel waited for
  // before it let this one start; `send` is read only after the wait.  The
  // kernel after this one (the next GEMV) may start streaming its weights
  // while this one exchanges; it waits for this grid before reading `recv`.
  if (threadIdx.x == 0) s_e = epoch[c] + 1;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  __syncthreads();
  const uint32_t e = (uint32_t)s_e;
  const size_t par = e & 1;
  const int per = (count + kArCtas - 1) / kArCtas;
  const int lo = c * per, hi = min(count, lo + per);
  for (int i = lo + threadIdx.x; i < hi; i += kArThreads) {
    const uint2 w = make_uint2(__float_as_uint(send[i]), e);
    for (int p = 0; p < nranks; ++p) {
      uint2 *dst = peers.area[p] + (par * kArMaxRanks + rank) * kArMaxFloats + i;
      asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(dst), "r"(w.x), "r"(w.y)
                   : "memory");
    }
  }
  const uint2 *mine = peers.area[rank] + par * kArMaxRanks * kArMaxFloats;
  bool ok = true;
  for (int i = lo + threadIdx.x; i < hi; i += kArThreads) {
    float acc = 0.f;
    for (int r = 0; r < nranks && ok; ++r) {  // rank order: every rank sums alike
      const uint2 *src = mine + (size_t)r * kArMaxFloats + i;
      uint32_t v, f;
      asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v), "=r"(f) : "l"(src)
                   : "memory");
      if (f != e) {
        const unsigned long long t0 = global_ns();
        for (int spin = 0; f != e; ++spin) {
          asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v), "=r"(f) : "l"(src)
                       : "memory");
          if ((spin & 255) == 255 && global_ns() - t0 > kWaitBudgetNs) {
            atomicExch(status, MLM_ERR_TIMEOUT);
            ok = false;
            break;
          }
        }
      }
      acc += __uint_as_float(v);
    }
    if (!ok) break;
    recv[i] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) epoch[c] = (int)e;
}

// maps every rank's receive area: IPC handles travel by an NCCL all-gather
int ar_setup(mlm_ctx *ctx) {
  const char *env = std::getenv("MLM_TP_ONESHOT");
  if ((env && env[0] == '0') || ctx->tp_size > kArMaxRanks) return MLM_OK;
  MLM_CUDA_TRY(ctx, cudaMalloc(&ctx->ar_own, kArBytes));
  MLM_CUDA_TRY(ctx, cudaMemset(ctx->ar_own, 0, kArBytes));
  MLM_CUDA_TRY(ctx, cudaMalloc(&ctx->ar_epoch, sizeof(int) * kArCtas));
  MLM_CUDA_TRY(ctx, cudaMemset(ctx->ar_epoch, 0, sizeof(int) * kArCtas));
  cudaIpcMemHandle_t h;
  MLM_CUDA_TRY(ctx, cudaIpcGetMemHandle(&h, ctx->ar_own));
  const int n = ctx->tp_size;
  void *dev = nullptr;
  MLM_CUDA_TRY(ctx, cudaMalloc(&dev, sizeof(h) * (n + 1)));
  std::vector<cudaIpcMemHandle_t> all(n);
  int st = MLM_OK;
  if (cudaMemcpy(dev, &h, sizeof(h), cudaMemcpyHostToDevice) != cudaSuccess)
    st = set_error(ctx, MLM_ERR_CUDA, "mlm_tp_init: handle upload");
  if (st == MLM_OK)
    st = tp_allgather_bytes(ctx, dev, static_cast<char *>(dev) + sizeof(h), sizeof(h),
                            ctx->stream);
  if (st == MLM_OK &&
      (cudaStreamSynchronize(ctx->stream) != cudaSuccess ||
       cudaMemcpy(all.data(), static_cast<char *>(dev) + sizeof(h), sizeof(h) * n,
                  cudaMemcpyDeviceToHost) != cudaSuccess))
    st = set_error(ctx, MLM_ERR_CUDA, "mlm_tp_init: handle exchange");
  cudaFree(dev);
  if (st != MLM_OK) return st;
  for (int p = 0; p < n; ++p) {
    if (p == ctx->tp_rank) {
      ctx->ar_peer[p] = ctx->ar_own;
      continue;
    }
    void *ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, all[p], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      return set_error(ctx, MLM_ERR_CUDA, "mlm_tp_init: opening rank %d's receive area", p);
    }
    ctx->ar_peer[p] = ptr;
  }
  ctx->ar_ready = true;
  return MLM_OK;
}

}  // namespace

int tp_allreduce_sum(mlm_ctx *ctx, const float *send, float *recv, size_t count,
                     cudaStream_t stream) {
  if (ctx->ar_ready && count <= (size_t)kArMaxFloats) {
    ArPeers peers{};
    for (int p = 0; p < ctx->tp_size; ++p) peers.area[p] = static_cast<uint2 *>(ctx->ar_peer[p]);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kArCtas);
    cfg.blockDim = dim3(kArThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, ar_oneshot_kernel, send, recv, (int)count,
                                             peers, ctx->tp_rank, ctx->tp_size, ctx->ar_epoch,
                                             ctx->dev_status);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return set_error(ctx, MLM_ERR_CUDA, "one-shot all-reduce: launch failed: %s",
                       cudaGetErrorString(e));
    }
    return MLM_OK;
  }
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
  for (int p = 0; p < 8; ++p)
    if (ctx->ar_peer[p] && ctx->ar_peer[p] != ctx->ar_own) cudaIpcCloseMemHandle(ctx->ar_peer[p]);
  for (int p = 0; p < 8; ++p) ctx->ar_peer[p] = nullptr;
  if (ctx->ar_own) cudaFree(ctx->ar_own);
  if (ctx->ar_epoch) cudaFree(ctx->ar_epoch);
  ctx->ar_own = nullptr;
  ctx->ar_epoch = nullptr;
  ctx->ar_ready = false;
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
  st = ar_setup(ctx);
  if (st != MLM_OK) tp_destroy(ctx);
  return st;
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
