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
// stores its slice of the partial into slot [rank] of every rank's area,
// then raises its flag there (the value is CTA c's epoch, a device counter
// that advances with every call, so a captured graph replays correctly);
// it waits (bounded) for the flags of CTA c of every rank in its own area
// and adds the slots in rank order, so every rank computes the same sum
// bit for bit.  Two areas alternate by epoch parity: a rank can only start
// call e+2 after every rank's part of call e+1 arrived, which each rank
// sends only after it finished reading call e.  Larger reductions (the
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
constexpr int kArCtas = 16;
constexpr int kArThreads = 256;
// receive area: data [2][ranks][kArMaxFloats] floats, then flags
// [2][ranks][kArCtas] ints
constexpr size_t kArDataFloats = (size_t)2 * kArMaxRanks * kArMaxFloats;
constexpr size_t kArBytes = kArDataFloats * sizeof(float) + 2 * kArMaxRanks * kArCtas * sizeof(int);

struct ArPeers {
  float *area[kArMaxRanks];
};

__device__ __forceinline__ int *ar_flags(float *area) {
  return reinterpret_cast<int *>(area + kArDataFloats);
}

__global__ void __launch_bounds__(kArThreads) ar_oneshot_kernel(const float *__restrict__ send,
                                                               float *__restrict__ recv, int count,
                                                               ArPeers peers, int rank, int nranks,
                                                               int *epoch, int *status) {
  __shared__ int s_e, s_ok;
  const int c = blockIdx.x;
  if (threadIdx.x == 0) {
    s_e = epoch[c] + 1;
    s_ok = 1;
  }
  __syncthreads();
  const int e = s_e, par = e & 1;
  // this CTA's slice, in float4s
  const int n4 = count >> 2, per = (n4 + kArCtas - 1) / kArCtas;
  const int lo = c * per, hi = min(n4, lo + per);
  const float4 *src = reinterpret_cast<const float4 *>(send);
  for (int p = 0; p < nranks; ++p) {
    float4 *dst = reinterpret_cast<float4 *>(peers.area[p] +
                                             ((size_t)par * kArMaxRanks + rank) * kArMaxFloats);
    for (int i = lo + threadIdx.x; i < hi; i += kArThreads) dst[i] = src[i];
  }
  // the barrier orders the CTA's stores before the flag's release store, and a
  // release is cumulative over what the releasing thread has observed
  __syncthreads();
  if (threadIdx.x < nranks) {  // raise this CTA's flag in rank threadIdx.x's area
    int *f = ar_flags(peers.area[threadIdx.x]) + ((size_t)par * kArMaxRanks + rank) * kArCtas + c;
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(f), "r"(e) : "memory");
  }
  if (threadIdx.x < nranks) {  // wait for source rank threadIdx.x in this rank's area
    const int *f = ar_flags(peers.area[rank]) +
                   ((size_t)par * kArMaxRanks + threadIdx.x) * kArCtas + c;
    const unsigned long long t0 = global_ns();
    for (int spin = 0;; ++spin) {
      int v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if (v == e) break;
      if ((spin & 255) == 255) {  // check the budget now and then; sleep once spinning is long
        if (global_ns() - t0 > kWaitBudgetNs) {
          atomicExch(status, MLM_ERR_TIMEOUT);
          s_ok = 0;
          break;
        }
        if (spin > 4096) __nanosleep(64);
      }
    }
  }
  __syncthreads();
  if (s_ok) {
    const float *mine = peers.area[rank] + (size_t)par * kArMaxRanks * kArMaxFloats;
    for (int i = lo + threadIdx.x; i < hi; i += kArThreads) {
      float4 a = __ldcg(reinterpret_cast<const float4 *>(mine) + i);
      for (int r = 1; r < nranks; ++r) {
        const float4 b = __ldcg(reinterpret_cast<const float4 *>(mine + (size_t)r * kArMaxFloats) + i);
        a.x += b.x;
        a.y += b.y;
        a.z += b.z;
        a.w += b.w;
      }
      reinterpret_cast<float4 *>(recv)[i] = a;
    }
  }
  if (threadIdx.x == 0) epoch[c] = e;
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
      ctx->ar_peer[p] = static_cast<float *>(ctx->ar_own);
      continue;
    }
    void *ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, all[p], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      return set_error(ctx, MLM_ERR_CUDA, "mlm_tp_init: opening rank %d's receive area", p);
    }
    ctx->ar_peer[p] = static_cast<float *>(ptr);
  }
  ctx->ar_ready = true;
  return MLM_OK;
}

}  // namespace

int tp_allreduce_sum(mlm_ctx *ctx, const float *send, float *recv, size_t count,
                     cudaStream_t stream) {
  if (ctx->ar_ready && count <= (size_t)kArMaxFloats && count % 4 == 0 && aligned16(send) &&
      aligned16(recv)) {
    ArPeers peers{};
    for (int p = 0; p < ctx->tp_size; ++p) peers.area[p] = ctx->ar_peer[p];
    ar_oneshot_kernel<<<kArCtas, kArThreads, 0, stream>>>(send, recv, (int)count, peers,
                                                          ctx->tp_rank, ctx->tp_size,
                                                          ctx->ar_epoch, ctx->dev_status);
    return check_launch(ctx, "one-shot all-reduce");
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
