// capi.cu -- context, memory, stream ("command buffer") and error plumbing of
// the C ABI (include/metallm_cuda.h).
//
// The reference's MetalService (MetalLM/Backend/Metal/MetalService.swift:
// 48-163) owns one device and one command queue, validates every call on the
// host and reports failure as a printed reason plus false/nil.  A context
// here owns one CUDA device, one stream and the scratch the split-K kernels
// need; failures return a negative status with the reason in
// mlm_last_error().
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>

#include "mlm_internal.h"

namespace mlm {

int gemv_init(mlm_ctx *ctx);
int attn_init(mlm_ctx *ctx);
int gemm_init(mlm_ctx *ctx);
int prefill_init(mlm_ctx *ctx);
int gemv_batch_init(mlm_ctx *ctx);
int gemv_max_ctas(int sm_count);
size_t attn_partial_floats_max(int max_heads);

int set_error(mlm_ctx *ctx, int code, const char *fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    ctx->last_error = buf;
  }
  return code;
}

int check_launch(mlm_ctx *ctx, const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(ctx, MLM_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return MLM_OK;
}

// Scratch limits: the GEMV needs one arrival counter per 32-row tile and two
// 32-float partials per CTA; attention needs (2 + 128) floats per head per
// sequence chunk.
constexpr int kMaxGemvRows = 1 << 20;
constexpr int kMaxAttnHeads = 128;

}  // namespace mlm

using namespace mlm;

extern "C" int mlm_abi_version(void) { return MLM_ABI_VERSION; }

extern "C" const char *mlm_status_string(int status) {
  switch (status) {
    case MLM_OK: return "ok";
    case MLM_ERR_ARG: return "invalid argument";
    case MLM_ERR_SHAPE: return "invalid shape";
    case MLM_ERR_ALIGN: return "misaligned pointer";
    case MLM_ERR_ALLOC: return "allocation failed";
    case MLM_ERR_CUDA: return "CUDA error";
    case MLM_ERR_NCCL: return "NCCL error";
    case MLM_ERR_TIMEOUT: return "timeout";
    case MLM_ERR_STATE: return "invalid state";
    case MLM_ERR_UNSUPPORTED: return "unsupported";
    default: return "unknown status";
  }
}

extern "C" const char *mlm_last_error(const mlm_ctx *ctx) {
  return ctx ? ctx->last_error.c_str() : "null context";
}

extern "C" int mlm_device_sm_count(const mlm_ctx *ctx) { return ctx ? ctx->sm_count : 0; }

extern "C" int mlm_create(int device, mlm_ctx **out) {
  if (!out) return MLM_ERR_ARG;
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    return MLM_ERR_CUDA;
  }
  if (device < 0 || device >= ndev) return MLM_ERR_ARG;
  mlm_ctx *ctx = new (std::nothrow) mlm_ctx();
  if (!ctx) return MLM_ERR_ALLOC;
  ctx->device = device;
  auto fail = [&](int code) {
    mlm_destroy(ctx);
    return code;
  };
  if (cudaSetDevice(device) != cudaSuccess) return fail(MLM_ERR_CUDA);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return fail(MLM_ERR_CUDA);
  if (prop.major < 10) {
    // this library is built for sm_100a only
    return fail(MLM_ERR_UNSUPPORTED);
  }
  ctx->sm_count = prop.multiProcessorCount;
  ctx->max_smem_optin = (int)prop.sharedMemPerBlockOptin;
  if (cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking) != cudaSuccess)
    return fail(MLM_ERR_CUDA);
  ctx->stream = ctx->own_stream;
  if (cudaEventCreateWithFlags(&ctx->commit_event, cudaEventDisableTiming) != cudaSuccess)
    return fail(MLM_ERR_CUDA);

  ctx->gemv_max_tiles = kMaxGemvRows / 32;
  ctx->gemv_max_ctas = gemv_max_ctas(ctx->sm_count);
  // split-K tile counters, then the gate/up pairing counters (half as many)
  const size_t counter_bytes = sizeof(int) * (ctx->gemv_max_tiles + ctx->gemv_max_tiles / 2);
  if (cudaMalloc(&ctx->gemv_counters, counter_bytes) != cudaSuccess ||
      cudaMalloc(&ctx->gemv_partials, sizeof(float) * 64 * ctx->gemv_max_ctas) != cudaSuccess)
    return fail(MLM_ERR_ALLOC);
  if (cudaMemset(ctx->gemv_counters, 0, counter_bytes) != cudaSuccess)
    return fail(MLM_ERR_CUDA);
  ctx->attn_partials_floats = attn_partial_floats_max(kMaxAttnHeads);
  if (cudaMalloc(&ctx->attn_partials, sizeof(float) * ctx->attn_partials_floats) != cudaSuccess)
    return fail(MLM_ERR_ALLOC);
  if (cudaMalloc(&ctx->argmax_scratch, 2 * sizeof(unsigned long long)) != cudaSuccess)
    return fail(MLM_ERR_ALLOC);
  if (cudaMemset(ctx->argmax_scratch, 0, 2 * sizeof(unsigned long long)) != cudaSuccess)
    return fail(MLM_ERR_CUDA);
  {
    void *hs = nullptr;
    if (cudaHostAlloc(&hs, sizeof(int), cudaHostAllocMapped) != cudaSuccess) return fail(MLM_ERR_ALLOC);
    ctx->host_status = reinterpret_cast<volatile int *>(hs);
    *ctx->host_status = 0;
    if (cudaHostGetDevicePointer(reinterpret_cast<void **>(&ctx->dev_status), hs, 0) != cudaSuccess)
      return fail(MLM_ERR_CUDA);
  }
  if (gemv_init(ctx) != MLM_OK || attn_init(ctx) != MLM_OK ||
      gemm_init(ctx) != MLM_OK || prefill_init(ctx) != MLM_OK ||
      gemv_batch_init(ctx) != MLM_OK || q6k_init(ctx) != MLM_OK)
    return fail(MLM_ERR_CUDA);
  if (cudaDeviceSynchronize() != cudaSuccess) return fail(MLM_ERR_CUDA);
  *out = ctx;
  return MLM_OK;
}

extern "C" void mlm_destroy(mlm_ctx *ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  if (ctx->own_stream) cudaStreamSynchronize(ctx->own_stream);
  tp_destroy(ctx);
  if (ctx->gemv_counters) cudaFree(ctx->gemv_counters);
  if (ctx->gemv_partials) cudaFree(ctx->gemv_partials);
  if (ctx->attn_partials) cudaFree(ctx->attn_partials);
  if (ctx->attn_arrivals) cudaFree(ctx->attn_arrivals);
  if (ctx->gemm_flags) cudaFree(ctx->gemm_flags);
  if (ctx->argmax_scratch) cudaFree(ctx->argmax_scratch);
  if (ctx->host_status) cudaFreeHost(const_cast<int *>(ctx->host_status));
  if (ctx->commit_event) cudaEventDestroy(ctx->commit_event);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
}

extern "C" int mlm_get_stream(mlm_ctx *ctx, void **stream) {
  MLM_CHECK_CTX(ctx);
  if (!stream) return set_error(ctx, MLM_ERR_ARG, "mlm_get_stream: null output");
  *stream = (void *)ctx->stream;
  return MLM_OK;
}

extern "C" int mlm_set_stream(mlm_ctx *ctx, void *stream) {
  MLM_CHECK_CTX(ctx);
  ctx->stream = stream ? (cudaStream_t)stream : ctx->own_stream;
  return MLM_OK;
}

extern "C" int mlm_alloc(mlm_ctx *ctx, size_t bytes, void **dptr) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, dptr, MLM_ERR_ARG, "mlm_alloc: null output");
  *dptr = nullptr;
  if (bytes == 0) bytes = 16;
  cudaError_t e = cudaMalloc(dptr, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(ctx, MLM_ERR_ALLOC, "mlm_alloc(%zu): %s", bytes, cudaGetErrorString(e));
  }
  return MLM_OK;
}

extern "C" int mlm_free(mlm_ctx *ctx, void *dptr) {
  MLM_CHECK_CTX(ctx);
  if (!dptr) return MLM_OK;
  MLM_CUDA_TRY(ctx, cudaFree(dptr));
  return MLM_OK;
}

extern "C" int mlm_memset(mlm_ctx *ctx, void *dptr, int value, size_t bytes) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, dptr || bytes == 0, MLM_ERR_ARG, "mlm_memset: null buffer");
  if (bytes) MLM_CUDA_TRY(ctx, cudaMemsetAsync(dptr, value, bytes, ctx->stream));
  return MLM_OK;
}

extern "C" int mlm_upload_async(mlm_ctx *ctx, void *dst, const void *src, size_t bytes) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, (dst && src) || bytes == 0, MLM_ERR_ARG, "mlm_upload: null buffer");
  if (bytes)
    MLM_CUDA_TRY(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  return MLM_OK;
}

extern "C" int mlm_download_async(mlm_ctx *ctx, void *dst, const void *src, size_t bytes) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, (dst && src) || bytes == 0, MLM_ERR_ARG, "mlm_download: null buffer");
  if (bytes)
    MLM_CUDA_TRY(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  return MLM_OK;
}

extern "C" int mlm_upload(mlm_ctx *ctx, void *dst, const void *src, size_t bytes) {
  int st = mlm_upload_async(ctx, dst, src, bytes);
  if (st != MLM_OK) return st;
  MLM_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  return MLM_OK;
}

extern "C" int mlm_download(mlm_ctx *ctx, void *dst, const void *src, size_t bytes) {
  int st = mlm_download_async(ctx, dst, src, bytes);
  if (st != MLM_OK) return st;
  MLM_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  return MLM_OK;
}

extern "C" int mlm_host_alloc(mlm_ctx *ctx, size_t bytes, void **hptr) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, hptr, MLM_ERR_ARG, "mlm_host_alloc: null output");
  cudaError_t e = cudaMallocHost(hptr, bytes ? bytes : 16);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(ctx, MLM_ERR_ALLOC, "mlm_host_alloc(%zu): %s", bytes, cudaGetErrorString(e));
  }
  return MLM_OK;
}

extern "C" int mlm_host_free(mlm_ctx *ctx, void *hptr) {
  MLM_CHECK_CTX(ctx);
  if (hptr) MLM_CUDA_TRY(ctx, cudaFreeHost(hptr));
  return MLM_OK;
}

extern "C" int mlm_commit(mlm_ctx *ctx) {
  MLM_CHECK_CTX(ctx);
  MLM_CUDA_TRY(ctx, cudaEventRecord(ctx->commit_event, ctx->stream));
  return MLM_OK;
}

extern "C" int mlm_wait(mlm_ctx *ctx) {
  MLM_CHECK_CTX(ctx);
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess)
    return set_error(ctx, MLM_ERR_CUDA, "command buffer failed: %s", cudaGetErrorString(e));
  const int dev = *ctx->host_status;
  if (dev != 0) {
    *ctx->host_status = 0;
    return set_error(ctx, dev, "command buffer failed: a kernel's bounded wait expired (%s)",
                     mlm_status_string(dev));
  }
  return MLM_OK;
}

struct mlm_graph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
};

extern "C" int mlm_graph_begin(mlm_ctx *ctx) {
  MLM_CHECK_CTX(ctx);
  MLM_CUDA_TRY(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  return MLM_OK;
}

extern "C" int mlm_graph_end(mlm_ctx *ctx, mlm_graph **out) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, out, MLM_ERR_ARG, "mlm_graph_end: null output");
  *out = nullptr;
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
  if (e != cudaSuccess) {
    cudaGetLastError();
    if (g) cudaGraphDestroy(g);
    return set_error(ctx, MLM_ERR_CUDA, "mlm_graph_end: capture failed: %s", cudaGetErrorString(e));
  }
  cudaGraphExec_t x = nullptr;
  e = cudaGraphInstantiate(&x, g, 0);
  if (e != cudaSuccess) {
    cudaGetLastError();
    cudaGraphDestroy(g);
    return set_error(ctx, MLM_ERR_CUDA, "mlm_graph_end: instantiate failed: %s",
                     cudaGetErrorString(e));
  }
  mlm_graph *mg = new (std::nothrow) mlm_graph();
  if (!mg) {
    cudaGraphExecDestroy(x);
    cudaGraphDestroy(g);
    return set_error(ctx, MLM_ERR_ALLOC, "mlm_graph_end: out of host memory");
  }
  mg->graph = g;
  mg->exec = x;
  *out = mg;
  return MLM_OK;
}

extern "C" int mlm_graph_launch(mlm_ctx *ctx, mlm_graph *graph) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, graph && graph->exec, MLM_ERR_ARG, "mlm_graph_launch: null graph");
  MLM_CUDA_TRY(ctx, cudaGraphLaunch(graph->exec, ctx->stream));
  return MLM_OK;
}

extern "C" void mlm_graph_destroy(mlm_graph *graph) {
  if (!graph) return;
  if (graph->exec) cudaGraphExecDestroy(graph->exec);
  if (graph->graph) cudaGraphDestroy(graph->graph);
  delete graph;
}

// MetalService.dequantizeQ4KM_to_f32/_f16: allocate, run, wait.
static int dequantize_sync(mlm_ctx *ctx, const void *blocks, uint64_t n, void **out,
                           size_t elem_bytes, bool f16) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, out, MLM_ERR_ARG, "mlm_dequantize_q4k: null output");
  std::lock_guard<std::mutex> guard(ctx->lock);
  *out = nullptr;
  void *buf = nullptr;
  int st = mlm_alloc(ctx, n * elem_bytes, &buf);
  if (st != MLM_OK) return st;
  st = f16 ? mlm_q4k_dequant_f16(ctx, blocks, buf, n)
           : mlm_q4k_dequant_f32(ctx, blocks, reinterpret_cast<float *>(buf), n);
  if (st == MLM_OK) st = mlm_wait(ctx);
  if (st != MLM_OK) {
    cudaFree(buf);
    return st;
  }
  *out = buf;
  return MLM_OK;
}

extern "C" int mlm_dequantize_q4k_to_f32(mlm_ctx *ctx, const void *blocks, uint64_t n,
                                         float **out) {
  return dequantize_sync(ctx, blocks, n, reinterpret_cast<void **>(out), sizeof(float), false);
}

extern "C" int mlm_dequantize_q4k_to_f16(mlm_ctx *ctx, const void *blocks, uint64_t n,
                                         void **out) {
  return dequantize_sync(ctx, blocks, n, out, 2, true);
}
