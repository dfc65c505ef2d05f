// mlm_internal.h -- context object and error plumbing shared by the CUDA
// translation units of libmetallm_cuda.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/metallm_cuda.h"

struct mlm_ctx {
  int device = 0;
  int sm_count = 0;
  int max_smem_optin = 0;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;  // the stream ops are enqueued on
  cudaEvent_t commit_event = nullptr;
  std::string last_error;
  std::mutex lock;  // serialises the synchronous helpers

  // split-K scratch of the Q4_K GEMV: one partial row-tile per (CTA, end)
  // and one arrival counter per row tile; counters return to zero after
  // every launch.
  float *gemv_partials = nullptr;
  int *gemv_counters = nullptr;  // [gemv_max_tiles] split-K, then [gemv_max_tiles / 2] pairing
  int gemv_max_ctas = 0;
  int gemv_max_tiles = 0;

  // error word written by kernels whose bounded waits ran out (mapped
  // pinned host memory: the host reads it after a wait without a copy)
  volatile int *host_status = nullptr;
  int *dev_status = nullptr;

  // split-K scratch of decode attention
  float *attn_partials = nullptr;
  size_t attn_partials_floats = 0;
  int *attn_arrivals = nullptr;  // per (sequence, KV head); zero between launches

  // stream-K hand-off flags of the prefill GEMM, one per output tile; zero
  // between launches (each launch's waiters count them back down)
  int *gemm_flags = nullptr;
  int gemm_max_tiles = 0;

  // device-wide argmax: the running 64-bit key and the CTA ticket, zero
  // between launches
  unsigned long long *argmax_scratch = nullptr;
  // tensor parallelism (mlm_tp_init): an NCCL communicator over the ranks,
  // one context per rank
  void *tp_comm = nullptr;  // ncclComm_t
  int tp_rank = 0, tp_size = 1;
  // one-shot all-reduce over NVLink peer memory (tp.cu): every rank's
  // receive area (its own, then the other ranks' IPC mappings), each CTA's
  // epoch counter
  bool ar_ready = false;
  void *ar_peer[8] = {};
  void *ar_own = nullptr;
  int *ar_epoch = nullptr;
};

namespace mlm {

int set_error(mlm_ctx *ctx, int code, const char *fmt, ...)
    __attribute__((format(printf, 3, 4)));
int check_launch(mlm_ctx *ctx, const char *what);
int q6k_init(mlm_ctx *ctx);  // q6k.cu: the GEMV's shared-memory limit
struct GemvInput;
// the Q6_K decode GEMV with the Q4_K GEMV's x modes (cols a multiple of 2048)
int q6k_gemv_launch(mlm_ctx *ctx, const void *W, int rows, int cols, const GemvInput &in,
                    float *y, const float *residual, cudaStream_t stream);
int q6k_dequant_bf16_launch(mlm_ctx *ctx, const void *blocks, void *out, uint64_t n,
                            cudaStream_t stream);
int interleave_rows_launch(mlm_ctx *ctx, const float *a, int ra, const float *b, int rb, int T,
                           float *out, cudaStream_t stream);
// the prompt GEMM on a bf16 weight [rows][cols] (tokens of bf16 x)
int gemm_dense_launch(mlm_ctx *ctx, const void *W_bf16, int rows, int cols, const void *x_bf16,
                      int tokens, float *y, const float *residual, cudaStream_t stream);
// the same for a Q6_K weight, dequantized to bf16 into scratch (rows x cols)
int q6k_gemm_launch(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_bf16,
                    int tokens, float *y, const float *residual, void *scratch_bf16,
                    cudaStream_t stream);

// Launch as a programmatic dependent of the previous kernel on the stream:
// the grid may be scheduled once every CTA of that kernel has executed
// griddepcontrol.launch_dependents (or exited), and must execute
// griddepcontrol.wait before it reads anything that kernel writes.  Every
// kernel of the decode step does both, so the launch latency of each kernel
// and the weight prefetch of each GEMV overlap the kernel before it.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// status of a launch_pdl call (clears the error it may have left)
inline int check_launch_pdl(mlm_ctx *ctx, cudaError_t e, const char *what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(ctx, MLM_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  return check_launch(ctx, what);
}

// Kernel launchers shared between translation units (stream-ordered; each
// returns an MLM_* status and records the reason in ctx on failure).
// The x of a Q4_K GEMV, staged by the kernel into fp16 values with one scale
// per 32-element sub-block:
//  kHalf     x = x_f16 (times x_scale[k/32] when x_scale is set);
//  kRmsNorm  x = fp16(a * rms_scale(a) * w): the RMSNorm of an fp32 hidden
//            state a with fp32 weights b (NormalizationKernels.metal:31-79),
//            computed by every CTA, so no separate norm kernel runs;
//  kSwiGLU   x = silu(a) * b from fp32 gate a and up b, stored with a
//            power-of-two scale per 32 elements.
struct GemvInput {
  enum Mode { kHalf = 0, kRmsNorm = 1, kSwiGLU = 2 };
  int mode = kHalf;
  const void *x_f16 = nullptr;
  const float *x_scale = nullptr;
  const float *a = nullptr;
  const float *b = nullptr;
  float eps = 0.f;
};
inline GemvInput gemv_half(const void *x, const float *x_scale = nullptr) {
  GemvInput in;
  in.x_f16 = x;
  in.x_scale = x_scale;
  return in;
}
int gemv_validate(mlm_ctx *ctx, const void *W, int rows, int cols, const GemvInput &in,
                  float *y);
// Gate/up pairing of a decode GEMV over [gate rows; up rows]: once both
// tiles t and t + rows / 64 of y are stored, the warp that stores the second
// one also writes h = silu(gate) * up of those 32 elements in the scaled fp16
// form of mlm_silu_mul_scaled (h_f16, one scale per 32), so the down
// projection stages a plain fp16 x.  counters: rows / 64 ints, zero between
// launches (the second arrival re-zeroes its own).
struct GemvPair {
  void *h_f16 = nullptr;  // fp16 [rows / 2]
  float *h_scale = nullptr;
  int *counters = nullptr;
};
// TMA map of a Q4_K weight as a 2D byte tensor [rows][cols / 256 * 144] with
// boxes of one block column x box_rows rows (rows past the end read as zero)
int encode_q4k_rows_map(mlm_ctx *ctx, const void *W, int rows, int nb, int box_rows,
                        CUtensorMap *map);
int gemv_launch(mlm_ctx *ctx, const void *W, int rows, int cols, const GemvInput &in, float *y,
                const float *residual, float *partials, int *counters, int max_ctas,
                int max_tiles, cudaStream_t stream, const GemvPair *pair = nullptr);
int rmsnorm_f32_launch(mlm_ctx *ctx, const float *x, const float *w, float *y32, void *y16,
                       int rows, int n, float eps, cudaStream_t stream);
int rope_qk_kv_launch(mlm_ctx *ctx, const float *q, const float *k, const float *v,
                      const float *freqs, const mlm_rope_args &a, int nq, int nkv, int d,
                      void *q_out, void *kc, void *vc, int pos, cudaStream_t stream,
                      const int *pos_dev);
// one decode step of one sequence with RoPE and the KV append folded in:
// qkv = the QKV projection in fp32 (q, then k, then v), the position at
// pos_dev; appends row pos_dev[0] to kc/vc (capacity positions) and writes
// the fp16 attention output [n_heads][128]
int attn_rope_decode_launch(mlm_ctx *ctx, const float *qkv, const float *freqs,
                            const mlm_rope_args &ra, int n_heads, int n_kv, int head_dim,
                            int capacity, void *kc, void *vc, void *out, cudaStream_t stream,
                            const int *pos_dev);
// the same for a batch of sequences, one new token each: sequence b reads
// qkv + b qkv_bs, the caches at b kv_bs elements, position pos_dev[b], and
// writes its bf16 output [n_heads][128] at out_bf16 + b n_heads 128
int attn_rope_decode_batch_launch(mlm_ctx *ctx, const float *qkv, size_t qkv_bs,
                                  const float *freqs, const mlm_rope_args &ra, int n_heads,
                                  int n_kv, int head_dim, int capacity, int batch, size_t kv_bs,
                                  void *kc, void *vc, void *out_bf16, cudaStream_t stream,
                                  const int *pos_dev);
int attn_decode_launch(mlm_ctx *ctx, const void *q, const void *kc, const void *vc, int n_heads,
                       int n_kv, int head_dim, int seq_len, void *out, float *partials,
                       size_t partial_floats, cudaStream_t stream, const int *pos_dev);
int silu_mul_launch(mlm_ctx *ctx, const float *g, const float *u, void *out, int n,
                    cudaStream_t stream);
// decode linears of a batch of up to 8 tokens (q4k_gemv_batch.cu): Y[t] =
// W X[t] (+ residual, which may be Y itself), X bf16 [tokens][cols]
// y_zeroed: y is known to be zero already (no residual): skips the memset
int gemv_batch_launch(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_bf16,
                      int tokens, float *y, const float *residual, cudaStream_t stream,
                      bool y_zeroed = false);
// batched prompt pass (prefill.cu, q4k_gemm.cu)
int gemm_launch(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_bf16, int tokens,
                float *y, const float *residual, cudaStream_t stream);
int embed_rows_launch(mlm_ctx *ctx, const void *table, int vocab, int dim, const int32_t *tokens,
                      int T, float *out, cudaStream_t stream);
int rmsnorm_rows_bf16_launch(mlm_ctx *ctx, const float *x, const float *w, void *y, int rows,
                             int n, float eps, cudaStream_t stream, float *zero = nullptr,
                             size_t zero_n = 0);
int rope_kv_rows_launch(mlm_ctx *ctx, const float *qkv, const float *freqs, const mlm_rope_args &a,
                        int nq, int nkv, int d, int pos0, int T, void *q_out, void *kc, void *vc,
                        cudaStream_t stream);
int attn_prefill_launch(mlm_ctx *ctx, const void *q16, const void *kc, const void *vc, int pos0,
                        int T, int n_heads, int n_kv, int head_dim, void *out, cudaStream_t stream);
int swiglu_rows_bf16_launch(mlm_ctx *ctx, const float *gu, int ffn, int T, void *out,
                            cudaStream_t stream);
int silu_mul_scaled_launch(mlm_ctx *ctx, const float *g, const float *u, void *out, float *scale,
                           int n, cudaStream_t stream);
int argmax_launch(mlm_ctx *ctx, const float *x, int n, int32_t *out, cudaStream_t stream);
// argmax of x[0..n) as a 64-bit key (value order, then ~(index + offset)),
// for combining the argmaxes of vocabulary shards; argmax_keys_launch then
// writes the index of the largest of `nkeys` keys
int argmax_key_launch(mlm_ctx *ctx, const float *x, int n, int offset, unsigned long long *key,
                      cudaStream_t stream);
int argmax_keys_launch(mlm_ctx *ctx, const unsigned long long *keys, int nkeys, int32_t *out,
                       cudaStream_t stream);
int argmax_keys_rows_launch(mlm_ctx *ctx, const unsigned long long *keys, int nkeys, int rows,
                            int32_t *out, cudaStream_t stream);
// NCCL collectives on ctx->tp_comm (tp.cu)
int tp_allreduce_sum(mlm_ctx *ctx, const float *send, float *recv, size_t count,
                     cudaStream_t stream);
int tp_allgather_bytes(mlm_ctx *ctx, const void *send, void *recv, size_t bytes,
                       cudaStream_t stream);
void tp_destroy(mlm_ctx *ctx);
int embed_launch(mlm_ctx *ctx, const void *table, int vocab, int dim, const int32_t *tok,
                 float *out, cudaStream_t stream);

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned4(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

}  // namespace mlm

#define MLM_CHECK_CTX(ctx) \
  do {                     \
    if (!(ctx)) return MLM_ERR_ARG; \
  } while (0)

#define MLM_REQUIRE(ctx, cond, code, ...)                   \
  do {                                                     \
    if (!(cond)) return mlm::set_error((ctx), (code), __VA_ARGS__); \
  } while (0)

#define MLM_CUDA_TRY(ctx, call)                                                     \
  do {                                                                              \
    cudaError_t e_ = (call);                                                        \
    if (e_ != cudaSuccess)                                                          \
      return mlm::set_error((ctx), MLM_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)
