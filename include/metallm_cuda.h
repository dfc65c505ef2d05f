/*
 * metallm_cuda.h -- C ABI of libmetallm_cuda.so, the B200 (sm_100a)
 * replacement for the Metal operator layer of MetalLM.
 *
 * The reference's operator API is the Swift singleton `MetalService`
 * (MetalLM/Backend/Metal/MetalService.swift:48-66).  Each entry point below
 * names the method or call site it replaces.  A Swift host binds this header
 * through a module map; the Python package metallm_b200 binds it with ctypes.
 *
 * Conventions (mirroring MetalService):
 *  - every entry point returns an int status: MLM_OK (0) or a negative
 *    MLM_ERR_* code; the reason is kept in mlm_last_error(ctx), the way the
 *    reference prints a reason and returns false/nil;
 *  - op entry points only enqueue work on the context's stream (the
 *    reference's caller-owned command buffer) and never wait; mlm_commit /
 *    mlm_wait give the commit / waitUntilCompleted pair;
 *  - buffers are device pointers owned by the caller (mlm_alloc or any CUDA
 *    allocation on the context's device); ops allocate nothing;
 *  - one context per thread / stream.  Ops on one context are not
 *    thread-safe; the synchronous dequant helpers (mlm_dequantize_*) take a
 *    context lock so concurrent loader tasks may share a context.
 */
#ifndef METALLM_CUDA_H
#define METALLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MLM_ABI_VERSION 1

enum mlm_status {
  MLM_OK = 0,
  MLM_ERR_ARG = -1,         /* null pointer or invalid argument          */
  MLM_ERR_SHAPE = -2,       /* size / shape validation failed            */
  MLM_ERR_ALIGN = -3,       /* pointer misaligned for the kernel         */
  MLM_ERR_ALLOC = -4,       /* device allocation failed                  */
  MLM_ERR_CUDA = -5,        /* CUDA runtime error (launch or execution)  */
  MLM_ERR_NCCL = -6,        /* NCCL error                                */
  MLM_ERR_TIMEOUT = -7,     /* bounded wait expired                      */
  MLM_ERR_STATE = -8,       /* call out of order (e.g. KV cache full)    */
  MLM_ERR_UNSUPPORTED = -9, /* shape / option this build does not handle */
};

typedef struct mlm_ctx mlm_ctx;

/* ---------------------------------------------------------------------------
 * Context, memory and the command-buffer stream
 * ------------------------------------------------------------------------ */

/* MetalService.init (MetalService.swift:68-163): binds `device`, creates the
 * stream and the per-context scratch used by split-K reductions. */
int mlm_create(int device, mlm_ctx **out);
void mlm_destroy(mlm_ctx *ctx);
const char *mlm_last_error(const mlm_ctx *ctx);
const char *mlm_status_string(int status);
int mlm_abi_version(void);
int mlm_device_sm_count(const mlm_ctx *ctx);

/* The stream ops are enqueued on (a cudaStream_t).  mlm_set_stream lets a
 * caller run the ops on its own stream (NULL restores the context's). */
int mlm_get_stream(mlm_ctx *ctx, void **stream);
int mlm_set_stream(mlm_ctx *ctx, void *stream);

/* device.makeBuffer / copyMemory (ModelLoader.swift:193-210) */
int mlm_alloc(mlm_ctx *ctx, size_t bytes, void **dptr);
int mlm_free(mlm_ctx *ctx, void *dptr);
int mlm_memset(mlm_ctx *ctx, void *dptr, int value, size_t bytes);
/* synchronous copies (stream-ordered, then waited) */
int mlm_upload(mlm_ctx *ctx, void *dst, const void *src, size_t bytes);
int mlm_download(mlm_ctx *ctx, void *dst, const void *src, size_t bytes);
/* stream-ordered copies; host memory should be pinned (mlm_host_alloc) */
int mlm_upload_async(mlm_ctx *ctx, void *dst, const void *src, size_t bytes);
int mlm_download_async(mlm_ctx *ctx, void *dst, const void *src, size_t bytes);
int mlm_host_alloc(mlm_ctx *ctx, size_t bytes, void **hptr);
int mlm_host_free(mlm_ctx *ctx, void *hptr);

/* commandBuffer.commit() / waitUntilCompleted() + commandBuffer.error
 * (LlamaRunner.swift:1087-1093) */
int mlm_commit(mlm_ctx *ctx);
int mlm_wait(mlm_ctx *ctx);

/* CUDA-graph capture of the context's stream: ops enqueued between
 * mlm_graph_begin and mlm_graph_end are recorded, not run; mlm_graph_launch
 * replays them.  The decode step of the reference encodes the same op
 * sequence into a fresh command buffer for every token
 * (LlamaRunner.swift:526-1128); a captured graph replays it with one launch.
 * Synchronous calls (mlm_wait, mlm_upload, mlm_download, the mlm_dequantize_*
 * helpers) are not allowed while capturing. */
typedef struct mlm_graph mlm_graph;
int mlm_graph_begin(mlm_ctx *ctx);
int mlm_graph_end(mlm_ctx *ctx, mlm_graph **out);
int mlm_graph_launch(mlm_ctx *ctx, mlm_graph *graph);
void mlm_graph_destroy(mlm_graph *graph);

/* ---------------------------------------------------------------------------
 * Seeded synthetic data (bit-identical to the CPU oracle's generators)
 * ------------------------------------------------------------------------ */

/* Q4_K blocks [first_block, first_block + nblocks) of tensor `stream` */
int mlm_gen_q4k(mlm_ctx *ctx, uint64_t seed, uint64_t stream, uint64_t first_block,
                uint64_t nblocks, void *out);
/* rows row0 .. row0+rows, block columns kb0 .. kb0+nkb of tensor `stream`
 * (nb_full block columns in all), stored densely as [rows][nkb] blocks: the
 * shard of a tensor whose input columns are split over ranks */
int mlm_gen_q4k_sub(mlm_ctx *ctx, uint64_t seed, uint64_t stream, uint64_t nb_full, uint64_t row0,
                    uint64_t rows, uint64_t kb0, uint64_t nkb, void *out);
/* Q6_K blocks [first_block, first_block + nblocks) of tensor `stream`: the
 * 208 bytes of ql, qh and scales uniform, d = fp16(|N(0,1)| * 0.01); out
 * 2-byte aligned */
int mlm_gen_q6k(mlm_ctx *ctx, uint64_t seed, uint64_t stream, uint64_t first_block,
                uint64_t nblocks, void *out);
/* Block columns [kb0, kb0 + nkb) of rows [row0, row0 + rows) of the tensor
 * mlm_gen_q6k generates with nb_full blocks per row: a rank's column shard
 * of a generated weight. */
int mlm_gen_q6k_sub(mlm_ctx *ctx, uint64_t seed, uint64_t stream, uint64_t nb_full,
                    uint64_t row0, uint64_t rows, uint64_t kb0, uint64_t nkb, void *out);
int mlm_gen_f16(mlm_ctx *ctx, uint64_t seed, uint64_t stream, uint64_t first,
                uint64_t n, float mean, float std, void *out_f16);
int mlm_gen_f32(mlm_ctx *ctx, uint64_t seed, uint64_t stream, uint64_t first,
                uint64_t n, float mean, float std, float *out);

/* ---------------------------------------------------------------------------
 * Q4_K super-blocks: 144 bytes = fp16 d, fp16 dmin, 12 bytes of packed
 * 6-bit scales/mins, 128 bytes of 4-bit quants (DequantKernels.metal:20-27).
 * Element i of a block reads qs[i/2], low nibble when i is even.
 * ------------------------------------------------------------------------ */

#define MLM_Q4K_BLOCK_ELEMS 256
#define MLM_Q4K_BLOCK_BYTES 144

/* kernel_dequantize_q4_K_f32 (DequantKernels.metal:63-92); the body of
 * MetalService.dequantizeQ4KM_to_f32 (MetalService.swift:170-239) without
 * its allocation and wait.  Bit-exact.  `blocks` holds ceil(n/256) blocks;
 * blocks and out 16-byte aligned. */
int mlm_q4k_dequant_f32(mlm_ctx *ctx, const void *blocks, float *out, uint64_t n);
/* kernel_dequantize_q4_K_f16 (DequantKernels.metal:96-125), half arithmetic */
int mlm_q4k_dequant_f16(mlm_ctx *ctx, const void *blocks, void *out_f16, uint64_t n);
/* bf16 rounding of the exact fp32 dequant (no reference counterpart; feeds
 * the tensor-core prefill path) */
int mlm_q4k_dequant_bf16(mlm_ctx *ctx, const void *blocks, void *out_bf16, uint64_t n);

/* GGUF (ggml) Q4_K blocks -> the element order the reference's kernels and
 * every kernel here read.  A GGUF file (GGUF.swift:271-297 hands its tensor
 * bytes over unchanged) stores element 64j + l of a super-block in the low
 * nibble of qs[32j + l] for l < 32 and in the high nibble of qs[32j + l - 32]
 * otherwise; DequantKernels.metal:86-88 reads element i from qs[i / 2], low
 * nibble for even i, which garbles real files.  This byte shuffle (d, dmin
 * and scales unchanged) makes a GGUF tensor usable by every op of this
 * library; dequantizing the result equals the GGUF dequant bit for bit.
 * Stream-ordered; src == dst allowed (other overlaps are rejected); both
 * 16-byte aligned. */
int mlm_q4k_repack_canonical(mlm_ctx *ctx, const void *src, void *dst, uint64_t nblocks);

/* Q6_K (210-byte blocks: ql[128], qh[64], int8 scales[16], fp16 d;
 * block_q6_K, DequantKernels.metal:29-34).  kernel_dequantize_q6_K_f32
 * (DequantKernels.metal:131-172) as MetalService.dequantizeQ6K_to_f32
 * (MetalService.swift:318-388) calls it, without its allocation and wait:
 * out = (d * scale) * (q - 32) in fp32, bit-exact.  The fp16 and bf16 forms
 * round that fp32 value (the reference's Q6_K -> fp16 kernel,
 * DequantKernels.metal:176-215, reads another element order and is not
 * followed).  n a multiple of 256; blocks 2-byte aligned. */
int mlm_q6k_dequant_f32(mlm_ctx *ctx, const void *blocks, float *out, uint64_t n);
int mlm_q6k_dequant_f16(mlm_ctx *ctx, const void *blocks, void *out_f16, uint64_t n);
int mlm_q6k_dequant_bf16(mlm_ctx *ctx, const void *blocks, void *out_bf16, uint64_t n);
/* y = W x (+ residual) on packed Q6_K weights W[rows][cols] (the Q6_K
 * tensors ModelLoader.swift:282-287 dequantizes for an MPS linear), x fp16,
 * fp32 accumulation; cols a multiple of 2048 and at most 32768; W and x
 * 16-byte aligned.  Stream-ordered. */
int mlm_q6k_gemv(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_f16, float *y,
                 const float *residual);
/* The same GEMV with the x stagings of the Q4_K GEMVs (mlm_q4k_gemv_xs,
 * _rmsnorm, _swiglu below), for the Q6_K linears of Q4_K_M files: attn_v and
 * ffn_down (read after RMSNorm and after the SiLU-gated product,
 * LlamaRunner.swift:547-609, 1036-1068) and the output head
 * (:1130-1178). */
int mlm_q6k_gemv_xs(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_f16,
                    const float *x_scale, float *y, const float *residual);
int mlm_q6k_gemv_rmsnorm(mlm_ctx *ctx, const void *W, int rows, int cols, const float *hidden,
                         const float *norm_w, float eps, float *y, const float *residual);
int mlm_q6k_gemv_swiglu(mlm_ctx *ctx, const void *W, int rows, int cols, const float *gate,
                        const float *up, float *y, const float *residual);

/* MetalService.dequantizeQ4KM_to_f32 / _f16 (MetalService.swift:170, 243):
 * allocate the output, run, wait.  *out receives a device pointer to free
 * with mlm_free.  Thread-safe (the loader calls these from concurrent
 * tasks, ModelLoaderWrapper.swift:172-201). */
int mlm_dequantize_q4k_to_f32(mlm_ctx *ctx, const void *blocks, uint64_t n, float **out);
int mlm_dequantize_q4k_to_f16(mlm_ctx *ctx, const void *blocks, uint64_t n, void **out);

/* y[r] = sum_k W[r][k] * x[k] (+ residual[r] when residual != NULL).
 * Replaces encodeMPSMatrixMultiply at the decode linears
 * (MetalService.swift:797-925; LlamaRunner.swift:563-609, 954-963,
 * 1008-1034, 1059-1068, 1169-1178) on the packed weights, with no
 * dequantized copy.  W row-major [rows][cols/256 blocks] (GGUF ne0 = cols);
 * x fp16 [cols]; y fp32 [rows]; fp32 accumulation.  cols % 256 == 0; W and
 * x 16-byte aligned.  Uses the context's split-K scratch: launches on one
 * context are stream-ordered and must not overlap. */
int mlm_q4k_gemv(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_f16,
                 float *y, const float *residual);

/* mlm_q4k_gemv on an x given as fp16 values times one fp32 scale per 32
 * elements (x[k] = x_f16[k] * x_scale[k/32]), as mlm_silu_mul_scaled writes
 * it: the down projection of the decode FFN (LlamaRunner.swift:1059-1068). */
int mlm_q4k_gemv_xs(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_f16,
                    const float *x_scale, float *y, const float *residual);

/* The GEMV with its input normalised on the fly: x = RMSNorm(hidden) as
 * mlm_rmsnorm_f32 computes it (NormalizationKernels.metal:31-79; fp32 hidden
 * and weights, the product rounded to fp16), each CTA reducing the sum of
 * squares itself -- the encodeRMSNormF16 + encodeMPSMatrixMultiply pairs of
 * LlamaRunner.swift:547-609 and 992-1034 in one launch.  hidden and norm_w
 * 16-byte aligned. */
int mlm_q4k_gemv_rmsnorm(mlm_ctx *ctx, const void *W, int rows, int cols, const float *hidden,
                         const float *norm_w, float eps, float *y, const float *residual);
/* The GEMV on x = silu(gate) * up formed on the fly (fp32 in, stored as fp16
 * with per-32 power-of-two scales as mlm_silu_mul_scaled does): applySILU,
 * applyElementWiseMul and the down projection of LlamaRunner.swift:1036-1068
 * in one launch. */
int mlm_q4k_gemv_swiglu(mlm_ctx *ctx, const void *W, int rows, int cols, const float *gate,
                        const float *up, float *y, const float *residual);
/* The decode FFN's gate and up projections as one GEMV over W = [gate rows;
 * up rows] (rows = 2F, F a multiple of 32) on x = RMSNorm(hidden), whose
 * epilogue also forms h = silu(gate) * up (LlamaRunner.swift:1008-1058:
 * gate, up, applySILU, multiply) in the scaled fp16 form of
 * mlm_silu_mul_scaled: h_f16 [F], h_scale [F/32], bit-identical to that op on
 * y.  h is the x of the down projection through mlm_q4k_gemv_xs; no CTA
 * evaluates the SiLU of an element more than once. */
int mlm_q4k_gemv_gate_up(mlm_ctx *ctx, const void *W, int rows, int cols, const float *hidden,
                         const float *norm_w, float eps, float *y, void *h_f16, float *h_scale);

/* Prefill GEMM on packed Q4_K weights: y[t][n] = sum_k x[t][k] * W[n][k] for
 * `tokens` rows of x at once (bf16 [tokens][cols] row-major; y fp32
 * [tokens][rows]).  The reference has no batched prefill: it runs forward()
 * per prompt token with encodeMPSMatrixMultiply on fp16 weights
 * (MetalService.swift:797-925).  W (GGUF layout) is dequantized tile by tile
 * to bf16 in shared memory and multiplied on the tensor cores (tcgen05, fp32
 * accumulation).  cols % 256 == 0; W and x 16-byte aligned; at most 65536
 * output tiles of 256 rows x 256 tokens.  One persistent CTA per SM; where a
 * tile's K range is shared by several CTAs, the parts after the first are
 * added into y with fp32 atomics (summation order may then differ from run
 * to run in the last bits).  residual (fp32 [tokens][rows], may be y
 * itself) is added when not NULL. */
/* The decode linears for a batch of 1..8 tokens (independent sequences):
 * y[t][n] = sum_k x[t][k] * W[n][k] (+ residual), x bf16 [tokens][cols], y
 * fp32 [tokens][rows].  The reference multiplies one token at a time
 * (encodeMPSMatrixMultiply, MetalService.swift:797-925); here the packed
 * weights are read once for the whole batch and go to the tensor cores as in
 * mlm_q4k_gemv, the tokens as the MMA's columns.  cols % 256 == 0; W and x
 * 16-byte aligned; residual may be y itself (fp32 atomics add the partial
 * sums of K chunks into y, so the last bits may differ from run to run). */
int mlm_q4k_gemv_batch(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_bf16,
                       int tokens, float *y, const float *residual);

int mlm_q4k_gemm(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_bf16,
                 int tokens, float *y, const float *residual);
/* The prompt linears on a Q6_K weight (encodeMPSMatrixMultiply on the
 * weight ModelLoader.swift:282-287 dequantizes): W is dequantized into the
 * caller's scratch (rows x cols bf16, 16-byte aligned: the fp32 value
 * rounded once, as mlm_q6k_dequant_bf16) and the tensor-core GEMM reads it
 * there; same X, Y and residual conventions as mlm_q4k_gemm. */
int mlm_q6k_gemm(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_bf16,
                 int tokens, float *y, const float *residual, void *scratch_bf16);

/* No counterpart in the reference.  mlm_q4k_gemv with its split-K scratch
 * in a static 80 KB device array inside the library instead of the
 * context's allocation: the call allocates nothing, for hosts that own all
 * device memory through their own pool or enqueue from places where an
 * allocation may not happen.  rows <= 131072 (MLM_ERR_SHAPE beyond).  The
 * calling thread's current device must be the context's device
 * (MLM_ERR_STATE otherwise: the array's address is per device).  The
 * first call on a device looks up and clears the array (make it before any
 * stream capture); later calls clear only the arrival counters, on the
 * context stream.  All calls on a device share the array: calls that overlap
 * on the GPU race -- keep them on one stream. */
int mlm_q4k_gemv_static(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_f16,
                        float *y, const float *residual);

/* Launch plans, computed on the host alone (no GPU call, no context): the
 * decode GEMV's CTAs and warps per CTA for a rows x cols weight on a GPU of
 * sm_count SMs, and whether every CTA owns whole 32-row tiles (no partial
 * sum crosses CTAs); the batched GEMV's K chunk (block columns) and CTAs. */
int mlm_q4k_gemv_plan(int rows, int cols, int sm_count, int *ctas, int *warps,
                      int *whole_tiles);
int mlm_q4k_gemv_batch_plan(int rows, int cols, int sm_count, int *chunk, int *ctas);

/* ---------------------------------------------------------------------------
 * Normalisation, RoPE, activations
 * ------------------------------------------------------------------------ */

/* kernel_rms_norm_f16 / encodeRMSNormF16 (NormalizationKernels.metal:9-80,
 * MetalService.swift:544-677): y = half(x * min(1/sqrt(max(mean(x^2),1e-10)
 * + eps), 1e6) * w), NaN/Inf weights read as 1. */
int mlm_rmsnorm_f16(mlm_ctx *ctx, const void *x_f16, const void *w_f16, void *y_f16,
                    int rows, int n, float eps);
/* the same formula on an fp32 hidden state with fp32 weights; writes fp32
 * (y_f32, may be NULL) and/or fp16 (y_f16, may be NULL; feeds the GEMV) */
int mlm_rmsnorm_f32(mlm_ctx *ctx, const float *x, const float *w, float *y_f32,
                    void *y_f16, int rows, int n, float eps);

/* MetalRopeArgs (PositionalEmbeddingsKernels.metal:15-42) */
typedef struct mlm_rope_args {
  uint32_t n_dims;
  float freq_base;   /* 500000 for Llama-3 */
  float freq_scale;
  int32_t pos_offset;
  int32_t n_ctx_orig;
  float ext_factor;  /* 0 disables the YaRN blend */
  float attn_factor;
  float beta_fast;
  float beta_slow;
  int32_t has_freq_factors;
} mlm_rope_args;

/* kernel_rope_f16_inplace / applyRoPE (PositionalEmbeddingsKernels.metal:
 * 137-204, MetalService.swift:685-777): data [seq_len][num_heads][head_dim]
 * fp16, adjacent pairs (i0, i0+1) rotated in place for i0 < n_dims.  freqs
 * (n_dims/2 divisors) is read when has_freq_factors != 0. */
int mlm_rope_f16(mlm_ctx *ctx, void *data_f16, const float *freqs,
                 const mlm_rope_args *args, int seq_len, int num_heads, int head_dim);

/* Decode-step QKV epilogue: RoPE on fp32 q [n_q_heads][d] and k
 * [n_kv_heads][d] at position args->pos_offset, q written as fp16 q_out,
 * rotated k and v (fp32 [n_kv_heads][d]) appended as fp16 at row `pos` of
 * the layer's caches [max_seq][n_kv_heads][d].  Replaces applyRoPE on Q and
 * K plus the KV-cache blit (LlamaRunner.swift:612-666). */
int mlm_rope_qk_kv_append(mlm_ctx *ctx, const float *q, const float *k, const float *v,
                          const float *freqs, const mlm_rope_args *args, int n_q_heads,
                          int n_kv_heads, int head_dim, void *q_out_f16, void *k_cache_f16,
                          void *v_cache_f16, int pos);

/* kernel_silu_f16 then kernel_mul_f16 (ActivationKernels.metal:6-27,
 * ElementwiseKernels.metal; LlamaRunner.swift:1036-1057):
 * out_f16[i] = half(silu(gate[i]) * up[i]) from fp32 gate/up */
int mlm_silu_mul(mlm_ctx *ctx, const float *gate, const float *up, void *out_f16, int n);
/* No counterpart in the reference (its SiLU and multiply store fp16, which
 * overflows on large activations): the same product stored as fp16 with one
 * power-of-two scale per 32 elements, out_f16[i] * scale[i/32] being the fp16
 * rounding of the product scaled to below 2^15 (a power-of-two scale is
 * exact).  n % 32 == 0; feeds mlm_q4k_gemv_xs. */
int mlm_silu_mul_scaled(mlm_ctx *ctx, const float *gate, const float *up, void *out_f16,
                        float *scale, int n);
/* kernel_add_f16 (residual adds, LlamaRunner.swift:969-980, 1074-1085), fp32 */
int mlm_add_f32(mlm_ctx *ctx, const float *a, const float *b, float *out, int n);

/* ---------------------------------------------------------------------------
 * Attention
 * ------------------------------------------------------------------------ */

/* Decode attention for one token over an fp16 KV cache: for every query head
 * h, out[h] = softmax(q[h] . K[0:seq_len, h/(n_heads/n_kv_heads)]^T / sqrt(d))
 * . V[...].  Replaces applyRepeatKVHeads, the per-head MPS GEMMs and
 * encodeMPSSoftMax (LlamaRunner.swift:669-952, AttentionKernels.metal:16-59,
 * MetalService.swift:937-1000).  q fp16 [n_heads][d]; caches
 * [>=seq_len][n_kv_heads][d] fp16; out fp16 [n_heads][d].  head_dim 128. */
int mlm_attn_decode(mlm_ctx *ctx, const void *q_f16, const void *k_cache_f16,
                    const void *v_cache_f16, int n_heads, int n_kv_heads, int head_dim,
                    int seq_len, void *out_f16);

/* ---------------------------------------------------------------------------
 * Embedding / argmax (the greedy loop of ContentView.swift:124-146, 274-343)
 * ------------------------------------------------------------------------ */

/* out[i] = float(table[token][i]) for an fp16 [vocab][dim] table
 * (embedding-row blit, LlamaRunner.swift:473-491) */
int mlm_embed_f16(mlm_ctx *ctx, const void *table_f16, int vocab, int dim,
                  const int32_t *token_dev, float *out);
/* index of the largest logit (first on ties), written to *out_index (device) */
int mlm_argmax_f32(mlm_ctx *ctx, const float *logits, int n, int32_t *out_index_dev);

/* ---------------------------------------------------------------------------
 * Tensor parallelism over NCCL, one context (one process) per GPU.  No
 * counterpart in the reference, which runs on one Metal device.  NCCL is
 * loaded at run time by its soname, libnccl.so.2: a copy already in the
 * process is reused, else the system's is loaded -- a process that will also
 * load another NCCL build (PyTorch's, say) must load that one first.
 * Collectives are enqueued on the context's stream; small fp32 sums run as
 * one kernel over NVLink peer memory mapped at mlm_tp_init (CUDA IPC), the
 * rest through NCCL.
 * ------------------------------------------------------------------------ */

/* a fresh NCCL unique id (NCCL_UNIQUE_ID_BYTES = 128 bytes) for rank 0 to
 * hand to the other ranks */
int mlm_tp_unique_id(mlm_ctx *ctx, void *out, size_t bytes);
/* join the group: every rank calls this with the same id (a collective) */
int mlm_tp_init(mlm_ctx *ctx, int nranks, int rank, const void *unique_id);
/* this context's rank and group size (size 0 when it has no group) */
int mlm_tp_info(const mlm_ctx *ctx, int *rank, int *size);
/* recv = sum over ranks of send (fp32, count elements; may be in place) */
int mlm_tp_allreduce_f32(mlm_ctx *ctx, const float *send, float *recv, size_t count);
/* recv = the ranks' `bytes`-byte send buffers, rank order */
int mlm_tp_allgather(mlm_ctx *ctx, const void *send, void *recv, size_t bytes);

/* ---------------------------------------------------------------------------
 * Llama decode runner: class LlamaRunner (LlamaRunner.swift:22-1210)
 * ------------------------------------------------------------------------ */

/* LlamaConfig (the fields LlamaRunner.swift:38-48 and forward() read) */
typedef struct mlm_llama_config {
  int32_t n_layers;
  int32_t dim;        /* embeddingDim */
  int32_t n_heads;
  int32_t n_kv_heads; /* numKeyValueHeads */
  int32_t head_dim;   /* 128 */
  int32_t ffn_dim;    /* hiddenDim */
  int32_t vocab;
  int32_t max_seq;    /* sequenceLength: KV-cache capacity, <= 8192 */
  float rms_eps;
  mlm_rope_args rope; /* freq_base (theta), YaRN parameters, n_dims */
} mlm_llama_config;

/* Device pointers of one layer's tensors inside the runner's buffers; a
 * loader uploads the GGUF tensors straight into them (LlamaModel's blocks,
 * ModelLoader.swift:104-219).  Q4_K tensors in GGUF layout [rows][cols/256]
 * (wq/wk/wv rows are contiguous, as are w_gate/w_up).  k_cache / v_cache are
 * this layer's fp16 [max_seq][n_kv_heads][head_dim] caches. */
typedef struct mlm_llama_layer {
  float *attn_norm; /* fp32 [dim] */
  void *wq, *wk, *wv, *wo;
  float *ffn_norm; /* fp32 [dim] */
  void *w_gate, *w_up, *w_down;
  void *k_cache, *v_cache;
  int32_t wv_type, w_down_type; /* MLM_TYPE_Q4_K or MLM_TYPE_Q6_K (210-byte blocks) */
} mlm_llama_layer;

typedef struct mlm_llama_globals {
  void *tok_embd;     /* fp16 [vocab][dim] */
  float *output_norm; /* fp32 [dim] */
  void *output;       /* Q4_K (or Q6_K) [vocab][dim/256] */
  float *rope_freqs;  /* fp32 [head_dim/2], read when rope.has_freq_factors */
  int32_t output_type;
} mlm_llama_globals;

/* GGUF tensor types (the ggml_type values of the file's tensor table,
 * GGUF.swift:63) a runner's linears may hold. */
#define MLM_TYPE_Q4_K 12
#define MLM_TYPE_Q6_K 14

/* Per-tensor types of a Q4_K_M file: its output head and, per layer, attn_v
 * and ffn_down may be Q6_K (ModelLoader.swift:274-296 dequantizes each
 * tensor by its own type).  NULL arrays: every layer Q4_K. */
typedef struct mlm_llama_types {
  int32_t output;
  const int32_t *attn_v;   /* [n_layers] */
  const int32_t *ffn_down; /* [n_layers] */
} mlm_llama_types;

typedef struct mlm_llama mlm_llama;

/* LlamaRunner.init: allocates the weights, the KV caches (2 x n_layers x
 * max_seq x n_kv_heads x head_dim fp16) and the activations of one decode
 * step on ctx's device.  The runner enqueues on ctx's stream.  When ctx has
 * a tensor-parallel group of R ranks (mlm_tp_init), this rank r holds only
 * its shard: heads [r H/R, (r+1) H/R) and KV heads likewise (wq/wk/wv rows,
 * caches), FFN rows [r F/R, (r+1) F/R) of w_gate / w_up, the same input
 * columns of wo / w_down (stored [dim][cols/R]), and vocabulary rows
 * [r V/R, (r+1) V/R) of the output head; cfg stays the whole model's.  Each
 * of these must divide evenly (MLM_ERR_SHAPE). */
int mlm_llama_create(mlm_ctx *ctx, const mlm_llama_config *cfg, mlm_llama **out);
void mlm_llama_destroy(mlm_llama *m);
int mlm_llama_layer_tensors(mlm_llama *m, int layer, mlm_llama_layer *out);
int mlm_llama_global_tensors(mlm_llama *m, mlm_llama_globals *out);

/* LlamaRunner.resetState / currentPosition.  mlm_llama_set_position lets a
 * caller that filled the caches itself continue at `pos`. */
int mlm_llama_reset(mlm_llama *m);
int mlm_llama_set_position(mlm_llama *m, int pos);
int mlm_llama_position(const mlm_llama *m);

/* One decoder layer of forward() at the current position (the body of the
 * layer loop, LlamaRunner.swift:537-1085): hidden fp32 [dim] in place,
 * K and V appended at the current position.  Does not advance. */
int mlm_llama_forward_layer(mlm_llama *m, int layer, float *hidden);

/* LlamaRunner.forward(tokenID:) (LlamaRunner.swift:320-1210): embedding,
 * all layers, final norm, output head; fp32 logits [vocab] (device) written
 * to `logits` (NULL: kept inside the runner).  Advances the position.
 * MLM_ERR_STATE when the cache is full, MLM_ERR_ARG for a bad token id. */
int mlm_llama_forward(mlm_llama *m, int token, float *logits);

/* The prompt (the reference calls forward() once per token): tokens[0..n)
 * (host array) at the current position, run batched on the tensor-core GEMM
 * (mlm_q4k_gemm; bf16 activations) in chunks of up to 1024 tokens, the KV
 * caches filled; then the output head on the last token: its fp32 logits go
 * to `logits` (device, may be NULL) and its greedy next token to
 * *next_token_dev (device, may be NULL).  Advances the position by n. */
int mlm_llama_prefill(mlm_llama *m, const int32_t *tokens, int n, float *logits,
                      int32_t *next_token_dev);

/* Greedy generation (the sampling loop of ContentView.swift:124-146 with the
 * argmax on the device): starting from `token` at the current position,
 * `steps` decode steps, each feeding back its argmax; tokens_out_dev[i]
 * receives the i-th generated token.  One decode step is captured once as a
 * CUDA graph and replayed; the first call captures it (make it outside any
 * other capture on ctx's stream). */
int mlm_llama_decode_greedy(mlm_llama *m, int token, int steps, int32_t *tokens_out_dev);

/* A batch of independent sequences on one runner (the reference decodes one
 * conversation at a time).  mlm_llama_create_batch allocates `batch`
 * (1 .. min(64, max_seq)) sets of KV caches; the calls above act on
 * sequence 0.  Each sequence's prompt goes through mlm_llama_prefill_seq
 * (as mlm_llama_prefill, on that sequence's caches and position).  A
 * batched step runs the batch's tokens together through the tensor-core
 * GEMM (the weights are streamed once for all of them, bf16 activations) and
 * attends per sequence: mlm_llama_forward_batch takes one host token per
 * sequence and writes fp32 logits [batch][vocab] (device, may be NULL);
 * mlm_llama_decode_greedy_batch runs `steps` greedy steps from one host
 * token per sequence, tokens_out_dev[i * batch + b] receiving sequence b's
 * i-th token (one batched step captured once as a CUDA graph and replayed).
 * Every sequence advances by one position per step. */
int mlm_llama_create_batch(mlm_ctx *ctx, const mlm_llama_config *cfg, int batch, mlm_llama **out);
/* mlm_llama_create_batch with per-tensor types (mlm_llama_types; NULL: all
 * Q4_K).  Q6_K tensors need a multiple of 2048 input columns per rank
 * (MLM_ERR_UNSUPPORTED otherwise); the prompt pass reads them through a bf16
 * copy the runner keeps for its largest Q6_K layer weight. */
int mlm_llama_create_typed(mlm_ctx *ctx, const mlm_llama_config *cfg, int batch,
                           const mlm_llama_types *types, mlm_llama **out);
int mlm_llama_prefill_seq(mlm_llama *m, int seq, const int32_t *tokens, int n, float *logits,
                          int32_t *next_token_dev);
int mlm_llama_seq_position(const mlm_llama *m, int seq);
int mlm_llama_forward_batch(mlm_llama *m, const int32_t *tokens, float *logits);
int mlm_llama_decode_greedy_batch(mlm_llama *m, const int32_t *tokens, int steps,
                                  int32_t *tokens_out_dev);

#ifdef __cplusplus
}
#endif
#endif /* METALLM_CUDA_H */
