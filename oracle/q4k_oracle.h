/*
 * q4k_oracle.h -- CPU oracle (test infrastructure only) for the Q4_K
 * quantized Llama-3 hot path of MetalLM.
 *
 * This is the checker, never the product: only the tests, the smoke entry
 * and the bench's CPU-baseline leg load it.  Every function restates, in
 * plain C, the arithmetic of one reference Metal kernel or MPS call site:
 *
 *   orc_q4k_dequant_f32   MetalLM/Backend/Metal/DequantKernels.metal:43-56,63-92
 *   orc_q4k_dequant_f16   MetalLM/Backend/Metal/DequantKernels.metal:96-125
 *   orc_q4k_matvec        MetalLM/Backend/LlamaRunner.swift:563-609 (MPS GEMM,
 *                         composed from the fp32 dequantizer; y = W x with
 *                         W[out][in] as GGUF stores it)
 *   orc_rmsnorm_f16       MetalLM/Backend/Metal/NormalizationKernels.metal:9-80
 *   orc_rmsnorm_f32       same formula, fp32 input/weight (layer config)
 *   orc_rope_f16          MetalLM/Backend/Metal/PositionalEmbeddingsKernels.metal:137-204
 *   orc_rope_f32          same rotation on fp32 data
 *   orc_attn_decode       MetalLM/Backend/LlamaRunner.swift:669-952 (per-head
 *                         QK^T * 1/sqrt(d), MPS softmax, P*V) with the GQA map
 *                         of MetalLM/Backend/Metal/AttentionKernels.metal:43
 *   orc_silu_mul          MetalLM/Backend/Metal/ActivationKernels.metal:6-27 and
 *                         ElementwiseKernels.metal (kernel_mul_f16)
 *   orc_q6k_dequant_f32   MetalLM/Backend/Metal/DequantKernels.metal:131-172
 *                         (kernel_dequantize_q6_K_f32, block_q6_K :29-34)
 *   orc_q6k_matvec        the Q6_K tensors of ModelLoader.swift:282-287 in a
 *                         linear: fp32 dequant, then the dot product
 *   orc_q4k_dequant_canonical_f32 / orc_q4k_canonical_to_interleaved
 *                         the GGUF (ggml, llama.cpp) Q4_K element order, which
 *                         the reference does not vendor: element 64j + l of a
 *                         super-block is the low nibble of qs[32j + l] for
 *                         l < 32 and the high nibble of qs[32j + l - 32]
 *                         otherwise; scales, mins and the arithmetic are those
 *                         of DequantKernels.metal:43-92
 *
 * The seeded generators (orc_gen_*) use integer-exact hashing plus IEEE
 * add/mul only, so the CUDA generators produce identical bytes.
 */
#ifndef MLM_Q4K_ORACLE_H
#define MLM_Q4K_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QK_K 256
#define ORC_Q4K_BLOCK_BYTES 144

/* ---- seeded generators (bit-identical to the CUDA generators) ---------- */
uint64_t orc_rng_u64(uint64_t seed, uint64_t stream, uint64_t idx);
/* approximately N(0,1): Irwin-Hall sum of 12 uniform u32, minus 6 */
double orc_normal(uint64_t seed, uint64_t stream, uint64_t idx);
/* Q4_K blocks [first_block, first_block+nblocks) of tensor `stream`:
 * d, dmin = fp16(|N(0,1)| * 0.01); 12 scale bytes and 128 nibble bytes uniform. */
void orc_gen_q4k(uint64_t seed, uint64_t stream, uint64_t first_block,
                 uint64_t nblocks, void *out);
/* out[i] = fp16(mean + std * N(0,1)) for i in [first, first+n) */
void orc_gen_f16(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n,
                 float mean, float std, uint16_t *out);
void orc_gen_f32(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n,
                 float mean, float std, float *out);

/* ---- half <-> float (IEEE binary16, round to nearest even) -------------- */
float orc_half_to_float(uint16_t h);
uint16_t orc_float_to_half(float f);

/* ---- Q4_K ---------------------------------------------------------------- */
void orc_q4k_scale_min(int j, const uint8_t *scales, uint8_t *sc, uint8_t *m);
void orc_q4k_dequant_f32(const void *blocks, uint64_t n, float *out, int nthreads);
void orc_q4k_dequant_f16(const void *blocks, uint64_t n, uint16_t *out, int nthreads);
/* y[r] = sum_k deq(W[r][k]) * x[k]; x fp16; accumulate fp32 (acc64=0) or fp64 */
void orc_q4k_matvec(const void *W, int rows, int cols, const uint16_t *x_f16,
                    float *y, int acc64, int nthreads);
/* same with fp32 x (used by the layer composition) */
void orc_q4k_matvec_f32x(const void *W, int rows, int cols, const float *x,
                         float *y, int nthreads);
/* GGUF element order: dequant, and the byte shuffle to the interleaved order
 * (scales and the two fp16 words are the same in both) */
void orc_q4k_dequant_canonical_f32(const void *blocks, uint64_t n, float *out);
void orc_q4k_canonical_to_interleaved(const void *src, void *dst, uint64_t nblocks);

/* ---- Q6_K (210-byte blocks: ql[128], qh[64], int8 scales[16], fp16 d) --- */
#define ORC_Q6K_BLOCK_BYTES 210
/* d = fp16(|N(0,1)| * 0.01); the 208 bytes of ql, qh and scales uniform */
void orc_gen_q6k(uint64_t seed, uint64_t stream, uint64_t first_block,
                 uint64_t nblocks, void *out);
void orc_q6k_dequant_f32(const void *blocks, uint64_t n, float *out, int nthreads);
/* y[r] = sum_k deq(W[r][k]) * x[k], x fp16, fp64 accumulation */
void orc_q6k_matvec(const void *W, int rows, int cols, const uint16_t *x_f16,
                    float *y, int nthreads);

/* ---- norms / rope / attention ------------------------------------------- */
void orc_rmsnorm_f16(const uint16_t *x, const uint16_t *w, uint16_t *y,
                     int rows, int n, float eps);
void orc_rmsnorm_f32(const float *x, const float *w, float *y, int rows, int n,
                     float eps);

typedef struct orc_rope_args {
  uint32_t n_dims;
  float freq_base;
  float freq_scale;
  int32_t pos_offset;
  int32_t n_ctx_orig;
  float ext_factor;
  float attn_factor;
  float beta_fast;
  float beta_slow;
  int32_t has_freq_factors;
} orc_rope_args;

/* data [seq][heads][head_dim], rotated in place (normal / adjacent-pair mode) */
void orc_rope_f16(const orc_rope_args *a, uint16_t *data, const float *freqs,
                  int seq_len, int num_heads, int head_dim);
void orc_rope_f32(const orc_rope_args *a, float *data, const float *freqs,
                  int seq_len, int num_heads, int head_dim);

/* q [n_heads][d] fp32; caches [seq][n_kv][d] fp16; out [n_heads][d] fp32 */
void orc_attn_decode(const float *q, const uint16_t *kcache,
                     const uint16_t *vcache, int n_heads, int n_kv_heads,
                     int head_dim, int seq_len, float *out, int nthreads);

/* out[i] = silu(g[i]) * u[i], fp32 */
void orc_silu_mul(const float *g, const float *u, float *out, int n);

#ifdef __cplusplus
}
#endif
#endif
