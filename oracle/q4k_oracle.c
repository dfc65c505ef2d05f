/*
 * q4k_oracle.c -- CPU oracle for the Q4_K Llama-3 hot path (TEST
 * INFRASTRUCTURE ONLY: the tests, the smoke entry and the bench's CPU
 * baseline use it as the checker; the CUDA library never links it).
 *
 * Each function restates the arithmetic of the reference kernel it names
 * (paths relative to the MetalLM project root).  See q4k_oracle.h.
 */
#include "q4k_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef _Float16 orc_half;

/* ------------------------------------------------------------------------ */
/* generators                                                               */
/* ------------------------------------------------------------------------ */

static inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

uint64_t orc_rng_u64(uint64_t seed, uint64_t stream, uint64_t idx) {
  uint64_t s = mix64(seed + 0x9E3779B97F4A7C15ULL * (stream + 1));
  return mix64(s ^ (idx * 0xD1B54A32D192ED03ULL + 0x632BE59BD9B4E019ULL));
}

double orc_normal(uint64_t seed, uint64_t stream, uint64_t idx) {
  uint64_t sum = 0;
  for (int k = 0; k < 6; ++k) {
    uint64_t r = orc_rng_u64(seed, stream, idx * 6 + (uint64_t)k);
    sum += (r & 0xffffffffULL) + (r >> 32);
  }
  /* sum < 12 * 2^32 < 2^36: exact in double */
  return (double)sum * (1.0 / 4294967296.0) - 6.0;
}

float orc_half_to_float(uint16_t h) {
  orc_half v;
  memcpy(&v, &h, 2);
  return (float)v;
}

uint16_t orc_float_to_half(float f) {
  orc_half v = (orc_half)f; /* IEEE round to nearest even */
  uint16_t h;
  memcpy(&h, &v, 2);
  return h;
}

/* stream tags keep the fields of one tensor independent */
#define ORC_TAG_BYTES 0x51ULL

void orc_gen_q4k(uint64_t seed, uint64_t stream, uint64_t first_block,
                 uint64_t nblocks, void *out) {
  uint8_t *o = (uint8_t *)out;
#pragma omp parallel for schedule(static)
  for (int64_t bi = 0; bi < (int64_t)nblocks; ++bi) {
    uint64_t b = first_block + (uint64_t)bi;
    uint8_t *blk = o + (uint64_t)bi * ORC_Q4K_BLOCK_BYTES;
    float d = (float)fabs(orc_normal(seed, stream, 2 * b));
    float dm = (float)fabs(orc_normal(seed, stream, 2 * b + 1));
    uint16_t hd = orc_float_to_half(d * 0.01f);
    uint16_t hm = orc_float_to_half(dm * 0.01f);
    memcpy(blk + 0, &hd, 2);
    memcpy(blk + 2, &hm, 2);
    /* 140 payload bytes: 12 packed 6-bit scale/min bytes + 128 nibble bytes.
     * The 12-byte packing is a bijection of 16 six-bit values, so uniform
     * bytes give uniform scales and mins in [0, 63]. */
    uint8_t tmp[144];
    for (int k = 0; k < 18; ++k) {
      uint64_t r = orc_rng_u64(seed, stream ^ (ORC_TAG_BYTES << 56), b * 18 + (uint64_t)k);
      memcpy(tmp + 8 * k, &r, 8);
    }
    memcpy(blk + 4, tmp, 140);
  }
}

void orc_gen_f16(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n,
                 float mean, float std, uint16_t *out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)n; ++i) {
    float v = (float)orc_normal(seed, stream, first + (uint64_t)i);
    out[i] = orc_float_to_half(mean + std * v);
  }
}

void orc_gen_f32(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n,
                 float mean, float std, float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)n; ++i) {
    float v = (float)orc_normal(seed, stream, first + (uint64_t)i);
    out[i] = mean + std * v;
  }
}

/* ------------------------------------------------------------------------ */
/* Q4_K                                                                     */
/* ------------------------------------------------------------------------ */

/* get_scale_min_k4_metal, DequantKernels.metal:43-56 */
void orc_q4k_scale_min(int j, const uint8_t *s, uint8_t *sc, uint8_t *m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (uint8_t)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
    *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
}

/* kernel_dequantize_q4_K_f32, DequantKernels.metal:63-92: element i of a
 * super-block reads byte qs[i/2], low nibble for even i, high for odd i;
 * out = (float(d)*sc) * q - float(dmin)*m in fp32. */
static inline float deq_elem_f32(const uint8_t *blk, unsigned i) {
  uint16_t hd, hm;
  memcpy(&hd, blk, 2);
  memcpy(&hm, blk + 2, 2);
  uint8_t sc, m;
  orc_q4k_scale_min((int)(i / 32), blk + 4, &sc, &m);
  float d = orc_half_to_float(hd);
  float dmin = orc_half_to_float(hm);
  float final_scale = d * (float)sc;
  float final_min = dmin * (float)m;
  uint8_t qb = blk[16 + i / 2];
  uint8_t q = (i % 2 == 0) ? (qb & 0xF) : (qb >> 4);
  return final_scale * (float)q - final_min;
}

void orc_q4k_dequant_f32(const void *blocks, uint64_t n, float *out, int nthreads) {
  const uint8_t *src = (const uint8_t *)blocks;
  uint64_t nb = (n + ORC_QK_K - 1) / ORC_QK_K;
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#endif
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t b = 0; b < (int64_t)nb; ++b) {
    const uint8_t *blk = src + (uint64_t)b * ORC_Q4K_BLOCK_BYTES;
    uint64_t base = (uint64_t)b * ORC_QK_K;
    for (unsigned i = 0; i < ORC_QK_K; ++i) {
      if (base + i < n) out[base + i] = deq_elem_f32(blk, i);
    }
  }
}

/* kernel_dequantize_q4_K_f16, DequantKernels.metal:96-125: the same formula
 * in half arithmetic.  final_scale and final_min are rounded to binary16 as
 * the half locals they are assigned to; the expression
 * final_scale*q - final_min is formed in fp32 and rounded once, as a
 * contracting (fast-math) compile of the kernel evaluates it. */
void orc_q4k_dequant_f16(const void *blocks, uint64_t n, uint16_t *out, int nthreads) {
  const uint8_t *src = (const uint8_t *)blocks;
  uint64_t nb = (n + ORC_QK_K - 1) / ORC_QK_K;
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#endif
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t b = 0; b < (int64_t)nb; ++b) {
    const uint8_t *blk = src + (uint64_t)b * ORC_Q4K_BLOCK_BYTES;
    uint16_t hd, hm;
    memcpy(&hd, blk, 2);
    memcpy(&hm, blk + 2, 2);
    float d = orc_half_to_float(hd), dmin = orc_half_to_float(hm);
    uint64_t base = (uint64_t)b * ORC_QK_K;
    for (unsigned i = 0; i < ORC_QK_K; ++i) {
      if (base + i >= n) break;
      uint8_t sc, m;
      orc_q4k_scale_min((int)(i / 32), blk + 4, &sc, &m);
      float fs = orc_half_to_float(orc_float_to_half(d * (float)sc));
      float fm = orc_half_to_float(orc_float_to_half(dmin * (float)m));
      uint8_t qb = blk[16 + i / 2];
      uint8_t q = (i % 2 == 0) ? (qb & 0xF) : (qb >> 4);
      out[base + i] = orc_float_to_half(fs * (float)q - fm);
    }
  }
}

/* y = W x with W[rows][cols] Q4_K (super-blocks along cols), composed from
 * the fp32 dequantizer above; the reference runs this product through MPS
 * (LlamaRunner.swift:563-609) on the dequantized weights. */
void orc_q4k_matvec(const void *W, int rows, int cols, const uint16_t *x_f16,
                    float *y, int acc64, int nthreads) {
  const uint8_t *src = (const uint8_t *)W;
  int nb = cols / ORC_QK_K;
  float *xf = (float *)malloc(sizeof(float) * (size_t)cols);
  for (int k = 0; k < cols; ++k) xf[k] = orc_half_to_float(x_f16[k]);
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#endif
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
  {
    float wrow[ORC_QK_K];
#pragma omp for schedule(static)
    for (int r = 0; r < rows; ++r) {
      double a64 = 0.0;
      float a32 = 0.0f;
      for (int b = 0; b < nb; ++b) {
        const uint8_t *blk = src + ((size_t)r * nb + b) * ORC_Q4K_BLOCK_BYTES;
        orc_q4k_dequant_f32(blk, ORC_QK_K, wrow, 1);
        const float *xb = xf + (size_t)b * ORC_QK_K;
        if (acc64) {
          for (int i = 0; i < ORC_QK_K; ++i) a64 += (double)wrow[i] * (double)xb[i];
        } else {
          for (int i = 0; i < ORC_QK_K; ++i) a32 += wrow[i] * xb[i];
        }
      }
      y[r] = acc64 ? (float)a64 : a32;
    }
  }
  free(xf);
}

void orc_q4k_matvec_f32x(const void *W, int rows, int cols, const float *x,
                         float *y, int nthreads) {
  const uint8_t *src = (const uint8_t *)W;
  int nb = cols / ORC_QK_K;
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#endif
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
  {
    float wrow[ORC_QK_K];
#pragma omp for schedule(static)
    for (int r = 0; r < rows; ++r) {
      double a64 = 0.0;
      for (int b = 0; b < nb; ++b) {
        const uint8_t *blk = src + ((size_t)r * nb + b) * ORC_Q4K_BLOCK_BYTES;
        orc_q4k_dequant_f32(blk, ORC_QK_K, wrow, 1);
        const float *xb = x + (size_t)b * ORC_QK_K;
        for (int i = 0; i < ORC_QK_K; ++i) a64 += (double)wrow[i] * (double)xb[i];
      }
      y[r] = (float)a64;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* RMSNorm: kernel_rms_norm_f16, NormalizationKernels.metal:9-80            */
/* ------------------------------------------------------------------------ */

static inline float rms_scale(double sum_sq, int n, float eps) {
  float mean_sq = (float)sum_sq / (float)n;
  float safe = mean_sq > 1e-10f ? mean_sq : 1e-10f;
  float rms = sqrtf(safe + eps);
  float scale = 1.0f / rms;
  return scale < 1e6f ? scale : 1e6f;
}

void orc_rmsnorm_f16(const uint16_t *x, const uint16_t *w, uint16_t *y,
                     int rows, int n, float eps) {
  for (int r = 0; r < rows; ++r) {
    const uint16_t *xr = x + (size_t)r * n;
    uint16_t *yr = y + (size_t)r * n;
    double ss = 0.0;
    for (int i = 0; i < n; ++i) {
      float v = orc_half_to_float(xr[i]);
      ss += (double)v * (double)v;
    }
    float scale = rms_scale(ss, n, eps);
    for (int i = 0; i < n; ++i) {
      float wv = orc_half_to_float(w[i]);
      if (isnan(wv) || isinf(wv)) wv = 1.0f; /* NormalizationKernels.metal:75-77 */
      yr[i] = orc_float_to_half((orc_half_to_float(xr[i]) * scale) * wv);
    }
  }
}

void orc_rmsnorm_f32(const float *x, const float *w, float *y, int rows, int n,
                     float eps) {
  for (int r = 0; r < rows; ++r) {
    const float *xr = x + (size_t)r * n;
    float *yr = y + (size_t)r * n;
    double ss = 0.0;
    for (int i = 0; i < n; ++i) ss += (double)xr[i] * (double)xr[i];
    float scale = rms_scale(ss, n, eps);
    for (int i = 0; i < n; ++i) {
      float wv = w[i];
      if (isnan(wv) || isinf(wv)) wv = 1.0f;
      yr[i] = (xr[i] * scale) * wv;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* RoPE: kernel_rope_f16_inplace + YaRN helpers,                            */
/* PositionalEmbeddingsKernels.metal:52-125,137-204                         */
/* ------------------------------------------------------------------------ */

static float yarn_ramp(float low, float high, int i0) {
  float diff = high - low;
  float den = diff > 0.001f ? diff : 0.001f;
  float y = ((float)i0 / 2.0f - low) / den;
  float c = y < 0.0f ? 0.0f : (y > 1.0f ? 1.0f : y);
  return 1.0f - c;
}

static float yarn_corr_factor(int n_dims, int n_ctx_orig, float n_rot, float base) {
  if (n_rot <= 0.0f || base <= 0.0f || n_ctx_orig <= 0) return 0.0f;
  float lb = logf(base);
  if (fabsf(lb) < 1e-6f) return 0.0f;
  float term = (float)n_ctx_orig / (n_rot * 2.0f * 3.14159265358979323846f);
  if (term <= 0.0f) return 0.0f;
  return (float)n_dims * logf(term) / (2.0f * lb);
}

/* cos/sin of the rotation angle for pair index p (i0 = 2p) at position pos */
static void rope_cs(const orc_rope_args *a, const float *freqs, int pos, int p,
                    float *c, float *s) {
  int i0 = 2 * p;
  float theta_base = (float)pos;
  float inv_ndims = -1.0f / (float)a->n_dims;
  float theta_extrap = theta_base * powf(a->freq_base, inv_ndims * (float)i0);
  float ff = a->has_freq_factors ? freqs[p] : 1.0f;
  float theta_scaled = theta_extrap / (ff > 0.0001f ? ff : 0.0001f);
  float fast = yarn_corr_factor((int)a->n_dims, a->n_ctx_orig, a->beta_fast, a->freq_base);
  float slow = yarn_corr_factor((int)a->n_dims, a->n_ctx_orig, a->beta_slow, a->freq_base);
  float c0 = floorf(fast);
  if (c0 < 0.0f) c0 = 0.0f;
  float c1 = ceilf(slow);
  if (c1 < c0) c1 = c0;
  if (c1 > (float)a->n_dims - 2.0f) c1 = (float)a->n_dims - 2.0f;
  float theta_interp = a->freq_scale * theta_scaled;
  float theta = theta_interp;
  float mscale = a->attn_factor;
  if (a->ext_factor != 0.0f) {
    float mix = yarn_ramp(c0, c1, i0) * a->ext_factor;
    theta = theta_interp * (1.0f - mix) + theta_scaled * mix;
    if (a->freq_scale > 0.0f) mscale *= (1.0f + 0.1f * logf(1.0f / a->freq_scale));
  }
  /* double-precision trig keeps the oracle accurate for large angles */
  *c = (float)cos((double)theta) * mscale;
  *s = (float)sin((double)theta) * mscale;
}

void orc_rope_f16(const orc_rope_args *a, uint16_t *data, const float *freqs,
                  int seq_len, int num_heads, int head_dim) {
  for (int t = 0; t < seq_len; ++t)
    for (int h = 0; h < num_heads; ++h)
      for (int p = 0; 2 * p < (int)a->n_dims && 2 * p + 1 < head_dim; ++p) {
        float c, s;
        rope_cs(a, freqs, a->pos_offset + t, p, &c, &s);
        float hc = orc_half_to_float(orc_float_to_half(c));
        float hs = orc_half_to_float(orc_float_to_half(s));
        uint16_t *e = data + ((size_t)t * num_heads + h) * head_dim + 2 * p;
        float x0 = orc_half_to_float(e[0]), x1 = orc_half_to_float(e[1]);
        /* half operands; each rotated value formed in fp32, rounded once */
        e[0] = orc_float_to_half(x0 * hc - x1 * hs);
        e[1] = orc_float_to_half(x0 * hs + x1 * hc);
      }
}

void orc_rope_f32(const orc_rope_args *a, float *data, const float *freqs,
                  int seq_len, int num_heads, int head_dim) {
  for (int t = 0; t < seq_len; ++t)
    for (int h = 0; h < num_heads; ++h)
      for (int p = 0; 2 * p < (int)a->n_dims && 2 * p + 1 < head_dim; ++p) {
        float c, s;
        rope_cs(a, freqs, a->pos_offset + t, p, &c, &s);
        float *e = data + ((size_t)t * num_heads + h) * head_dim + 2 * p;
        float x0 = e[0], x1 = e[1];
        e[0] = x0 * c - x1 * s;
        e[1] = x0 * s + x1 * c;
      }
}

/* ------------------------------------------------------------------------ */
/* decode attention: LlamaRunner.swift:669-952 (QK^T/sqrt(d), softmax, PV)   */
/* with kv head = h / (n_heads / n_kv_heads) (AttentionKernels.metal:43)     */
/* ------------------------------------------------------------------------ */

void orc_attn_decode(const float *q, const uint16_t *kc, const uint16_t *vc,
                     int n_heads, int n_kv, int d, int seq_len, float *out,
                     int nthreads) {
  int group = n_heads / n_kv;
  double scale = 1.0 / sqrt((double)d);
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#endif
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
  for (int h = 0; h < n_heads; ++h) {
    int kvh = h / group;
    const float *qh = q + (size_t)h * d;
    double *sc = (double *)malloc(sizeof(double) * (size_t)(seq_len > 0 ? seq_len : 1));
    double mx = -INFINITY;
    for (int t = 0; t < seq_len; ++t) {
      const uint16_t *kr = kc + ((size_t)t * n_kv + kvh) * d;
      double acc = 0.0;
      for (int i = 0; i < d; ++i) acc += (double)qh[i] * (double)orc_half_to_float(kr[i]);
      sc[t] = acc * scale;
      if (sc[t] > mx) mx = sc[t];
    }
    double den = 0.0;
    for (int t = 0; t < seq_len; ++t) {
      sc[t] = exp(sc[t] - mx);
      den += sc[t];
    }
    for (int i = 0; i < d; ++i) {
      double acc = 0.0;
      for (int t = 0; t < seq_len; ++t)
        acc += sc[t] * (double)orc_half_to_float(vc[((size_t)t * n_kv + kvh) * d + i]);
      out[(size_t)h * d + i] = (float)(acc / den);
    }
    free(sc);
  }
}

/* kernel_silu_f16 (ActivationKernels.metal:6-27) then kernel_mul_f16 */
void orc_silu_mul(const float *g, const float *u, float *out, int n) {
  for (int i = 0; i < n; ++i) {
    double x = g[i];
    out[i] = (float)(x / (1.0 + exp(-x)) * (double)u[i]);
  }
}

/* ------------------------------------------------------------------------ */
/* Q4_K in the GGUF element order                                           */
/* ------------------------------------------------------------------------ */

/* the quant of element i (0..255) of a block in the GGUF order: 64-element
 * group j = i/64 owns qs[32j .. 32j+31]; its first 32 elements are the low
 * nibbles, the last 32 the high nibbles */
static inline uint8_t canon_q(const uint8_t *qs, unsigned i) {
  unsigned j = i / 64, l = i % 64;
  return l < 32 ? (uint8_t)(qs[32 * j + l] & 0xF) : (uint8_t)(qs[32 * j + l - 32] >> 4);
}

void orc_q4k_dequant_canonical_f32(const void *blocks, uint64_t n, float *out) {
  const uint8_t *src = (const uint8_t *)blocks;
  for (uint64_t e = 0; e < n; ++e) {
    const uint8_t *blk = src + (e / ORC_QK_K) * ORC_Q4K_BLOCK_BYTES;
    unsigned i = (unsigned)(e % ORC_QK_K);
    uint16_t hd, hm;
    memcpy(&hd, blk, 2);
    memcpy(&hm, blk + 2, 2);
    uint8_t sc, m;
    orc_q4k_scale_min((int)(i / 32), blk + 4, &sc, &m);
    float final_scale = orc_half_to_float(hd) * (float)sc;
    float final_min = orc_half_to_float(hm) * (float)m;
    out[e] = final_scale * (float)canon_q(blk + 16, i) - final_min;
  }
}

void orc_q4k_canonical_to_interleaved(const void *src, void *dst, uint64_t nblocks) {
  const uint8_t *s = (const uint8_t *)src;
  uint8_t *d = (uint8_t *)dst;
  for (uint64_t b = 0; b < nblocks; ++b) {
    uint8_t blk[ORC_Q4K_BLOCK_BYTES];
    memcpy(blk, s + b * ORC_Q4K_BLOCK_BYTES, ORC_Q4K_BLOCK_BYTES);
    uint8_t *o = d + b * ORC_Q4K_BLOCK_BYTES;
    memcpy(o, blk, 16);
    /* interleaved: element i in byte i/2, low nibble for even i */
    for (unsigned k = 0; k < 128; ++k)
      o[16 + k] = (uint8_t)(canon_q(blk + 16, 2 * k) | (canon_q(blk + 16, 2 * k + 1) << 4));
  }
}

/* ------------------------------------------------------------------------ */
/* Q6_K                                                                     */
/* ------------------------------------------------------------------------ */

#define ORC_TAG_Q6K 0x66ULL

void orc_gen_q6k(uint64_t seed, uint64_t stream, uint64_t first_block,
                 uint64_t nblocks, void *out) {
  uint8_t *o = (uint8_t *)out;
#pragma omp parallel for schedule(static)
  for (int64_t bi = 0; bi < (int64_t)nblocks; ++bi) {
    uint64_t b = first_block + (uint64_t)bi;
    uint8_t *blk = o + (uint64_t)bi * ORC_Q6K_BLOCK_BYTES;
    /* 26 words = 208 bytes of ql, qh and scales */
    for (int k = 0; k < 26; ++k) {
      uint64_t r = orc_rng_u64(seed, stream ^ (ORC_TAG_Q6K << 56), b * 26 + (uint64_t)k);
      memcpy(blk + 8 * k, &r, 8);
    }
    float d = (float)fabs(orc_normal(seed, stream ^ (ORC_TAG_Q6K << 56), b));
    uint16_t hd = orc_float_to_half(d * 0.01f);
    memcpy(blk + 208, &hd, 2);
  }
}

/* kernel_dequantize_q6_K_f32, DequantKernels.metal:131-172: element e of a
 * block, half h = e/128, t = e%128, l = t%32, quarter k = t/32; the 6-bit
 * quant is a nibble of ql (ql[64h + l] for k = 0, 2, ql[64h + l + 32] for
 * k = 1, 3; low nibble for k < 2) with bits 2k..2k+1 of qh[32h + l] above
 * it, minus 32; out = (d * scales[8h + l/16 + 2k]) * q in fp32. */
static inline float q6k_elem(const uint8_t *blk, unsigned e) {
  const uint8_t *ql = blk + 64 * (e / 128);
  const uint8_t *qh = blk + 128 + 32 * (e / 128);
  const int8_t *sc = (const int8_t *)(blk + 192) + 8 * (e / 128);
  uint16_t hd;
  memcpy(&hd, blk + 208, 2);
  float d = orc_half_to_float(hd);
  unsigned t = e % 128, l = t % 32, k = t / 32;
  int is = (int)(l / 16);
  uint8_t lo = (k == 0 || k == 2) ? ql[l] : ql[l + 32];
  lo = (k < 2) ? (uint8_t)(lo & 0xF) : (uint8_t)(lo >> 4);
  int q = (int)(int8_t)(uint8_t)(lo | (((qh[l] >> (2 * k)) & 3) << 4)) - 32;
  return d * (float)sc[is + 2 * (int)k] * (float)q;
}

void orc_q6k_dequant_f32(const void *blocks, uint64_t n, float *out, int nthreads) {
  const uint8_t *src = (const uint8_t *)blocks;
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#endif
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t e = 0; e < (int64_t)n; ++e)
    out[e] = q6k_elem(src + (uint64_t)(e / ORC_QK_K) * ORC_Q6K_BLOCK_BYTES,
                      (unsigned)(e % ORC_QK_K));
}

void orc_q6k_matvec(const void *W, int rows, int cols, const uint16_t *x_f16,
                    float *y, int nthreads) {
  const uint8_t *src = (const uint8_t *)W;
  int nb = cols / ORC_QK_K;
  float *xf = (float *)malloc(sizeof(float) * (size_t)cols);
  for (int k = 0; k < cols; ++k) xf[k] = orc_half_to_float(x_f16[k]);
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#endif
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
  for (int r = 0; r < rows; ++r) {
    double a = 0.0;
    for (int b = 0; b < nb; ++b) {
      const uint8_t *blk = src + ((size_t)r * nb + b) * ORC_Q6K_BLOCK_BYTES;
      for (unsigned i = 0; i < ORC_QK_K; ++i)
        a += (double)q6k_elem(blk, i) * (double)xf[(size_t)b * ORC_QK_K + i];
    }
    y[r] = (float)a;
  }
  free(xf);
}
