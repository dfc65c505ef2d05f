/*
 * ref_driver.cpp -- runs the reference's own Metal kernels on the CPU
 * (TEST INFRASTRUCTURE ONLY).
 *
 * The Makefile target `ref` turns the .metal sources of
 * MetalLM/Backend/Metal/ into host C++ (attributes stripped, msl_host.h in
 * place of <metal_stdlib>) under oracle/_ref/, and this file includes that
 * translation unit and drives each kernel the way the Metal runtime would:
 * one call per grid position.  The result is the reference's arithmetic,
 * executed here, used to pin the C restatement in q4k_oracle.c and, through
 * the committed golden vectors, the CUDA kernels.
 *
 * Dispatch shapes follow the reference's host wrappers:
 *   dequant:  grid = nelements, one thread per element (MetalService.swift:222-229)
 *   rmsnorm:  one threadgroup per row (MetalService.swift:611-667); run here
 *             with one thread per threadgroup
 *   rope:     grid (n_dims/2, heads, seq) (MetalService.swift:757-774)
 */
#include "metal_kernels_host.cpp"

#include <cstring>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

void ref_q4k_dequant_f32(const void *blocks, float *out, uint64_t n, int nthreads) {
  uint64_t ne = n;
  const block_q4_K *src = (const block_q4_K *)blocks;
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t gid = 0; gid < (int64_t)n; ++gid)
    kernel_dequantize_q4_K_f32(src, out, ne, (uint)gid);
}

void ref_q4k_dequant_f16(const void *blocks, uint16_t *out, uint64_t n, int nthreads) {
  uint64_t ne = n;
  const block_q4_K *src = (const block_q4_K *)blocks;
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t gid = 0; gid < (int64_t)n; ++gid)
    kernel_dequantize_q4_K_f16(src, (half *)out, ne, (uint)gid);
}

/* Q6_K -> fp32 with the reference's kernel (dispatch: one thread per
 * element, MetalService.swift:370-374) */
void ref_q6k_dequant_f32(const void *blocks, float *out, uint64_t n, int nthreads) {
  uint64_t ne = n;
  const block_q6_K *src = (const block_q6_K *)blocks;
  static_assert(sizeof(block_q6_K) == 210, "block_q6_K is 210 bytes");
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t gid = 0; gid < (int64_t)n; ++gid)
    kernel_dequantize_q6_K_f32(src, out, ne, (uint)gid);
}

/* y = W x: each row dequantized by the reference kernel, then an fp32 dot
 * product (the reference feeds the dequantized weights to MPS). */
void ref_q4k_matvec(const void *W, int rows, int cols, const uint16_t *x_f16,
                    float *y, int nthreads) {
  const block_q4_K *src = (const block_q4_K *)W;
  const int nb = cols / 256;
  std::vector<float> xf((size_t)cols);
  for (int k = 0; k < cols; ++k) {
    half h;
    std::memcpy(&h, &x_f16[k], 2);
    xf[(size_t)k] = (float)h;
  }
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
  {
    float wb[256];
#pragma omp for schedule(static)
    for (int r = 0; r < rows; ++r) {
      float acc = 0.0f;
      const block_q4_K *row = src + (size_t)r * nb;
      for (int b = 0; b < nb; ++b) {
        uint64_t ne = 256;
        for (uint i = 0; i < 256; ++i) kernel_dequantize_q4_K_f32(row + b, wb, ne, i);
        const float *xb = xf.data() + (size_t)b * 256;
        for (int i = 0; i < 256; ++i) acc += wb[i] * xb[i];
      }
      y[r] = acc;
    }
  }
}

void ref_rmsnorm_f16(const uint16_t *x, const uint16_t *w, uint16_t *y, int rows,
                     int n, float eps) {
  MetalRMSNormArgs args;
  args.eps = eps;
  args.ne00 = (uint64_t)n;
  float shmem[32];
  for (int r = 0; r < rows; ++r)
    kernel_rms_norm_f16((const half *)x, (const half *)w, (half *)y, args, shmem,
                        (uint)r, /*tpitg*/ 0, /*sgitg*/ 0, /*tiisg*/ 0, /*ntg*/ 1);
}

void ref_rope_f16(uint16_t *data, const float *freqs, uint32_t n_dims,
                  float freq_base, float freq_scale, int32_t pos_offset,
                  int32_t n_ctx_orig, float ext_factor, float attn_factor,
                  float beta_fast, float beta_slow, int has_freq_factors,
                  int seq_len, int num_heads) {
  MetalRopeArgs a;
  std::memset(&a, 0, sizeof(a));
  a.n_dims = n_dims;
  a.freq_base = freq_base;
  a.freq_scale = freq_scale;
  a.pos_offset = pos_offset;
  a.n_ctx_orig = n_ctx_orig;
  a.ext_factor = ext_factor;
  a.attn_factor = attn_factor;
  a.beta_fast = beta_fast;
  a.beta_slow = beta_slow;
  a.has_freq_factors = has_freq_factors != 0;
  uint3 gdim = {n_dims / 2, (uint)num_heads, (uint)seq_len};
  for (uint z = 0; z < gdim.z; ++z)
    for (uint yy = 0; yy < gdim.y; ++yy)
      for (uint xx = 0; xx < gdim.x; ++xx) {
        uint3 tid = {xx, yy, z};
        kernel_rope_f16_inplace(a, (half *)data, freqs, tid, gdim);
      }
}

void ref_silu_f16(const uint16_t *x, uint16_t *y, uint64_t n) {
  uint64_t ne = n;
  for (uint64_t i = 0; i < n; ++i) kernel_silu_f16((const half *)x, (half *)y, ne, (uint)i);
}

void ref_mul_f16(const uint16_t *a, const uint16_t *b, uint16_t *y, uint64_t n) {
  uint64_t ne = n;
  for (uint64_t i = 0; i < n; ++i)
    kernel_mul_f16((const half *)a, (const half *)b, (half *)y, ne, (uint)i);
}

void ref_repeat_kv_f16(const uint16_t *src, uint16_t *dst, uint32_t num_kv_heads,
                       uint32_t num_query_groups, uint32_t head_dim, uint32_t seq_len) {
  RepeatKVHeadsArgs a = {num_kv_heads, num_query_groups, head_dim, seq_len};
  uint64_t total = (uint64_t)seq_len * num_kv_heads * num_query_groups * head_dim;
  for (uint64_t i = 0; i < total; ++i)
    kernel_repeat_kv_heads_f16((const half *)src, (half *)dst, a, (uint)i);
}

int ref_threads_available(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // extern "C"
