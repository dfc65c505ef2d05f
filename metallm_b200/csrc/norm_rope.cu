// norm_rope.cu -- RMSNorm, RoPE and the small elementwise kernels of the
// decode step.
//
// RMSNorm follows kernel_rms_norm_f16 (MetalLM/Backend/Metal/
// NormalizationKernels.metal:9-80): fp32 sum of squares,
// scale = min(1 / sqrt(max(mean, 1e-10) + eps), 1e6), y = (x*scale)*w with
// NaN/Inf weights read as 1.  One CTA per row; the row is read once into
// registers, reduced with warp shuffles, then scaled and written.
//
// RoPE follows kernel_rope_f16_inplace and its YaRN helpers
// (PositionalEmbeddingsKernels.metal:52-125, 137-204): normal (adjacent
// pair) mode, theta = pos * base^(-i0/n_dims) / freq_factor, optional YaRN
// blend when ext_factor != 0.  cos/sin are evaluated in double precision so
// large angles (pos ~ 2047 rad) keep full fp32 accuracy.
#include "mlm_device.cuh"
#include "mlm_internal.h"
#include "mlm_rope.cuh"

namespace mlm {

// ---- RMSNorm ------------------------------------------------------------------

__device__ __forceinline__ float block_sum(float v, float *red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float s = 0.f;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

__global__ void __launch_bounds__(256) rmsnorm_f16_kernel(const __half *__restrict__ x,
                                                         const __half *__restrict__ w,
                                                         __half *__restrict__ y, int n,
                                                         float eps) {
  __shared__ float red[32];
  const __half *xr = x + (size_t)blockIdx.x * n;
  __half *yr = y + (size_t)blockIdx.x * n;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = __half2float(xr[i]);
    ss += v * v;
  }
  const float scale = rms_scale(block_sum(ss, red), n, eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float wv = safe_weight(__half2float(w[i]));
    yr[i] = __float2half_rn((__half2float(xr[i]) * scale) * wv);
  }
}

__global__ void __launch_bounds__(512) rmsnorm_f32_kernel(const float *__restrict__ x,
                                                         const float *__restrict__ w,
                                                         float *__restrict__ y32,
                                                         __half *__restrict__ y16, int n,
                                                         float eps) {
  __shared__ float red[32];
  const float *xr = x + (size_t)blockIdx.x * n;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = xr[i];
    ss += v * v;
  }
  const float scale = rms_scale(block_sum(ss, red), n, eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float o = (xr[i] * scale) * safe_weight(w[i]);
    if (y32) y32[(size_t)blockIdx.x * n + i] = o;
    if (y16) y16[(size_t)blockIdx.x * n + i] = __float2half_rn(o);
  }
}

// ---- RoPE -----------------------------------------------------------------------

// grid: (ceil(n_dims/2 / 32), heads, seq) -- the reference's dispatch shape
__global__ void rope_f16_kernel(mlm_rope_args a, RopeConsts k, const float *__restrict__ freqs,
                                __half *__restrict__ data, int num_heads, int head_dim) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  const int h = blockIdx.y, t = blockIdx.z;
  if (2 * p >= (int)a.n_dims || 2 * p + 1 >= head_dim) return;
  float c, s;
  rope_cos_sin(a, k, freqs, a.pos_offset + t, p, c, s);
  const float hc = __half2float(__float2half_rn(c));
  const float hs = __half2float(__float2half_rn(s));
  __half *e = data + ((size_t)t * num_heads + h) * head_dim + 2 * p;
  const float x0 = __half2float(e[0]), x1 = __half2float(e[1]);
  // half operands, each rotated value formed in fp32 and rounded once
  e[0] = __float2half_rn(__fsub_rn(__fmul_rn(x0, hc), __fmul_rn(x1, hs)));
  e[1] = __float2half_rn(__fadd_rn(__fmul_rn(x0, hs), __fmul_rn(x1, hc)));
}

// decode: rotate fp32 q, k at position pos; q -> fp16 q_out, k and v -> fp16
// cache rows.  One thread per rotation pair of q and k, plus v copies.
__global__ void rope_qk_kv_kernel(mlm_rope_args a, RopeConsts k, const float *__restrict__ freqs,
                                  const float *__restrict__ q, const float *__restrict__ kin,
                                  const float *__restrict__ v, int nq, int nkv, int d,
                                  __half *__restrict__ q_out, __half *__restrict__ kc,
                                  __half *__restrict__ vc, int pos,
                                  const int *__restrict__ pos_dev) {
  pdl_wait_then_release();
  // graph-replayed decode reads the position from device memory: it is both
  // the rotation angle's position and the cache row
  const int apos = pos_dev ? *pos_dev : a.pos_offset;
  if (pos_dev) pos = apos;
  const int pairs = d / 2;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int nqp = nq * pairs, nkp = nkv * pairs;
  if (i < nqp + nkp) {
    const bool is_q = i < nqp;
    const int j = is_q ? i : i - nqp;
    const int h = j / pairs, pp = j - h * pairs;
    const float *src = (is_q ? q : kin) + (size_t)h * d + 2 * pp;
    float x0 = src[0], x1 = src[1];
    if (2 * pp < (int)a.n_dims) {
      float c, s;
      rope_cos_sin(a, k, freqs, apos, pp, c, s);
      const float r0 = x0 * c - x1 * s;
      const float r1 = x0 * s + x1 * c;
      x0 = r0;
      x1 = r1;
    }
    __half2 o = __floats2half2_rn(x0, x1);
    if (is_q) {
      *reinterpret_cast<__half2 *>(q_out + (size_t)h * d + 2 * pp) = o;
    } else {
      *reinterpret_cast<__half2 *>(kc + ((size_t)pos * nkv + h) * d + 2 * pp) = o;
    }
  } else if (i < nqp + 2 * nkp) {
    const int j = i - nqp - nkp;
    const int h = j / pairs, pp = j - h * pairs;
    const float *src = v + (size_t)h * d + 2 * pp;
    *reinterpret_cast<__half2 *>(vc + ((size_t)pos * nkv + h) * d + 2 * pp) =
        __floats2half2_rn(src[0], src[1]);
  }
}

// ---- elementwise ------------------------------------------------------------------

__global__ void silu_mul_kernel(const float *__restrict__ g, const float *__restrict__ u,
                                __half *__restrict__ out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  out[i] = __float2half_rn(swiglu(g[i], u[i]));
}

// The same product stored as fp16 with one power-of-two scale per 32
// elements: out[i] * scale[i / 32] is fp16 rounding of the product, with the
// scale chosen so that the sub-block's largest magnitude stays below 2^15.
// (A plain fp16 store overflows for large products; scaling by a power of
// two is exact.)  n is a multiple of 32.
__global__ void silu_mul_scaled_kernel(const float *__restrict__ g, const float *__restrict__ u,
                                       __half *__restrict__ out, float *__restrict__ scale,
                                       int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;  // whole warps: n % 32 == 0
  const float h = swiglu(g[i], u[i]);
  const float m = warp_max(fabsf(h));
  const int e = max(0, (int)((__float_as_uint(m) >> 23) & 0xFF) - 127 - 14);
  out[i] = __float2half_rn(h * __uint_as_float((uint32_t)(127 - e) << 23));
  if ((threadIdx.x & 31) == 0) scale[i >> 5] = __uint_as_float((uint32_t)(127 + e) << 23);
}

__global__ void add_f32_kernel(const float *__restrict__ a, const float *__restrict__ b,
                               float *__restrict__ out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = a[i] + b[i];
}

int rope_qk_kv_launch(mlm_ctx *ctx, const float *q, const float *k, const float *v,
                      const float *freqs, const mlm_rope_args &a, int nq, int nkv, int d,
                      void *q_out, void *kc, void *vc, int pos, cudaStream_t stream,
                      const int *pos_dev) {
  const RopeConsts kc_ = rope_consts(a);
  const int total = nq * (d / 2) + 2 * nkv * (d / 2);
  const cudaError_t e = launch_pdl(
      rope_qk_kv_kernel, dim3((total + 255) / 256), dim3(256), 0, stream, a, kc_, freqs, q, k, v,
      nq, nkv, d, reinterpret_cast<__half *>(q_out), reinterpret_cast<__half *>(kc),
      reinterpret_cast<__half *>(vc), pos, pos_dev);
  return check_launch_pdl(ctx, e, "mlm_rope_qk_kv_append");
}

int silu_mul_launch(mlm_ctx *ctx, const float *g, const float *u, void *out, int n,
                    cudaStream_t stream) {
  silu_mul_kernel<<<(n + 255) / 256, 256, 0, stream>>>(g, u, reinterpret_cast<__half *>(out), n);
  return check_launch(ctx, "mlm_silu_mul");
}

int silu_mul_scaled_launch(mlm_ctx *ctx, const float *g, const float *u, void *out, float *scale,
                           int n, cudaStream_t stream) {
  silu_mul_scaled_kernel<<<(n + 255) / 256, 256, 0, stream>>>(
      g, u, reinterpret_cast<__half *>(out), scale, n);
  return check_launch(ctx, "mlm_silu_mul_scaled");
}

int rmsnorm_f32_launch(mlm_ctx *ctx, const float *x, const float *w, float *y32, void *y16,
                       int rows, int n, float eps, cudaStream_t stream) {
  rmsnorm_f32_kernel<<<rows, 512, 0, stream>>>(x, w, y32, reinterpret_cast<__half *>(y16), n,
                                                eps);
  return check_launch(ctx, "mlm_rmsnorm_f32");
}

}  // namespace mlm

using namespace mlm;

extern "C" int mlm_rmsnorm_f16(mlm_ctx *ctx, const void *x, const void *w, void *y, int rows,
                               int n, float eps) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, x && w && y, MLM_ERR_ARG, "mlm_rmsnorm_f16: null buffer");
  MLM_REQUIRE(ctx, rows > 0 && n > 0, MLM_ERR_SHAPE, "mlm_rmsnorm_f16: rows=%d n=%d", rows, n);
  rmsnorm_f16_kernel<<<rows, 256, 0, ctx->stream>>>(reinterpret_cast<const __half *>(x),
                                                     reinterpret_cast<const __half *>(w),
                                                     reinterpret_cast<__half *>(y), n, eps);
  return check_launch(ctx, "mlm_rmsnorm_f16");
}

extern "C" int mlm_rmsnorm_f32(mlm_ctx *ctx, const float *x, const float *w, float *y32,
                               void *y16, int rows, int n, float eps) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, x && w && (y32 || y16), MLM_ERR_ARG, "mlm_rmsnorm_f32: null buffer");
  MLM_REQUIRE(ctx, rows > 0 && n > 0, MLM_ERR_SHAPE, "mlm_rmsnorm_f32: rows=%d n=%d", rows, n);
  return rmsnorm_f32_launch(ctx, x, w, y32, y16, rows, n, eps, ctx->stream);
}

extern "C" int mlm_rope_f16(mlm_ctx *ctx, void *data, const float *freqs,
                            const mlm_rope_args *args, int seq_len, int num_heads,
                            int head_dim) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, data && args, MLM_ERR_ARG, "mlm_rope_f16: null argument");
  MLM_REQUIRE(ctx, !args->has_freq_factors || freqs, MLM_ERR_ARG,
              "mlm_rope_f16: has_freq_factors set without a freqs buffer");
  MLM_REQUIRE(ctx, seq_len > 0 && num_heads > 0 && head_dim > 0 && args->n_dims >= 2,
              MLM_ERR_SHAPE, "mlm_rope_f16: invalid grid [%u, %d, %d]", args->n_dims / 2,
              num_heads, seq_len);
  const RopeConsts k = rope_consts(*args);
  const int pairs = (int)args->n_dims / 2;
  dim3 grid((pairs + 31) / 32, num_heads, seq_len);
  rope_f16_kernel<<<grid, 32, 0, ctx->stream>>>(*args, k, freqs,
                                                reinterpret_cast<__half *>(data), num_heads,
                                                head_dim);
  return check_launch(ctx, "mlm_rope_f16");
}

extern "C" int mlm_rope_qk_kv_append(mlm_ctx *ctx, const float *q, const float *k,
                                     const float *v, const float *freqs,
                                     const mlm_rope_args *args, int n_q_heads, int n_kv_heads,
                                     int head_dim, void *q_out, void *k_cache, void *v_cache,
                                     int pos) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, q && k && v && args && q_out && k_cache && v_cache, MLM_ERR_ARG,
              "mlm_rope_qk_kv_append: null argument");
  MLM_REQUIRE(ctx, !args->has_freq_factors || freqs, MLM_ERR_ARG,
              "mlm_rope_qk_kv_append: has_freq_factors set without a freqs buffer");
  MLM_REQUIRE(ctx, n_q_heads > 0 && n_kv_heads > 0 && head_dim > 0 && head_dim % 2 == 0 &&
                       pos >= 0,
              MLM_ERR_SHAPE, "mlm_rope_qk_kv_append: heads=%d/%d d=%d pos=%d", n_q_heads,
              n_kv_heads, head_dim, pos);
  return rope_qk_kv_launch(ctx, q, k, v, freqs, *args, n_q_heads, n_kv_heads, head_dim, q_out,
                           k_cache, v_cache, pos, ctx->stream, nullptr);
}

extern "C" int mlm_silu_mul(mlm_ctx *ctx, const float *gate, const float *up, void *out, int n) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, gate && up && out, MLM_ERR_ARG, "mlm_silu_mul: null buffer");
  MLM_REQUIRE(ctx, n > 0, MLM_ERR_SHAPE, "mlm_silu_mul: n=%d", n);
  return silu_mul_launch(ctx, gate, up, out, n, ctx->stream);
}

extern "C" int mlm_silu_mul_scaled(mlm_ctx *ctx, const float *gate, const float *up,
                                   void *out_f16, float *scale, int n) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, gate && up && out_f16 && scale, MLM_ERR_ARG, "mlm_silu_mul_scaled: null buffer");
  MLM_REQUIRE(ctx, n > 0 && n % 32 == 0, MLM_ERR_SHAPE,
              "mlm_silu_mul_scaled: n=%d is not a positive multiple of 32", n);
  return silu_mul_scaled_launch(ctx, gate, up, out_f16, scale, n, ctx->stream);
}

extern "C" int mlm_add_f32(mlm_ctx *ctx, const float *a, const float *b, float *out, int n) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, a && b && out, MLM_ERR_ARG, "mlm_add_f32: null buffer");
  MLM_REQUIRE(ctx, n > 0, MLM_ERR_SHAPE, "mlm_add_f32: n=%d", n);
  add_f32_kernel<<<(n + 255) / 256, 256, 0, ctx->stream>>>(a, b, out, n);
  return check_launch(ctx, "mlm_add_f32");
}
